"""batched bf16 greedy decode of a GPT-2-XL-shaped model
(48 layers, d 1600, 25 heads x 64, MLP 6400, vocab 50257, batch 16, prompts
of 128 ids, 256 decode steps, KV cache 1024), tensor-parallel over the GPUs
of one box.

    python -m thvm_b200.bench_xl [--steps 256] [--warmup 3] [--layers 48]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m thvm_b200.bench_xl --steps 256

Weights are random-init N(0, 0.02) bf16 (biases f32, LayerNorm 1 / 0) drawn
on the device from a seeded torch generator, each rank keeping its shard.
Each step is one CUDA-graph replay (all kernels and the NCCL collectives of
the step); the prompt fills the cache by teacher-forced steps first, then K
decode steps are timed with CUDA events between barriers (max over ranks).
One JSON line: tokens/s over the whole job (batch x steps / time; every rank
decodes the same 16 sequences, so N GPUs share one job: strong scaling), and
the HBM roofline of the step: the weights (3.112 GB) and the KV rows the
step reads, over the time, against N x the measured copy bandwidth.
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path

import numpy as np

from .gpt2_xl import GPT2_XL, HEAD_DIM, XLConfig, XLModel, shard_of, split_even

ROOT = Path(__file__).resolve().parents[1]


def device_weights(cfg: XLConfig, sh, seed: int = 0) -> dict:
    """This rank's shard of synthetic weights, generated on the device."""
    import torch
    g = torch.Generator(device="cuda")
    dev = torch.device("cuda", torch.cuda.current_device())
    D, F, V = cfg.dim, cfg.hidden, cfg.vocab
    c = slice(sh.h0 * HEAD_DIM, sh.h1 * HEAD_DIM)
    f = slice(sh.f0, sh.f1)
    counter = [seed * 100003]

    def randn(*shape):
        counter[0] += 1
        g.manual_seed(counter[0])
        return torch.randn(*shape, generator=g, device=dev) * 0.02

    def bf(t):
        return t.to(torch.bfloat16).contiguous().view(torch.int16)

    w = {"wte": bf(randn(V, D)), "wpe": bf(randn(cfg.max_ctx, D))}
    for i in range(cfg.n_layers):
        p = f"h.{i}."
        wa, ba = randn(3 * D, D), randn(3 * D)
        w[p + "attn.w"] = bf(torch.cat([wa[c], wa[D:][c], wa[2 * D:][c]]))
        w[p + "attn.b"] = torch.cat([ba[c], ba[D:][c], ba[2 * D:][c]]).contiguous()
        w[p + "proj.w"], w[p + "proj.b"] = bf(randn(D, D)[:, c]), randn(D)
        w[p + "fc.w"], w[p + "fc.b"] = bf(randn(F, D)[f]), randn(F)[f].contiguous()
        w[p + "p2.w"], w[p + "p2.b"] = bf(randn(D, F)[:, f]), randn(D)
        for k in ("ln_1", "ln_2"):
            w[p + k + ".w"], w[p + k + ".b"] = torch.ones(D, device=dev), torch.zeros(D, device=dev)
    w["ln_f.w"], w["ln_f.b"] = torch.ones(D, device=dev), torch.zeros(D, device=dev)
    w["lm_head"] = bf(randn(V, D)[sh.v0:sh.v1])
    return w


def step_bytes(cfg: XLConfig, pos: int) -> int:
    """Algorithmic HBM bytes of one step over the whole job: every weight
    once (bf16) and the K and V rows 0..pos of every layer (bf16)."""
    D, F, V = cfg.dim, cfg.hidden, cfg.vocab
    per_layer = (3 * D * D + D * D + F * D + D * F) * 2 + (3 * D + D + F + D) * 4
    weights = cfg.n_layers * per_layer + V * D * 2
    kv = cfg.n_layers * 2 * cfg.batch * (pos + 1) * D * 2
    return weights + kv


def main():
    import torch
    import torch.distributed as dist
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--layers", type=int, default=GPT2_XL.n_layers)
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        group = dist.group.WORLD
    cfg = XLConfig(n_layers=args.layers)
    assert args.prompt + args.warmup + args.steps <= cfg.max_ctx
    sh = shard_of(cfg, rank, world)
    model = XLModel.__new__(XLModel)
    # the weights come from the device generator (no host copy of 3 GB)
    XLModel.__init__(model, cfg, {}, sh, group)
    model.w = device_weights(cfg, sh)
    prompts = torch.from_numpy(np.random.default_rng(1).integers(0, cfg.vocab, (cfg.batch, args.prompt))
                               .astype(np.int32)).cuda()
    if world > 1:   # a collective before capture
        t = torch.zeros(1, device="cuda")
        dist.all_reduce(t)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        model.step()   # warm: tensor maps, function attributes
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    model.pos.zero_()
    n0 = model.launches
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        model.step()
    per_step = model.launches - n0
    # prompt: teacher-forced steps fill the cache
    for t in range(args.prompt):
        model.tok.copy_(prompts[:, t])
        graph.replay()
    for _ in range(args.warmup):
        graph.replay()
    pos0 = args.prompt + args.warmup
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    e1.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    toks = cfg.batch * args.steps / (ms / 1e3)
    byts = sum(step_bytes(cfg, pos0 + i) for i in range(args.steps))
    achieved = byts / (ms / 1e3) / 1e9
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    if rank == 0:
        print(json.dumps({
            "metric": "decode tok/s (GPT-2 XL bf16 b16, tensor-parallel)", "value": round(toks, 1), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 3: GPT-2 XL-shaped bf16 decode", "layers": cfg.n_layers,
                       "batch": cfg.batch, "prompt": args.prompt, "positions": [pos0, pos0 + args.steps - 1],
                       "parallelism": f"tp{world}"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": round(hbm * world, 1),
                         "unit": "GB/s", "frac": round(achieved / (hbm * world), 4),
                         "traffic": None, "peak_source": "measured" if peaks else "fallback",
                         "bytes_per_step": byts // args.steps},
            "gpu_launches_per_step": per_step,
        }), flush=True)
    del graph
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
