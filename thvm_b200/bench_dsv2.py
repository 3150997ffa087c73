"""batched greedy decode of a DeepSeek-V2-Lite-shaped MoE
decoder (27 layers, d 2048, MLA 16 heads, 64 routed fp8 experts top-6 + 2
shared, vocab 102400, batch 32, prompts of 64 ids, 128 decode steps),
expert-parallel over the GPUs of one box.

    python -m thvm_b200.bench_dsv2 [--steps 128] [--warmup 3] [--layers 27]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m thvm_b200.bench_dsv2 --steps 128

Weights are random-init (bf16 N(0, 0.02); fp8 expert codes of N(0, 1) draws
with block scales U[0.5, 2] * 0.02) drawn on the device from a seeded torch
generator, each rank keeping its experts.  Each step is one CUDA-graph
replay; the prompt fills the cache by teacher-forced steps, then K decode
steps are timed with CUDA events between barriers (max over ranks).  One
JSON line: tokens/s over the whole job (batch x steps / time; the ranks share
one batch: strong scaling) and the HBM roofline of a step: the non-expert
weights, the shared experts, the routed experts a step is expected to touch
(64 (1 - (58/64)^32) = 61.3 distinct per layer for uniform routing) and the
compressed KV rows, against N x the measured copy bandwidth.
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path

import numpy as np

from .dsv2 import DSV2_LITE, DSConfig, DSModel, ep_shard

ROOT = Path(__file__).resolve().parents[1]


def device_weights(cfg: DSConfig, sh, seed: int = 0) -> dict:
    import torch
    g = torch.Generator(device="cuda")
    dev = torch.device("cuda", torch.cuda.current_device())
    counter = [seed * 100003]
    D, H, KV, DN, DR, DV = cfg.dim, cfg.heads, cfg.kv_lora, cfg.d_nope, cfg.d_rope, cfg.d_v
    E, I, DI = cfg.n_exp, cfg.moe_inter, cfg.dense_inter
    keep = list(range(sh.e0, sh.e1)) + [E + k for k in sh.shared]

    def gen():
        counter[0] += 1
        g.manual_seed(counter[0])
        return g

    def mat(*shape):
        return (torch.randn(*shape, generator=gen(), device=dev) * 0.02).to(torch.bfloat16).view(torch.int16)

    def fp8(n, rows, cols):
        codes = torch.empty(n, rows, cols, dtype=torch.uint8, device=dev)
        for i in range(n):
            codes[i] = torch.randn(rows, cols, generator=gen(), device=dev).to(torch.float8_e4m3fn).view(torch.uint8)
        sc = torch.rand(n, -(-rows // 128), -(-cols // 128), generator=gen(), device=dev) * 1.5 + 0.5
        return codes, (sc * 0.02).contiguous()

    w = {"embed": mat(cfg.vocab, D), "lm_head": mat(cfg.vocab, D), "norm_f": torch.ones(D, device=dev)}
    for l in range(cfg.n_layers):
        p = f"l{l}."
        w[p + "attn_norm"], w[p + "ffn_norm"] = torch.ones(D, device=dev), torch.ones(D, device=dev)
        w[p + "kv_norm"] = torch.ones(KV, device=dev)
        w[p + "w_qkva"] = mat(cfg.n_qkva, D)
        w[p + "w_uk"], w[p + "w_uv"], w[p + "w_o"] = mat(H, DN, KV), mat(H, DV, KV), mat(D, H * DV)
        if l < cfg.n_dense:
            w[p + "d_gu"], w[p + "d_down"] = mat(2 * DI, D), mat(D, DI)
        else:
            w[p + "router"] = mat(E, D)
            w[p + "e_gu"], w[p + "e_gu_s"] = fp8(len(keep), 2 * I, D)
            w[p + "e_d"], w[p + "e_d_s"] = fp8(len(keep), D, I)
    return w


def step_bytes(cfg: DSConfig, pos: int) -> int:
    D, H, KV, DN, DR, DV = cfg.dim, cfg.heads, cfg.kv_lora, cfg.d_nope, cfg.d_rope, cfg.d_v
    E, I, DI, B = cfg.n_exp, cfg.moe_inter, cfg.dense_inter, cfg.batch
    attn = (cfg.n_qkva * D + H * DN * KV + H * DV * KV + D * H * DV) * 2
    expert = 3 * I * D + (2 * (-(-2 * I // 128)) * (D // 128)) * 4   # fp8 codes + scales (gate|up, down)
    distinct = E * (1.0 - ((E - cfg.top_k) / E) ** B)
    moe_layers = cfg.n_layers - cfg.n_dense
    total = cfg.n_layers * attn + cfg.n_dense * 3 * DI * D * 2
    total += moe_layers * (E * D * 2 + distinct * expert + cfg.n_shared * expert)
    total += cfg.vocab * D * 2   # lm_head (the embedding reads only B rows)
    total += cfg.n_layers * B * (pos + 1) * (KV + DR) * 2
    return int(total)


def main():
    import torch
    import torch.distributed as dist
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--prompt", type=int, default=64)
    ap.add_argument("--layers", type=int, default=DSV2_LITE.n_layers)
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
    cfg = DSConfig(n_layers=args.layers)
    assert args.prompt + args.warmup + args.steps <= cfg.max_ctx
    sh = ep_shard(cfg, rank, world)
    model = DSModel(cfg, {}, sh, group)
    model.w = device_weights(cfg, sh)
    prompts = torch.from_numpy(np.random.default_rng(1).integers(0, cfg.vocab, (cfg.batch, args.prompt))
                               .astype(np.int32)).cuda()
    if world > 1:
        t = torch.zeros(1, device="cuda")
        dist.all_reduce(t)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        model.step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    model.pos.zero_()
    n0 = model.launches
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        model.step()
    per_step = model.launches - n0
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
            "metric": "decode tok/s (DeepSeek-V2-Lite-shaped MoE fp8 b32, expert-parallel)", "value": round(toks, 1),
            "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "strong",
            "dtype": "fp8 experts / bf16", "data": "synthetic",
            "config": {"workload": "config 5: DSV2-Lite-shaped MoE decode", "layers": cfg.n_layers,
                       "batch": cfg.batch, "prompt": args.prompt, "positions": [pos0, pos0 + args.steps - 1],
                       "parallelism": f"ep{world}"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": round(hbm * world, 1),
                         "unit": "GB/s", "frac": round(achieved / (hbm * world), 4), "traffic": None,
                         "peak_source": "measured" if peaks else "fallback",
                         "bytes_per_step": byts // args.steps},
            "gpu_launches_per_step": per_step,
        }), flush=True)
    del graph
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
