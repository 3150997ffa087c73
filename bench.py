"""Decode throughput of GPT-2 small (fp32, batch 1) on the sm_100a device.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Workload: GPT-2 small, seeded random weights, a 16-id
prompt, 64 greedy decode tokens through the KV cache with the TinyJit replay
as a CUDA graph.  A "step" is one full 64-token generation (positions 16..79)
replayed from one captured graph; `value` is whole-job tokens/s.  N > 1 runs N
independent replicas (the model does not shard: one process per GPU, no
data-path collective), so scaling is weak.

Also reported: `e2e` (the same 64 tokens per step through the C-ABI with the
token and position written from pinned host memory and the next id read back
every token), `roofline` (the fused decode kernel: algorithmic bytes of its
64-token launch over the event-timed launch, against the measured HBM copy
bandwidth; `traffic` from the committed ncu summary), `cpu_baseline` (the CPU
oracle port on
the host cores), the SM clocks sampled during the timed region, and the
kernel launch count.  `--impl reference` times the CPU path instead.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_PROMPT, N_NEW = 16, 64
METRIC = "GPT-2 124M b1 fp32 decode tok/s"


def _env_int(name, default):
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during timing."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.out = ROOT / "gpurun_out" / f"clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.out.parent.mkdir(exist_ok=True)
            self.f = open(self.out, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if not self.proc or not self.out.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.read_text().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def _ncu_traffic(kernel):
    """DRAM bytes (read + write) of one launch of `kernel` from its committed
    ncu summary (a `traffic_bytes_per_launch:` line in profiles/<kernel>_*.md),
    or None when no capture of the current kernel is committed."""
    for p in sorted((ROOT / "profiles").glob(f"{kernel}_*.md")):
        for line in p.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                try:
                    return int(line.split(":", 1)[1].strip())
                except ValueError:
                    return None
    return None


def linear_bytes(cfg, T=1):
    """Algorithmic bytes of the decode step's linear launches: every weight,
    bias and LayerNorm parameter once, the x rows read, the outputs written
    (and the residual read) in float32."""
    d, h, V = cfg.dim, cfg.hidden, cfg.vocab
    per_layer = 0
    for (n, k, ln, res) in ((3 * d, d, True, False), (d, d, False, True), (h, d, True, False), (d, h, False, True)):
        per_layer += 4 * (n * k + n + T * k + T * n + (2 * k if ln else 0) + (T * n if res else 0))
    head = 4 * (V * d + d + V + 2 * d)
    return cfg.n_layers * per_layer + head, cfg.n_layers * 4 + 1


def weight_params(cfg):
    """Parameters one decode token reads: every block (c_attn 3d x d, c_proj
    d x d, c_fc h x d, mlp.c_proj d x h, their biases, two LayerNorms), ln_f
    and lm_head; the embeddings contribute one row each (counted per token)."""
    d, h = cfg.dim, cfg.hidden
    block = 3 * d * d + d * d + h * d + d * h + (3 * d + d + h + d) + 4 * d
    return cfg.n_layers * block + 2 * d + cfg.vocab * d


def tokens_bytes(cfg, pos0, n):
    """Algorithmic HBM bytes of n decode tokens at positions pos0..pos0+n-1:
    per token all weights once, the wte and wpe rows, the keys and values of
    the earlier positions (pos rows per layer) and the new row written."""
    d = cfg.dim
    per_tok = 4 * weight_params(cfg) + 2 * 4 * d + cfg.n_layers * 2 * 4 * d
    kv_rows = sum(range(pos0, pos0 + n))
    return n * per_tok + cfg.n_layers * 2 * 4 * d * kv_rows


def cpu_baseline(cfg, weights, prompt, seconds=15.0):
    """The CPU oracle port (oracle/oracle.c, pthreads over all cores): the
    prompt forward, then greedy tokens until ~`seconds` of decode work."""
    import oracle as O
    m = O.GPT2(cfg, weights)
    tok = m.forward(prompt, 0)
    pos, n, t0 = len(prompt), 0, time.perf_counter()
    while n < N_NEW and time.perf_counter() - t0 < seconds:
        tok = m.forward([tok], pos)
        pos += 1
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 3), "unit": "tok/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"{n} greedy decode tokens after the 16-id prompt (positions 16..{15 + n}), full model"}


def run_reference(args, rank, world):
    """--impl reference: the CPU path of the decode on the host cores."""
    if rank != 0:
        return
    from thvm_b200.synthetic import GPT2_SMALL, gpt2_weights, prompt_tokens
    cfg = GPT2_SMALL
    weights = gpt2_weights(cfg, seed=0)
    prompt = prompt_tokens(N_PROMPT, cfg.vocab, seed=1)
    import oracle as O
    m = O.GPT2(cfg, weights)
    tok = m.forward(prompt, 0)
    pos = N_PROMPT
    per_step = 4   # tokens per timed step: a bounded sample of the 64-token decode
    for _ in range(args.warmup):
        tok = m.forward([tok], pos)
        pos += 1
    t0 = time.perf_counter()
    n = 0
    for _ in range(args.steps):
        for _ in range(per_step):
            if pos >= N_PROMPT + N_NEW:
                tok, pos = m.forward(prompt, 0), N_PROMPT
            tok = m.forward([tok], pos)
            pos += 1
            n += 1
    dt = time.perf_counter() - t0
    v = n / dt
    line = {"metric": METRIC, "value": round(v, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "gpt2-small decode, b1, 16-id prompt, greedy tokens at positions 16..79",
                       "tokens_per_step": per_step},
            "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": O.num_threads(), "kind": "port",
                             "sample": f"{per_step} decode tokens per step, full model"},
            "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="sm100", choices=["sm100", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    rank, world, local = _env_int("RANK", 0), _env_int("WORLD_SIZE", 1), _env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    args.warmup = max(args.warmup, 3)

    import torch
    torch.cuda.set_device(local)
    os.environ["THVM_SM100_DEVICE"] = str(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))

    from thvm_b200.device import Device
    from thvm_b200.gpt2 import Transformer
    from thvm_b200.synthetic import GPT2_SMALL, gpt2_weights, prompt_tokens
    cfg = GPT2_SMALL
    weights = gpt2_weights(cfg, seed=0)
    prompt = prompt_tokens(N_PROMPT, cfg.vocab, seed=1)
    dev = Device.get()
    model = Transformer(cfg, weights, dev)
    stream = torch.cuda.ExternalStream(dev.stream)

    first = model.forward(prompt, 0)
    model.capture_run(N_NEW, first, N_PROMPT)
    for _ in range(args.warmup):
        model.replay_run()
    dev.sync()

    def barrier():
        if dist is not None:
            dist.barrier()

    # ---- timed region: K replays of the 64-token generation ---------------
    launches0 = dev.launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        barrier()
        torch.cuda.synchronize()
        dev.sync()
        e0.record(stream)
        for _ in range(args.steps):
            model.replay_run()
        e1.record(stream)
        dev.sync()
        torch.cuda.synchronize()
        barrier()
    launches = dev.launches() - launches0
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    last_tok = model.current_token()
    value = world * N_NEW * args.steps / (ms / 1e3)

    # ---- roofline of the dominant kernel --------------------------------
    hbm, peak_kind = _peaks()
    run_bytes = tokens_bytes(cfg, N_PROMPT, N_NEW)
    step_gbs = run_bytes * args.steps / (ms / 1e3) / 1e9
    if model.fused:
        # the run graph is one decode_kernel launch over the 64 tokens plus
        # two 4-byte copy nodes that reset (token, position): the replay's
        # event-timed duration is the launch's duration (copies included)
        kern_us = ms * 1e3 / args.steps
        ach = run_bytes / (kern_us / 1e6) / 1e9
        roof = {"bound": "hbm", "kernel": "decode_kernel (fused GPT-2 decode, 64 tokens per launch)",
                "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(ach / hbm, 4), "peak_source": peak_kind,
                "bytes_per_launch": run_bytes, "avg_launch_us": round(kern_us, 3),
                "traffic": _ncu_traffic("decode_kernel")}
    else:
        lin_ops = [op for op in model.forward_ops(1, bump=False) if op.kernel.kind == 1]
        dev.write(model.s.io, np.array([N_PROMPT + 32, first], np.int32))
        reps, slot = 20, dev.new_graph_slot()
        dev.capture_begin(slot)
        for op in lin_ops:
            dev.dispatch(op.kernel, op.in_ids, op.out_id)
        dev.capture_end(slot)
        dev.replay(slot)
        dev.sync()
        l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0.record(stream)
        for _ in range(reps):
            dev.replay(slot)
        l1.record(stream)
        dev.sync()
        torch.cuda.synchronize()
        dev.drop(slot)
        lin_ms = l0.elapsed_time(l1) / reps
        lb, nl = linear_bytes(cfg)
        achieved = lb / (lin_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "kernel": "linear_kernel (all 49 projections of one decode step)",
                "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                "peak_source": peak_kind, "bytes_per_launch": round(lb / nl), "launches": nl,
                "avg_launch_us": round(lin_ms * 1e3 / nl, 3), "traffic": None}
    roof["step"] = {"algorithmic_bytes_per_token": round(run_bytes / N_NEW), "achieved_gbs": round(step_gbs, 1),
                    "frac": round(step_gbs / hbm, 4)}
    status = model.decode_status()
    if status:
        raise RuntimeError(f"decode kernel status {status:#x}")

    # ---- e2e through the C-ABI with host buffers -------------------------
    e2e_steps = max(1, min(args.steps, 5))
    model.capture_step()
    io = torch.empty(2, dtype=torch.int32, pin_memory=True)
    out = torch.empty(1, dtype=torch.int32, pin_memory=True)
    L = dev.lib
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        tok = first
        for i in range(N_NEW):
            io[0], io[1] = N_PROMPT + i, tok
            L.sm100_buf_write(model.s.io, io.data_ptr(), 8)
            L.sm100_graph_replay(model.GRAPH_STEP)
            L.sm100_buf_read(model.s.tok, out.data_ptr(), 4)
            tok = int(out[0])
    e2e_s = time.perf_counter() - t0
    if dist is not None:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * N_NEW * e2e_steps / e2e_s

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg, weights, prompt)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "gpt2-small fp32 b1: 16-id prompt, 64 greedy decode tokens (positions 16..79) "
                                   "per step, one CUDA-graph replay per step",
                       "model": "gpt2 124M (12L d768 12x64 MLP3072 vocab 50257 ctx 1024), seeded N(0,0.02)",
                       "global_batch": world, "seq_len": N_PROMPT + N_NEW, "tokens_per_step": N_NEW,
                       "parallelism": f"replicas{world}",
                       "l2": "weights (495 MB) exceed L2 (126 MB): every step streams them from HBM"},
            "ms_per_token": round(ms / args.steps / N_NEW, 5),
            "last_token": last_tok,
            "gpu_launches": int(launches),
            "roofline": roof,
            "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": 8 * N_NEW,
                    "d2h_bytes_per_step": 4 * N_NEW, "steps": e2e_steps},
            "clocks": clk.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
