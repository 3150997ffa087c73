"""BASELINE config 4 over the GPUs of one box: causal attention prefill, bf16,
batch 4, 16 heads, head_dim 128, seq_len 2048, with the (batch, head) pairs
split across ranks.

    python -m thvm_b200.bench_prefill [--steps 20] [--warmup 3] [--fast-p]
    python -m torch.distributed.run --nnodes 1 --nproc-per-node N --master-addr 127.0.0.1 \\
        -m thvm_b200.bench_prefill

The pairs are independent (scaled_dot_product_attention.c computes every
(b, h) on its own), so rank r takes a contiguous share of the B x H pairs of
the [B, H, S, D] tensors and no collective touches the data path: strong
scaling of one fixed prefill.  Q, K, V are N(0, 1) draws from a seeded torch
generator; several input copies rotate so that one step's inputs are not in
L2 from the step before.  Each step is one launch of the fused kernel over
the rank's pairs, timed with CUDA events between barriers, max over ranks.
One JSON line: TFLOP/s of the whole job (2 B H S^2 D per step) and the
tensor roofline against N x the measured bf16 peak.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
B, H, S, D = 4, 16, 2048, 128
L2_BYTES = 126 * 1024 * 1024


def pair_range(n_pairs: int, rank: int, world: int) -> tuple[int, int]:
    """The contiguous (batch, head) pairs [p0, p1) of a rank: an even split."""
    return n_pairs * rank // world, n_pairs * (rank + 1) // world


def main():
    import torch
    import torch.distributed as dist
    from . import _lib as L
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--fast-p", action="store_true", help="single bf16 P (the 2e-2 path) instead of hi + lo")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    lib = L.lib()
    L.check(lib.sm100_init(), "init")
    p0, p1 = pair_range(B * H, rank, world)
    n = p1 - p0
    g = torch.Generator(device="cuda")
    g.manual_seed(1000 + rank)
    per_copy = 3 * n * S * D * 2
    copies = max(1, -(-2 * L2_BYTES // max(per_copy, 1)))
    sets = [[torch.randn(n, S, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3)]
            for _ in range(copies)]
    o = torch.empty(n, S, D, dtype=torch.float32, device="cuda")
    scale = 1.0 / D ** 0.5
    precise = 0 if args.fast_p else 1

    def launch(i):
        q, k, v = sets[i % copies]
        L.check(lib.sm100_attn_prefill_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), 1, n, S, D,
                                            scale, precise, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
                "attn_prefill")

    for i in range(args.warmup):
        launch(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        launch(i)
    e1.record()
    e1.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    assert lib.sm100_attn_prefill_status() == 0, "prefill kernel status"
    flops = 2 * B * H * S * S * D
    tf = flops * args.steps / (ms / 1e3) / 1e12
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    if rank == 0:
        print(json.dumps({
            "metric": "causal prefill TFLOP/s (B4 H16 S2048 D128 bf16)", "value": round(tf, 1), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 4: causal attention prefill", "B": B, "H": H, "S": S, "D": D,
                       "p": "bf16 hi+lo" if precise else "bf16", "pairs_per_rank": n, "parallelism": f"bh{world}",
                       "l2": f"{copies} input copies rotated per rank (> 2x L2)"},
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": round(peak * world, 1),
                         "unit": "TFLOP/s", "frac": round(tf / (peak * world), 4),
                         "peak_source": "measured" if peaks else "fallback"},
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
