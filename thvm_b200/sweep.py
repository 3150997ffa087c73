"""The standalone contraction sweep on the sm_100a device.

    python -m thvm_b200.sweep [--iters N] [--only matvec|gemm|prefill|skinny|skinny_ds]

Seeded N(0,1) inputs, fp32 accumulate:
  * decode matvec x[1, 4096] against W (11008 x 4096) in bf16, and in fp8 e4m3
    with one f32 scale per 128 x 128 block (scales uniform in [0.5, 2]);
  * bf16 GEMM C[M, N] = A[M, K] B[N, K]^T at M=N=K=4096 and M=8192, N=K=4096
    (when the tcgen05 GEMM is built into the library);
  * the skinny bf16 GEMM of batched decode at the GPT-2-XL projection shapes
    (batch 16);
  * causal attention prefill: bf16 Q, K, V [4, 16, 2048,
    128] N(0,1), f32 O, with P split into bf16 hi + lo (the parity setting)
    and as a single bf16 P; FLOPs counted as 2 B H S^2 D (the causal half of
    the two S x S x D products).
The launches of a case are captured into one CUDA graph and replayed between
one pair of CUDA events on the library's stream, rotating over operand copies
that together exceed twice L2 (every launch reads cold operands); one JSON
line per case with the roofline fraction against MEASURED_PEAKS.json.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import numpy as np

from . import _lib as L
from .device import Device
from .gpt2 import make_op

ROOT = Path(__file__).resolve().parents[1]


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bits, round to nearest even (the storage format)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def fp8_codes(a: np.ndarray) -> np.ndarray:
    """f32 -> e4m3 codes for |a| < 448 (finite draws of N(0,1)): round to nearest even."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()


class Timer:
    """The launches captured once into a CUDA graph (the library's TinyJit
    graph slots) and replayed between one pair of CUDA events on the
    library's stream, so host dispatch cost is outside the measurement.
    Callers rotate over operand copies whose total is larger than L2, so
    every launch reads operands the previous launches evicted."""

    def __init__(self, dev: Device):
        import torch
        self.torch = torch
        self.dev = dev
        self.stream = torch.cuda.ExternalStream(dev.stream)

    def time(self, launches, iters: int) -> float:
        """Mean ms per launch over iters launches (launches[i % len] each)."""
        torch, dev = self.torch, self.dev
        slot = dev.new_graph_slot()
        dev.capture_begin(slot)
        try:
            for i in range(iters):
                launches[i % len(launches)]()
        finally:
            dev.capture_end(slot)
        for _ in range(2):
            dev.replay(slot)
        dev.sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        dev.replay(slot)
        e1.record(self.stream)
        e1.synchronize()
        dev.drop(slot)
        return e0.elapsed_time(e1) / iters


def copies_for(nbytes: int, l2: int = 126 << 20) -> int:
    """Operand copies so that the rotation covers more than twice L2."""
    return max(2, -(-2 * l2 // max(nbytes, 1)))


def matvec_cases(dev: Device, timer: Timer, iters: int):
    hbm, _, kind = peaks()
    rng = np.random.default_rng(0)
    M, K, N = 1, 4096, 11008
    x = rng.standard_normal((M, K)).astype(np.float32)
    x = (bf16_bits(x).astype(np.uint32) << 16).view(np.float32)
    y = dev.alloc(M * N * 4)
    xb = dev.upload(x)
    out = []
    for name in ("bf16", "fp8e4m3_bs128"):
        w = rng.standard_normal((N, K)).astype(np.float32)
        if name == "bf16":
            host, dt, wbytes, sc = bf16_bits(w), L.DT_BF16, N * K * 2, None
        else:
            sc = rng.uniform(0.5, 2.0, ((N + 127) // 128, (K + 127) // 128)).astype(np.float32)
            host, dt, wbytes = fp8_codes(w), L.DT_FP8E4M3, N * K + sc.nbytes
        ops, bufs = [], []
        for _ in range(copies_for(wbytes)):
            wb = dev.upload(host)
            slots = {} if sc is None else {6: dev.upload(sc)}
            bufs += [wb] + list(slots.values())
            op = make_op(L.K_LINEAR, y, {0: xb, 1: wb, **slots}, m=M, n=N, k=K)
            op.kernel.dtype = dt
            ops.append(op)
        ms = timer.time([lambda o=o: dev.dispatch(o.kernel, o.in_ids, o.out_id) for o in ops], iters)
        byts = wbytes + x.nbytes + M * N * 4
        gbs = byts / (ms / 1e3) / 1e9
        out.append({"case": f"matvec_{name}", "M": M, "N": N, "K": K, "kernel": "gemv_kernel",
                    "us": round(ms * 1e3, 2), "bytes": byts, "achieved": round(gbs, 1), "unit": "GB/s",
                    "peak": hbm, "frac": round(gbs / hbm, 4), "peak_source": kind,
                    "l2": f"{len(ops)} weight copies rotated (> 2x L2)"})
        for bid in bufs:
            dev.free(bid)
    return out


def gemm_cases(dev: Device, timer: Timer, iters: int):
    lib = dev.lib
    if not hasattr(lib, "sm100_gemm_bf16"):
        return []
    _, tflops, kind = peaks()
    rng = np.random.default_rng(1)
    out = []
    for (M, N, K) in ((4096, 4096, 4096), (8192, 4096, 4096)):
        ha = bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
        hb = bf16_bits(rng.standard_normal((N, K)).astype(np.float32))
        c = dev.alloc(M * N * 4)
        sets = [(dev.upload(ha), dev.upload(hb)) for _ in range(copies_for(ha.nbytes + hb.nbytes))]
        pc = dev.dptr(c)

        def mk(a, b):
            pa, pb = dev.dptr(a), dev.dptr(b)
            return lambda: L.check(lib.sm100_gemm_bf16(pa, pb, pc, M, N, K, dev.stream), "gemm_bf16")
        ms = timer.time([mk(a, b) for a, b in sets], iters)
        tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
        out.append({"case": "gemm_bf16", "M": M, "N": N, "K": K, "kernel": "gemm_bf16_kernel",
                    "us": round(ms * 1e3, 2), "flops": 2 * M * N * K, "achieved": round(tf, 1),
                    "unit": "TFLOP/s", "peak": tflops, "frac": round(tf / tflops, 4), "peak_source": kind})
        for a, b in sets:
            dev.free(a)
            dev.free(b)
        dev.free(c)
    return out


def prefill_cases(dev: Device, timer: Timer, iters: int):
    lib = dev.lib
    _, tflops, kind = peaks()
    rng = np.random.default_rng(4)
    B, H, S, D = 4, 16, 2048, 128
    host = [bf16_bits(rng.standard_normal((B, H, S, D)).astype(np.float32)) for _ in range(3)]
    o = dev.alloc(B * H * S * D * 4)
    po = dev.dptr(o)
    sets = [[dev.upload(h) for h in host] for _ in range(copies_for(sum(h.nbytes for h in host)))]
    out = []
    for precise in (1, 0):
        def mk(ids):
            pq, pk, pv = (dev.dptr(i) for i in ids)
            return lambda: L.check(lib.sm100_attn_prefill_bf16(pq, pk, pv, po, B, H, S, D, 1.0 / np.sqrt(D),
                                                               precise, dev.stream), "attn_prefill")
        ms = timer.time([mk(ids) for ids in sets], iters)
        assert lib.sm100_attn_prefill_status() == 0
        flops = 2 * B * H * S * S * D
        tf = flops / (ms / 1e3) / 1e12
        out.append({"case": "attn_prefill_causal", "B": B, "H": H, "S": S, "D": D,
                    "p": "bf16 hi+lo" if precise else "bf16", "kernel": "attn_prefill_kernel",
                    "us": round(ms * 1e3, 2), "flops": flops, "achieved": round(tf, 1), "unit": "TFLOP/s",
                    "peak": tflops, "frac": round(tf / tflops, 4), "peak_source": kind,
                    "l2": f"{len(sets)} q/k/v copies rotated"})
    for ids in sets:
        for i in ids:
            dev.free(i)
    dev.free(o)
    return out


XL_SHAPES = (("c_attn", 4800, 1600), ("attn.c_proj", 1600, 1600), ("c_fc", 6400, 1600),
             ("mlp.c_proj", 1600, 6400), ("lm_head", 50257, 1600))
# DeepSeek-V2-Lite-shaped projections of BASELINE config 5 (batch 32)
DS_SHAPES = (("ds_qkva", 3648, 2048), ("ds_w_o", 2048, 2048), ("ds_router", 64, 2048),
             ("ds_dense_gu", 21888, 2048), ("ds_dense_down", 2048, 10944), ("ds_lm_head", 102400, 2048))


def skinny_cases(dev: Device, timer: Timer, iters: int, M: int = 16, shapes=XL_SHAPES):
    """Skinny bf16 GEMM launches (bf16 weights streamed once per launch;
    HBM-bound): the GPT-2-XL projections of BASELINE config 3 at batch 16, or
    the given shapes at batch M."""
    import ctypes
    lib = dev.lib
    hbm, _, kind = peaks()
    rng = np.random.default_rng(5)
    out = []
    for name, N, K in shapes:
        x = bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
        w = bf16_bits((0.02 * rng.standard_normal((N, K))).astype(np.float32))
        xb, y = dev.upload(x), dev.alloc(M * N * 4)
        ws, cnt = dev.alloc(lib.sm100_skinny_ws_bytes(M)), dev.alloc(((N + 127) // 128) * 4)
        lib.sm100_buf_zero(cnt)
        ws_ = [dev.upload(w) for _ in range(copies_for(w.nbytes))]
        args = []
        for wb in ws_:
            a = L.Sm100SkinnyArgs()
            a.x, a.w, a.y, a.ws, a.counters = dev.dptr(xb), dev.dptr(wb), dev.dptr(y), dev.dptr(ws), dev.dptr(cnt)
            a.M, a.N, a.K = M, N, K
            args.append(a)
        ms = timer.time([lambda a=a: L.check(lib.sm100_skinny_bf16(ctypes.byref(a), dev.stream), "skinny")
                         for a in args], iters)
        assert lib.sm100_skinny_status() == 0
        byts = w.nbytes + x.nbytes + M * N * 4
        gbs = byts / (ms / 1e3) / 1e9
        out.append({"case": f"skinny_{name}", "M": M, "N": N, "K": K, "kernel": "skinny_kernel",
                    "us": round(ms * 1e3, 2), "bytes": byts, "achieved": round(gbs, 1), "unit": "GB/s",
                    "peak": hbm, "frac": round(gbs / hbm, 4), "peak_source": kind,
                    "l2": f"{len(ws_)} weight copies rotated (> 2x L2)"})
        for bid in ws_ + [xb, y, ws, cnt]:
            dev.free(bid)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", choices=["matvec", "gemm", "prefill", "skinny", "skinny_ds"], default=None)
    args = ap.parse_args()
    dev = Device.get()
    timer = Timer(dev)
    rows = []
    if args.only in (None, "matvec"):
        rows += matvec_cases(dev, timer, args.iters)
    if args.only in (None, "gemm"):
        rows += gemm_cases(dev, timer, args.iters)
    if args.only in (None, "skinny"):
        rows += skinny_cases(dev, timer, args.iters)
    if args.only in (None, "skinny_ds"):
        rows += skinny_cases(dev, timer, args.iters, 32, DS_SHAPES)
        rows += skinny_cases(dev, timer, args.iters, 16, DS_SHAPES[:2])
    if args.only in (None, "prefill"):
        rows += prefill_cases(dev, timer, args.iters)
    for r in rows:
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
