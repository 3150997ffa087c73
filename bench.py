"""Decode throughput on the sm_100a device, for BASELINE.json's metric.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                    [--workload moe|gpt2|xl|prefill|kernels] [--layers L] [--no-extras]

Default workload (every N): BASELINE config 5, a DeepSeek-V2-Lite-shaped MoE
decoder (27 layers, d 2048, MLA 16 heads, 64 routed fp8-e4m3 experts with
128 x 128 f32 block scales, top-6 + 2 shared, vocab 102400), batch 32, 64
prompt ids per sequence fed one position per step, then greedy decode.  A
"step" is one decode step of the 32 sequences, one CUDA-graph replay;
`value` = 32 x K / the max over ranks of the event-timed K steps.  With N
ranks the model is split (thvm_b200.dsv2): attention heads, the dense
layer's hidden units, the experts and the vocabulary rows, one all-reduce of
the residual stream after each attention block and each MLP / expert block,
so the N GPUs share one batch: scaling is strong.

At N = 1 the same JSON line also carries, under "gpt2_small", BASELINE
config 1 (GPT-2 small fp32 b1, 64 greedy tokens per replay of one fused
decode kernel) with its own roofline, e2e and cpu_baseline, and under
"kernels" the config-2 and config-4 kernel cases (bf16 / fp8 matvec, tcgen05
GEMM, causal prefill) with theirs (--no-extras skips both).

Keys: `roofline` (the dominant kernel, timed live with CUDA events:
algorithmic bytes / duration against MEASURED_PEAKS.json; `traffic` from the
committed ncu summary under profiles/), `e2e` (the same decode with the
token ids copied in from pinned host memory and the next ids read back every
step), `cpu_baseline` (rank 0 at N = 1: the oracle port on the host cores on
a bounded sample), `clocks` (nvidia-smi during the timed region),
`gpu_launches` (this library's kernel launches in the timed region).

`--impl reference` times the reference's own CPU path of the workload: for
config 5 its DeepSeek-V2 decode bench (oracle/_ref/dsv2_decode_bench, built
from the reference's sources) at full width on a bounded sample; for `xl` and
`gpt2` the oracle port of the reference's CPU forward on the host cores, for
`prefill` the oracle port of its causal attention.
The other workloads: `gpt2` (config 1 alone; N > 1 runs N replicas), `xl`
(config 3, tensor-parallel: decode steps and the prompt pass), `prefill`
(config 4, the (batch, head) pairs
split over the ranks), `kernels` (config 2 / 4 kernel cases, one line each).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import tempfile
import time
import zlib
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s (GPT-2 124M b1; MoE fp8 b32 @1/2/4/8 GPU) and % of HBM roofline"
L2_BYTES = 126 << 20


# ============================================================================
# common
# ============================================================================

def _env_int(name, default):
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


def peaks():
    """(HBM GB/s, bf16 dense TFLOP/s burst, source) for the roofline denominators."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class Ctx:
    """Rank, world and the torch.distributed module (None at N = 1)."""

    def __init__(self):
        self.rank, self.world = _env_int("RANK", 0), _env_int("WORLD_SIZE", 1)
        self.local = _env_int("LOCAL_RANK", 0)
        self.dist = None
        self.group = None

    def init_cuda(self):
        import torch
        torch.cuda.set_device(self.local)
        os.environ["THVM_SM100_DEVICE"] = str(self.local)
        if self.world > 1 and self.dist is None:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.dist, self.group = dist, dist.group.WORLD

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()

    def max(self, v: float) -> float:
        if self.dist is None:
            return v
        import torch
        t = torch.tensor([v], device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.dist is not None:
            self.dist.barrier()
            self.dist.destroy_process_group()
            self.dist = None


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during timing
    (written to a temporary file)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.out = Path(tempfile.gettempdir()) / f"thvm_bench_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
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
        try:
            self.out.unlink()
        except OSError:
            pass
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def ncu_traffic(kernel, key="traffic_bytes_per_launch"):
    """DRAM bytes (read + write) of one launch of `kernel` from its committed
    ncu summary (a `traffic_bytes_per_launch:` line in profiles/<kernel>_*.md),
    or None when no capture of the current kernel is committed."""
    for p in sorted((ROOT / "profiles").glob(f"{kernel}_*.md")):
        for line in p.read_text().splitlines():
            if line.startswith(key + ":"):
                try:
                    return int(line.split(":", 1)[1].strip())
                except ValueError:
                    return None
    return None


def base_line(args, world, value, ms, **kw):
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "vs_baseline": None, "data": "synthetic"}
    line.update(kw)
    return line


# ============================================================================
# config 5: DeepSeek-V2-Lite-shaped MoE decode, batch 32
# ============================================================================

N_PROMPT_DS = 64


def ds_device_weights(cfg, sh, seed: int = 0) -> dict:
    """This rank's slices of one seeded model, generated on the device:
    every tensor (and every expert, head and dense-layer slice) has its own
    seed, so any N builds the same model.  bf16 matrices N(0, 0.02); fp8
    expert codes of N(0, 1) draws with block scales U[0.5, 2] * 0.02; norm
    gains 1."""
    import torch
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device="cuda")
    D, H, KV, DN, DR, DV = cfg.dim, cfg.heads, cfg.kv_lora, cfg.d_nope, cfg.d_rope, cfg.d_v
    E, I, DI, QS = cfg.n_exp, cfg.moe_inter, cfg.dense_inter, cfg.d_nope + cfg.d_rope

    def gen(*key):   # a seed per tensor name (crc32: the same in every process)
        g.manual_seed(zlib.crc32(repr((seed,) + key).encode()))
        return g

    def bf(*shape, key):
        return (torch.randn(*shape, generator=gen(*key), device=dev) * 0.02).to(torch.bfloat16).view(torch.int16)

    def fp8(rows, cols, key):
        codes = torch.randn(rows, cols, generator=gen(*key, "c"), device=dev).to(torch.float8_e4m3fn).view(torch.uint8)
        sc = torch.rand(-(-rows // 128), -(-cols // 128), generator=gen(*key, "s"), device=dev) * 1.5 + 0.5
        return codes, sc * 0.02

    keep = list(range(sh.e0, sh.e1)) + [E + k for k in sh.shared]
    w = {"embed": bf(cfg.vocab, D, key=("embed",)), "norm_f": torch.ones(D, device=dev),
         "lm_head": bf(cfg.vocab, D, key=("lm_head",))[sh.v0:sh.v1].contiguous()}
    for l in range(cfg.n_layers):
        p = f"l{l}."
        w[p + "attn_norm"], w[p + "ffn_norm"] = torch.ones(D, device=dev), torch.ones(D, device=dev)
        w[p + "kv_norm"] = torch.ones(KV, device=dev)
        q = [bf(QS, D, key=(l, "q", h)) for h in range(sh.h0, sh.h1)]
        w[p + "w_qkva"] = torch.cat(q + [bf(KV + DR, D, key=(l, "kva"))]).contiguous()
        w[p + "w_uk"] = torch.stack([bf(DN, KV, key=(l, "uk", h)) for h in range(sh.h0, sh.h1)]).contiguous()
        w[p + "w_uv"] = torch.stack([bf(DV, KV, key=(l, "uv", h)) for h in range(sh.h0, sh.h1)]).contiguous()
        w[p + "w_o"] = torch.cat([bf(D, DV, key=(l, "o", h)) for h in range(sh.h0, sh.h1)], 1).contiguous()
        if l < cfg.n_dense:
            gu = bf(2 * DI, D, key=(l, "d_gu"))
            w[p + "d_gu"] = torch.cat([gu[sh.f0:sh.f1], gu[DI + sh.f0:DI + sh.f1]]).contiguous()
            w[p + "d_down"] = bf(D, DI, key=(l, "d_down"))[:, sh.f0:sh.f1].contiguous()
            del gu
        else:
            w[p + "router"] = bf(E, D, key=(l, "router"))
            gu = [fp8(2 * I, D, key=(l, "e_gu", e)) for e in keep]
            dn = [fp8(D, I, key=(l, "e_d", e)) for e in keep]
            w[p + "e_gu"] = torch.stack([c for c, _ in gu]).contiguous()
            w[p + "e_gu_s"] = torch.stack([s for _, s in gu]).contiguous()
            w[p + "e_d"] = torch.stack([c for c, _ in dn]).contiguous()
            w[p + "e_d_s"] = torch.stack([s for _, s in dn]).contiguous()
    return w


def ds_expert_bytes(cfg) -> int:
    """fp8 codes and block scales of one expert (gate | up and down)."""
    D, I = cfg.dim, cfg.moe_inter
    return 3 * I * D + (2 * (-(-2 * I // 128)) * (D // 128)) * 4


def ds_step_bytes(cfg, pos: int) -> int:
    """Algorithmic HBM bytes of one decode step over the whole job: every
    non-expert weight once (bf16; the embedding B rows), the shared experts,
    the routed experts a step is expected to touch (E (1 - ((E - K) / E)^B) =
    61.3 of 64 per layer for uniform routing) and the compressed KV rows
    0..pos of every sequence and layer."""
    D, H, KV, DN, DR, DV = cfg.dim, cfg.heads, cfg.kv_lora, cfg.d_nope, cfg.d_rope, cfg.d_v
    E, DI, B = cfg.n_exp, cfg.dense_inter, cfg.batch
    attn = (cfg.n_qkva * D + H * DN * KV + H * DV * KV + D * H * DV) * 2
    distinct = E * (1.0 - ((E - cfg.top_k) / E) ** B)
    moe_layers = cfg.n_layers - cfg.n_dense
    total = cfg.n_layers * attn + cfg.n_dense * 3 * DI * D * 2
    total += moe_layers * (E * D * 2 + (distinct + cfg.n_shared) * ds_expert_bytes(cfg))
    total += cfg.vocab * D * 2 + B * D * 2
    total += cfg.n_layers * B * (pos + 1) * (KV + DR) * 2
    return int(total)


def moe_cpu_baseline(batch: int):
    """The oracle port (oracle.c orc_ds_step, pthreads over the host cores) on
    a bounded sample of the workload: one decode step of the full-width model
    at batch 32 with 1 layer (the dense layer) and with 2 (dense + one MoE
    layer); the 27-layer step time is t1 + 26 (t2 - t1)."""
    import oracle as O
    from thvm_b200.dsv2 import DSConfig, ds_weights, yarn_tables
    cfg2 = DSConfig(n_layers=2, batch=batch)
    w = ds_weights(cfg2, seed=0)
    cos, sin = yarn_tables(cfg2.d_rope, cfg2.max_ctx)
    tok = np.random.default_rng(1).integers(0, cfg2.vocab, batch).astype(np.int32)
    times = []
    for n in (1, 2):
        cfg = DSConfig(n_layers=n, batch=batch, max_ctx=64)
        layer_of = lambda k: int(k[1:].split(".")[0]) if k[0] == "l" and k[1].isdigit() else -1
        m = O.DSModel(cfg, {k: v for k, v in w.items() if layer_of(k) < n}, cos[:64], sin[:64])
        m.step(tok, 0)
        t0 = time.perf_counter()
        m.step(tok, 1)
        times.append(time.perf_counter() - t0)
    t27 = times[0] + (DSConfig().n_layers - 1) * (times[1] - times[0])
    return {"value": round(batch / t27, 3), "unit": "tok/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"one batch-{batch} decode step of the full-width model with 1 and 2 layers "
                      f"({times[0]:.2f} s, {times[1]:.2f} s); 27-layer step = t1 + 26 (t2 - t1) = {t27:.2f} s"}


def moe_run(args, ctx):
    import torch
    from thvm_b200.dsv2 import DSConfig, DSModel, ds_shard
    ctx.init_cuda()
    cfg = DSConfig(n_layers=args.layers or DSConfig().n_layers)
    B = cfg.batch
    assert N_PROMPT_DS + args.warmup + args.steps + 16 <= cfg.max_ctx, "positions beyond the cache"
    sh = ds_shard(cfg, ctx.rank, ctx.world)
    model = DSModel(cfg, {}, sh, ctx.group)
    model.w = ds_device_weights(cfg, sh)
    lib = model.lib
    prompts = torch.from_numpy(np.random.default_rng(1).integers(0, cfg.vocab, (B, N_PROMPT_DS))
                               .astype(np.int32)).cuda()
    if ctx.world > 1:   # a collective before capture
        t = torch.zeros(1, device="cuda")
        ctx.dist.all_reduce(t)
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
    for t in range(N_PROMPT_DS):   # the prompt: one teacher-forced position per step
        model.tok.copy_(prompts[:, t])
        graph.replay()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if ctx.max(float(model.status())) != 0:
        raise RuntimeError("MoE kernels' status word set during warm-up")
    pos0 = N_PROMPT_DS + args.warmup
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(ctx.local) as clk:
        ctx.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ctx.barrier()
    ms = ctx.max(e0.elapsed_time(e1))
    if ctx.max(float(model.status())) != 0:
        raise RuntimeError("MoE kernels' status word set during the timed steps: the steps did not finish")
    value = B * args.steps / (ms / 1e3)
    hbm, _, peak_kind = peaks()
    byts = sum(ds_step_bytes(cfg, pos0 + i) for i in range(args.steps))
    step_gbs = byts / (ms / 1e3) / 1e9

    # ---- the dominant kernel, timed alone: one MoE layer's expert launch pair
    # (ds_x8_kernel<up> + <down>) on this rank, rotating over the 26 layers'
    # expert weights (13.8 GB at N = 1, far beyond L2) with the slot lists of the
    # last routed layer; output into a scratch buffer
    moe_layers = [l for l in range(cfg.n_layers) if l >= cfg.n_dense]
    roof = None
    if moe_layers:
        off = model.slot_off.cpu().numpy()
        counts = np.diff(off)
        n_local = len(counts)
        y = torch.zeros_like(model.h)
        st = ctypes.c_void_p(stream.cuda_stream)
        w = model.w

        def experts(l):
            p = f"l{l}."
            rc = lib.sm100_ds_experts(model.xn.data_ptr(), w[p + "e_gu"].data_ptr(), w[p + "e_gu_s"].data_ptr(),
                                      w[p + "e_d"].data_ptr(), w[p + "e_d_s"].data_ptr(), model.slot_off.data_ptr(),
                                      model.slot_tok.data_ptr(), model.slot_w.data_ptr(), model.a.data_ptr(),
                                      y.data_ptr(), n_local, cfg.dim, cfg.moe_inter, st)
            if rc != 0:
                raise RuntimeError(f"ds_experts: {rc}")
        reps = 2 * len(moe_layers)
        for l in moe_layers[:3]:
            experts(l)
        torch.cuda.synchronize()
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record(stream)
        for i in range(reps):
            experts(moe_layers[i % len(moe_layers)])
        k1.record(stream)
        torch.cuda.synchronize()
        if model.status() != 0:
            raise RuntimeError("expert kernels' status word set while timing them")
        us = k0.elapsed_time(k1) * 1e3 / reps
        touched = int((counts > 0).sum())
        slots = int(off[-1])
        kb = touched * ds_expert_bytes(cfg) + B * cfg.dim * 2 + 2 * slots * cfg.moe_inter * 2 + 2 * B * cfg.dim * 4
        ach = kb / (us / 1e6) / 1e9
        # the ncu capture's launch pair touched a different set of experts: its
        # DRAM bytes per algorithmic byte, times this launch's algorithmic bytes
        t_ncu, a_ncu = ncu_traffic("ds_x8_kernel"), ncu_traffic("ds_x8_kernel", "algorithmic_bytes_per_launch")
        traffic = round(t_ncu / a_ncu * kb) if t_ncu and a_ncu else None
        roof = {"bound": "hbm", "kernel": "ds_x8_kernel<up> + ds_x8_kernel<down> (one MoE layer's fp8 experts)",
                "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s", "frac": round(ach / hbm, 4),
                "peak_source": peak_kind, "bytes_per_launch": kb, "avg_launch_us": round(us, 2),
                "experts_touched": touched, "experts_local": n_local, "slots": slots,
                "traffic": traffic,
                "traffic_note": "ncu DRAM read + write bytes of one up + down pair (profiles/ds_x8_kernel_moe_config5.md) "
                                "per algorithmic byte, times this pair's algorithmic bytes",
                "step": {"algorithmic_bytes_per_step": byts // args.steps, "achieved_gbs": round(step_gbs, 1),
                         "peak_gbs": round(hbm * ctx.world, 1), "frac": round(step_gbs / (hbm * ctx.world), 4)}}
        del y

    # ---- e2e: ids in from host memory and the next ids back, every step.  One
    # GPU: through the C host (sm100_ds_model_step: the ids copied in, the
    # captured step replayed, the next ids copied out, all inside the call);
    # several: through this rank's captured step with pinned copies
    e2e_steps = max(1, min(args.steps, 10))
    e2e_path = "python host: pinned copies around the captured step"
    if ctx.world == 1:
        from thvm_b200.ds_host import CDSModel
        del graph
        torch.cuda.synchronize()
        cm = CDSModel(cfg, {**model.w, "cos": model.cos, "sin": model.sin})
        pr = prompts.cpu().numpy()
        for t in range(N_PROMPT_DS):
            cm.step(pr[:, t], read=False)
        ids = None
        for _ in range(args.warmup):
            ids = cm.step(ids)
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            ids = cm.step(ids)
        e2e_s = time.perf_counter() - t0
        cm.close()
        if model.status() != 0:
            raise RuntimeError("MoE kernels' status word set in the C host's steps")
        e2e_path = "C host: sm100_ds_model_step (ids host -> device, the captured step, next ids device -> host)"
    else:
        host_in = torch.from_numpy(np.random.default_rng(2).integers(0, cfg.vocab, B).astype(np.int32)).pin_memory()
        host_out = torch.empty(B, dtype=torch.int32).pin_memory()
        ctx.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            model.tok.copy_(host_in, non_blocking=True)
            graph.replay()
            host_out.copy_(model.tok, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            host_in.copy_(host_out)
        e2e_s = ctx.max(time.perf_counter() - t0)
        del graph
    e2e = B * e2e_steps / e2e_s
    launches = per_step * args.steps
    torch.cuda.synchronize()
    line = base_line(
        args, ctx.world, round(value, 1), ms, scaling="strong", dtype="fp8 e4m3 experts, bf16 activations / weights",
        config={"workload": "config 5: DeepSeek-V2-Lite-shaped MoE decode, batch 32, 64 prompt ids then greedy steps",
                "model": f"{cfg.n_layers}L d{cfg.dim} MLA 16x(128+64) kv_lora 512, 64 fp8 experts x 1408 top-6 + 2 "
                         "shared, dense layer 0 (10944), vocab 102400; seeded random weights",
                "global_batch": B, "positions": [pos0, pos0 + args.steps - 1], "tokens_per_step": B,
                "parallelism": f"tp{ctx.world} attention heads / dense units / vocab, ep{ctx.world} experts",
                "l2": "weights (15.7 GB per step) exceed L2 (126 MB): every step streams them from HBM"},
        ms_per_token=round(ms / args.steps / B, 5), gpu_launches=int(launches), gpu_launches_per_step=per_step,
        roofline=roof,
        e2e={"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B,
             "steps": e2e_steps, "path": e2e_path},
        clocks=clk.summary())
    del model
    torch.cuda.empty_cache()
    return line


def spec_run(args, ctx):
    """Blind speculative decode of the config-5 model (thvm_b200.spec.SpecDecoder,
    the reference's DSV2_SPEC step): 8 sequences x S = 4 verify rows (the 32
    rows of the base batch), prompts of 64 ids prefilled 4 positions per pass,
    then W untimed and K timed steps of draft / verify / accept, captured as
    one graph.  value = committed tokens / s over the timed steps; with forced
    (seeded) drafts every step would commit 32 tokens, the base batch-32 rate."""
    import torch
    from thvm_b200.dsv2 import DSConfig, ds_shard
    from thvm_b200.spec import SpecDecoder
    ctx.init_cuda()
    n_seq, S = 8, 4
    cfg = DSConfig(n_layers=args.layers or DSConfig().n_layers, batch=n_seq * S)
    sh = ds_shard(cfg, ctx.rank, ctx.world)
    sd = SpecDecoder(cfg, {}, sh, n_seq, S, group=ctx.group)
    sd.model.w = ds_device_weights(cfg, sh)
    prompts = np.random.default_rng(1).integers(0, cfg.vocab, (n_seq, N_PROMPT_DS)).astype(np.int32)
    if ctx.world > 1:
        t = torch.zeros(1, device="cuda")
        ctx.dist.all_reduce(t)
    sd.prefill(prompts)
    n0 = sd.model.launches
    sd.capture()
    per_step = sd.model.launches - n0
    limit = cfg.max_ctx - S - 1
    sd.replay(args.warmup)
    torch.cuda.synchronize()
    c0 = int(sd.committed.item())
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(ctx.local) as clk:
        ctx.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        sd.replay(args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
        ctx.barrier()
    ms = ctx.max(e0.elapsed_time(e1))
    ids, ln = sd.stream_ids()
    if ctx.max(float(sd.status())) != 0 or ln.max() >= limit:
        raise RuntimeError(f"speculative steps did not finish cleanly (status {sd.status()}, lengths {ln.tolist()})")
    committed = int(sd.committed.item()) - c0
    value = committed / (ms / 1e3)
    # e2e: every step also reads the sequences' lengths back to pinned host memory
    host_len = torch.empty(n_seq, dtype=torch.int32).pin_memory()
    e2e_steps = max(1, min(args.steps, 10))
    c1 = int(sd.committed.item())
    ctx.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        sd.replay()
        host_len.copy_(sd.len, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e2e_s = ctx.max(time.perf_counter() - t0)
    e2e = (int(sd.committed.item()) - c1) / e2e_s
    line = base_line(
        args, ctx.world, round(value, 1), ms, scaling="strong", dtype="fp8 e4m3 experts, bf16 activations / weights",
        config={"workload": "config 5 model, blind speculative decode: 8 sequences x 4 verify rows (32 rows a step), "
                            "64 prompt ids, bigram drafts (bench/dsv2_decode_bench.c DSV2_SPEC)",
                "global_batch": n_seq * S, "sequences": n_seq, "verify_rows": S,
                "positions": [int(ln.min()), int(ln.max())],
                "parallelism": f"tp{ctx.world} attention heads / dense units / vocab, ep{ctx.world} experts"},
        committed_per_sequence_step=round(committed / (n_seq * args.steps), 3),
        forced_upper_bound_tok_s=round(n_seq * S * args.steps / (ms / 1e3), 1),
        gpu_launches=per_step * args.steps, gpu_launches_per_step=per_step,
        e2e={"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4 * n_seq,
             "steps": e2e_steps},
        clocks=clk.summary())
    del sd
    torch.cuda.empty_cache()
    return line


def moe_reference(args, ctx):
    """The reference's own DeepSeek-V2 decode bench (bench/dsv2_decode_bench.c,
    built CPU-only into oracle/_ref) at full width, batch 1 (the only batch it
    has), one process per core group: P processes with 2 and then 3 layers
    (dense layer 0, then MoE layers) each time WARM=1, STEPS=2 replays; the
    27-layer token time is t2 + 25 (t3 - t2) and `value` = P / that."""
    exe = ROOT / "oracle" / "_ref" / "dsv2_decode_bench"
    line = {"metric": METRIC, "unit": "tok/s", "impl": "reference", "n_gpus": ctx.world}
    if not exe.exists():
        line["unavailable"] = "oracle/_ref/dsv2_decode_bench not built (build() compiles it where the reference is)"
        print(json.dumps(line), flush=True)
        return
    P = max(1, min(8, os.cpu_count() or 1))
    # one process first, so the CPU JIT's kernel cache (compiled once, keyed by
    # source) is complete before the concurrent runs look it up
    warm = subprocess.run([str(exe)], env=dict(os.environ, DEV="cpu", DSV2_LAYERS="2", WARM="0", STEPS="1"),
                          capture_output=True, text=True, timeout=900)
    if warm.returncode != 0:
        raise RuntimeError(f"reference dsv2 bench failed ({warm.returncode}): {warm.stdout[-2000:]}")
    per = {}
    for layers in (2, 3):
        env = dict(os.environ, DEV="cpu", DSV2_LAYERS=str(layers), WARM="1", STEPS="2")
        procs = [subprocess.Popen([str(exe)], env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
                 for _ in range(P)]
        ms = []
        for pr in procs:
            out, _ = pr.communicate(timeout=900)
            for ln in out.splitlines():
                if "timed" in ln and "mean" in ln:
                    ms.append(float(ln.split("mean")[1].split("ms/step")[0]))
            if pr.returncode != 0:
                raise RuntimeError(f"reference dsv2 bench failed ({pr.returncode}): {out[-2000:]}")
        per[layers] = float(np.mean(ms))
    t27 = per[2] + 25 * (per[3] - per[2])
    value = P / (t27 / 1e3)
    line.update({
        "value": round(value, 3), "steps": 2, "warmup": 1, "ms_per_step": round(t27, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16 (the reference's decode bench has no fp8 experts)",
        "data": "synthetic",
        "config": {"workload": "config 5: DeepSeek-V2-Lite-shaped MoE decode (the reference's batch-1 step)",
                   "sample": f"{P} processes x (2 and 3 layers, 1 warm + 2 timed replays); ms/token {per[2]:.1f} "
                             f"and {per[3]:.1f}; 27 layers = t2 + 25 (t3 - t2)"},
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": P, "kind": "reference",
                         "sample": f"{P} concurrent single-threaded decoders, full width, 2 and 3 layers"},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    print(json.dumps(line), flush=True)


# ============================================================================
# config 1: GPT-2 small fp32 b1 (fused decode kernel, 64 tokens per replay)
# ============================================================================

N_PROMPT, N_NEW = 16, 64


def gpt2_weight_params(cfg):
    """Parameters one decode token reads: every block (c_attn 3d x d, c_proj
    d x d, c_fc h x d, mlp.c_proj d x h, their biases, two LayerNorms), ln_f
    and lm_head; the embeddings contribute one row each (counted per token)."""
    d, h = cfg.dim, cfg.hidden
    block = 3 * d * d + d * d + h * d + d * h + (3 * d + d + h + d) + 4 * d
    return cfg.n_layers * block + 2 * d + cfg.vocab * d


def gpt2_tokens_bytes(cfg, pos0, n):
    """Algorithmic HBM bytes of n decode tokens at positions pos0..pos0+n-1:
    per token all weights once, the wte and wpe rows, the keys and values of
    the earlier positions (pos rows per layer) and the new row written."""
    d = cfg.dim
    per_tok = 4 * gpt2_weight_params(cfg) + 2 * 4 * d + cfg.n_layers * 2 * 4 * d
    kv_rows = sum(range(pos0, pos0 + n))
    return n * per_tok + cfg.n_layers * 2 * 4 * d * kv_rows


def gpt2_cpu_baseline(cfg, weights, prompt, seconds=15.0):
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


def gpt2_run(args, ctx, cpu: bool):
    import torch
    from thvm_b200.device import Device
    from thvm_b200.gpt2 import Transformer
    from thvm_b200.synthetic import GPT2_SMALL, gpt2_weights, prompt_tokens
    ctx.init_cuda()
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
    launches0 = dev.launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(ctx.local) as clk:
        ctx.barrier()
        torch.cuda.synchronize()
        dev.sync()
        e0.record(stream)
        for _ in range(args.steps):
            model.replay_run()
        e1.record(stream)
        dev.sync()
        torch.cuda.synchronize()
        ctx.barrier()
    launches = dev.launches() - launches0
    ms = ctx.max(e0.elapsed_time(e1))
    last_tok = model.current_token()
    value = ctx.world * N_NEW * args.steps / (ms / 1e3)
    hbm, _, peak_kind = peaks()
    run_bytes = gpt2_tokens_bytes(cfg, N_PROMPT, N_NEW)
    step_gbs = run_bytes * args.steps / (ms / 1e3) / 1e9
    if not model.fused:
        raise RuntimeError("the fused decode kernel is not in use")
    # the run graph is one decode_kernel launch over the 64 tokens plus two
    # 4-byte copy nodes that reset (token, position): the replay's event-timed
    # duration is the launch's duration (copies included)
    kern_us = ms * 1e3 / args.steps
    ach = run_bytes / (kern_us / 1e6) / 1e9
    roof = {"bound": "hbm", "kernel": "decode_kernel (fused GPT-2 decode, 64 tokens per launch)",
            "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s", "frac": round(ach / hbm, 4),
            "peak_source": peak_kind, "bytes_per_launch": run_bytes, "avg_launch_us": round(kern_us, 3),
            "traffic": ncu_traffic("decode_kernel"),
            "step": {"algorithmic_bytes_per_token": round(run_bytes / N_NEW), "achieved_gbs": round(step_gbs, 1),
                     "frac": round(step_gbs / hbm, 4)}}
    status = model.decode_status()
    if status:
        raise RuntimeError(f"decode kernel status {status:#x}")
    # e2e through the C-ABI with host buffers: token and position in, next id out, every token
    e2e_steps = max(1, min(args.steps, 5))
    model.capture_step()
    io = torch.empty(2, dtype=torch.int32, pin_memory=True)
    out = torch.empty(1, dtype=torch.int32, pin_memory=True)
    L = dev.lib
    ctx.barrier()
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
    e2e_s = ctx.max(time.perf_counter() - t0)
    e2e = ctx.world * N_NEW * e2e_steps / e2e_s
    line = base_line(
        args, ctx.world, round(value, 1), ms, scaling="weak", dtype="f32",
        config={"workload": "config 1: gpt2-small fp32 b1, 16-id prompt, 64 greedy decode tokens (positions 16..79) "
                            "per step, one CUDA-graph replay per step",
                "model": "gpt2 124M (12L d768 12x64 MLP3072 vocab 50257 ctx 1024), seeded N(0,0.02)",
                "global_batch": ctx.world, "seq_len": N_PROMPT + N_NEW, "tokens_per_step": N_NEW,
                "parallelism": f"replicas{ctx.world}",
                "l2": "weights (495 MB) exceed L2 (126 MB): every step streams them from HBM"},
        ms_per_token=round(ms / args.steps / N_NEW, 5), last_token=last_tok, gpu_launches=int(launches),
        roofline=roof,
        e2e={"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": 8 * N_NEW,
             "d2h_bytes_per_step": 4 * N_NEW, "steps": e2e_steps},
        clocks=clk.summary())
    line["metric"] = "GPT-2 124M b1 fp32 decode tok/s"
    if cpu and ctx.rank == 0 and ctx.world == 1:
        line["cpu_baseline"] = gpt2_cpu_baseline(cfg, weights, prompt)
    return line


def gpt2_reference(args, ctx):
    """The CPU path of config 1 on the host cores (the oracle port, bit-identical
    to the reference's CPU path on these weights)."""
    if ctx.rank != 0:
        return
    import oracle as O
    from thvm_b200.synthetic import GPT2_SMALL, gpt2_weights, prompt_tokens
    cfg = GPT2_SMALL
    m = O.GPT2(cfg, gpt2_weights(cfg, seed=0))
    prompt = prompt_tokens(N_PROMPT, cfg.vocab, seed=1)
    tok = m.forward(prompt, 0)
    pos, per_step = N_PROMPT, 4
    for _ in range(args.warmup):
        tok = m.forward([tok], pos)
        pos += 1
    t0, n = time.perf_counter(), 0
    for _ in range(args.steps):
        for _ in range(per_step):
            if pos >= N_PROMPT + N_NEW:
                tok, pos = m.forward(prompt, 0), N_PROMPT
            tok = m.forward([tok], pos)
            pos += 1
            n += 1
    dt = time.perf_counter() - t0
    v = n / dt
    print(json.dumps({"metric": "GPT-2 124M b1 fp32 decode tok/s", "value": round(v, 3), "unit": "tok/s",
                      "n_gpus": ctx.world, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": round(dt * 1e3 / args.steps, 3), "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
                      "config": {"workload": "gpt2-small decode, b1, 16-id prompt, greedy tokens at positions 16..79",
                                 "tokens_per_step": per_step},
                      "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": O.num_threads(),
                                       "kind": "port", "sample": f"{per_step} decode tokens per step, full model"},
                      "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)


# ============================================================================
# configs 2 and 4: kernel cases on one GPU (cold operands, graph-replayed)
# ============================================================================

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

    def __init__(self, dev):
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
        for _ in range(3):
            dev.replay(slot)
        dev.sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        dev.replay(slot)
        e1.record(self.stream)
        e1.synchronize()
        dev.drop(slot)
        return e0.elapsed_time(e1) / iters


def copies_for(nbytes: int, l2: int = L2_BYTES) -> int:
    """Operand copies so that the rotation covers more than twice L2."""
    return max(2, -(-2 * l2 // max(nbytes, 1)))


def matvec_cases(dev, timer, iters: int):
    from thvm_b200 import _lib as L
    from thvm_b200.gpt2 import make_op
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
        out.append({"case": f"config 2: matvec {name}", "M": M, "N": N, "K": K, "kernel": "gemv_tma_kernel",
                    "us": round(ms * 1e3, 2), "bytes": byts, "achieved": round(gbs, 1), "unit": "GB/s",
                    "peak": hbm, "frac": round(gbs / hbm, 4), "peak_source": kind,
                    "l2": f"{len(ops)} weight copies rotated (> 2x L2)"})
        for bid in bufs:
            dev.free(bid)
    dev.free(xb)
    dev.free(y)
    return out


def gemm_cases(dev, timer, iters: int):
    from thvm_b200 import _lib as L
    lib = dev.lib
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
        out.append({"case": "config 2: bf16 GEMM", "M": M, "N": N, "K": K, "kernel": "gemm_bf16_kernel",
                    "us": round(ms * 1e3, 2), "flops": 2 * M * N * K, "achieved": round(tf, 1),
                    "unit": "TFLOP/s", "peak": tflops, "frac": round(tf / tflops, 4), "peak_source": kind})
        for a, b in sets:
            dev.free(a)
            dev.free(b)
        dev.free(c)
    return out


def prefill_cases(dev, timer, iters: int):
    from thvm_b200 import _lib as L
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
        if lib.sm100_attn_prefill_status() != 0:
            raise RuntimeError("prefill kernel status word set")
        flops = 2 * B * H * S * S * D
        tf = flops / (ms / 1e3) / 1e12
        out.append({"case": "config 4: causal attention prefill", "B": B, "H": H, "S": S, "D": D,
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
DS_SHAPES = (("ds_qkva", 3648, 2048), ("ds_w_o", 2048, 2048), ("ds_router", 64, 2048),
             ("ds_dense_gu", 21888, 2048), ("ds_dense_down", 2048, 10944), ("ds_lm_head", 102400, 2048))


def skinny_cases(dev, timer, iters: int, M: int = 16, shapes=XL_SHAPES):
    """Skinny bf16 GEMM launches (bf16 weights streamed once per launch;
    HBM-bound): the GPT-2-XL projections of config 3 at batch 16, or the
    given shapes at batch M."""
    from thvm_b200 import _lib as L
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
        if lib.sm100_skinny_status() != 0:
            raise RuntimeError("skinny kernel status word set")
        byts = w.nbytes + x.nbytes + M * N * 4
        gbs = byts / (ms / 1e3) / 1e9
        out.append({"case": f"skinny {name}", "M": M, "N": N, "K": K, "kernel": "skinny_kernel",
                    "us": round(ms * 1e3, 2), "bytes": byts, "achieved": round(gbs, 1), "unit": "GB/s",
                    "peak": hbm, "frac": round(gbs / hbm, 4), "peak_source": kind,
                    "l2": f"{len(ws_)} weight copies rotated (> 2x L2)"})
        for bid in ws_ + [xb, y, ws, cnt]:
            dev.free(bid)
    return out


def kernel_cases(iters: int = 20, skinny: bool = False):
    from thvm_b200.device import Device
    dev = Device.get()
    timer = Timer(dev)
    rows = matvec_cases(dev, timer, iters) + gemm_cases(dev, timer, iters) + prefill_cases(dev, timer, iters)
    if skinny:
        rows += skinny_cases(dev, timer, iters) + skinny_cases(dev, timer, iters, 32, DS_SHAPES)
    return rows


# ============================================================================
# config 3: GPT-2-XL-shaped bf16 decode, batch 16, tensor-parallel
# ============================================================================

def xl_device_weights(cfg, sh, seed: int = 0) -> dict:
    """This rank's shard of synthetic weights, generated on the device."""
    import torch
    from thvm_b200.gpt2_xl import HEAD_DIM
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


def xl_step_bytes(cfg, pos: int) -> int:
    """Algorithmic HBM bytes of one step over the whole job: every weight
    once (bf16) and the K and V rows 0..pos of every layer (bf16)."""
    D, F, V = cfg.dim, cfg.hidden, cfg.vocab
    per_layer = (3 * D * D + D * D + F * D + D * F) * 2 + (3 * D + D + F + D) * 4
    weights = cfg.n_layers * per_layer + V * D * 2
    kv = cfg.n_layers * 2 * cfg.batch * (pos + 1) * D * 2
    return weights + kv


_XL_CPU_WEIGHTS: dict = {}


def xl_cpu_sample(batch: int = 16, seed: int = 0):
    """The oracle port (oracle.c orc_xl_step: the reference's CPU GPT-2 forward
    with bf16 weights, pthreads over the host cores) on a bounded sample of
    config 3: one batch-16 decode step of the full-width model (d 1600, 25
    heads, vocab 50257) with 1 and with 2 layers after one warm step each;
    the 48-layer step time is t1 + 47 (t2 - t1).  -> (tok/s, sample text, s)."""
    import oracle as O
    from thvm_b200.gpt2_xl import GPT2_XL, XLConfig, xl_weights
    key = (batch, seed)
    if key not in _XL_CPU_WEIGHTS:   # generated once per process
        _XL_CPU_WEIGHTS[key] = xl_weights(XLConfig(n_layers=2, max_ctx=64, batch=batch), seed=seed)
    w = _XL_CPU_WEIGHTS[key]
    tok = np.random.default_rng(1).integers(0, GPT2_XL.vocab, batch).astype(np.int32)
    times = []
    for n in (1, 2):
        cfg = XLConfig(n_layers=n, max_ctx=64, batch=batch)
        m = O.XLModel(cfg, {k: v for k, v in w.items() if not k.startswith("h.") or int(k.split(".")[1]) < n})
        m.step(tok, 0)
        t0 = time.perf_counter()
        m.step(tok, 1)
        times.append(time.perf_counter() - t0)
    t48 = times[0] + (GPT2_XL.n_layers - 1) * (times[1] - times[0])
    return (batch / t48, f"one batch-{batch} decode step of the full-width model with 1 and 2 layers "
                         f"({times[0]:.2f} s, {times[1]:.2f} s); 48-layer step = t1 + 47 (t2 - t1) = {t48:.2f} s", t48)


def xl_reference(args, ctx):
    """The CPU path of config 3 on the host cores: the oracle port of the
    reference's GPT-2 forward with bf16 weights (xl_cpu_sample), args.steps
    samples after args.warmup untimed ones (each sample a 1- and 2-layer
    step pair: the whole run stays within minutes)."""
    import oracle as O
    for _ in range(max(args.warmup, 0)):
        xl_cpu_sample()
    vals, ts, text = [], [], ""
    for _ in range(max(args.steps, 1)):
        v, text, t48 = xl_cpu_sample()
        vals.append(v)
        ts.append(t48)
    v = float(np.mean(vals))
    print(json.dumps({"metric": "decode tok/s (GPT-2 XL bf16 b16, tensor-parallel)", "value": round(v, 3),
                      "unit": "tok/s", "n_gpus": ctx.world, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": round(float(np.mean(ts)) * 1e3, 1), "higher_is_better": True,
                      "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                      "impl": "reference",
                      "config": {"workload": "config 3: GPT-2 XL-shaped bf16 decode, batch 16", "sample": text},
                      "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": O.num_threads(), "kind": "port",
                                       "sample": text},
                      "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)


def prefill_reference(args, ctx):
    """The CPU path of config 4 on the host cores: the oracle port of the
    reference's scaled_dot_product_attention with the causal mask
    (oracle.c orc_sdpa_f32, f32 on the bf16-valued inputs) over a bounded
    sample, 2 of the 64 (batch, head) pairs at S = 2048, D = 128 per step;
    TFLOP/s = the pairs' algorithmic FLOPs (2 S^2 D each, the config's count)
    / time."""
    import oracle as O
    S, D, pairs = 2048, 128, 2
    rng = np.random.default_rng(4)
    q, k, v = (O.bf16_to_f32(bf16_bits(rng.standard_normal((pairs, S, D)).astype(np.float32))) for _ in range(3))
    for _ in range(max(args.warmup, 0)):
        O.sdpa(q, k, v, causal=True)
    t0 = time.perf_counter()
    for _ in range(max(args.steps, 1)):
        O.sdpa(q, k, v, causal=True)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    tf = pairs * 2.0 * S * S * D / dt / 1e12
    sample = f"{pairs} of the 64 (batch, head) pairs per step, S {S}, D {D}, causal, f32 on bf16 values"
    print(json.dumps({"metric": "causal prefill TFLOP/s (B4 H16 S2048 D128 bf16)", "value": round(tf, 5),
                      "unit": "TFLOP/s", "n_gpus": ctx.world, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": round(dt * 1e3, 1), "higher_is_better": True, "scaling": "strong",
                      "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
                      "config": {"workload": "config 4: causal attention prefill B4 H16 S2048 D128", "sample": sample},
                      "cpu_baseline": {"value": round(tf, 5), "unit": "TFLOP/s", "cores": O.num_threads(),
                                       "kind": "port", "sample": sample},
                      "e2e": {"value": round(tf, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)


def xl_prefill_flops(cfg, P: int) -> int:
    """Algorithmic FLOPs of the prompt pass over the whole job: the four
    projections of every layer on all B P rows, the causal q k^T and p v
    (P (P + 1) / 2 query-key pairs per sequence and head, 64 wide), and
    lm_head on the B last rows."""
    D, F, M = cfg.dim, cfg.hidden, cfg.batch * P
    proj = 2 * M * (3 * D * D + D * D + 2 * F * D)
    attn = 2 * 2 * 64 * (P * (P + 1) // 2) * cfg.batch * cfg.heads
    return cfg.n_layers * (proj + attn) + 2 * cfg.batch * D * cfg.vocab


def xl_run(args, ctx):
    import torch
    from thvm_b200.gpt2_xl import GPT2_XL, XLConfig, XLModel, shard_of
    ctx.init_cuda()
    cfg = XLConfig(n_layers=args.layers or GPT2_XL.n_layers)
    n_prompt = 128
    assert n_prompt + args.warmup + args.steps <= cfg.max_ctx
    sh = shard_of(cfg, ctx.rank, ctx.world)
    model = XLModel(cfg, {}, sh, ctx.group)
    model.w = xl_device_weights(cfg, sh)
    prompts = torch.from_numpy(np.random.default_rng(1).integers(0, cfg.vocab, (cfg.batch, n_prompt))
                               .astype(np.int32)).cuda()
    if ctx.world > 1:
        t = torch.zeros(1, device="cuda")
        ctx.dist.all_reduce(t)
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
    # the prompt pass: every prompt position through each layer at once
    # (tcgen05 GEMM with fused epilogues, tcgen05 causal prefill attention);
    # once untimed (buffers, launch attributes), then timed
    # (at N = 1 a CUDA graph of its launches, captured after one eager pass;
    # split over ranks its per-block NCCL all-reduces run eagerly, uncaptured)
    model.prefill_ids(prompts.cpu().numpy())
    with torch.cuda.stream(s):
        model.prefill_run(n_prompt)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    pf_graph = None
    if ctx.world == 1:
        pf_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(pf_graph):
            model.prefill_run(n_prompt)
        pf_graph.replay()
    else:
        model.prefill_run(n_prompt)
    torch.cuda.synchronize()
    ctx.barrier()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    if pf_graph is not None:
        pf_graph.replay()
    else:
        model.prefill_run(n_prompt)
    p1.record()
    p1.synchronize()
    pf_ms = ctx.max(p0.elapsed_time(p1))
    del pf_graph
    pf_flops = xl_prefill_flops(cfg, n_prompt)
    _, bf16_peak, _ = peaks()
    for _ in range(args.warmup):
        graph.replay()
    pos0 = n_prompt + args.warmup
    torch.cuda.synchronize()
    ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(ctx.local) as clk:
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        e1.synchronize()
    ms = ctx.max(e0.elapsed_time(e1))
    toks = cfg.batch * args.steps / (ms / 1e3)
    byts = sum(xl_step_bytes(cfg, pos0 + i) for i in range(args.steps))
    achieved = byts / (ms / 1e3) / 1e9
    hbm, _, kind = peaks()
    del graph
    line = base_line(args, ctx.world, round(toks, 1), ms, scaling="strong", dtype="bf16",
                     config={"workload": "config 3: GPT-2 XL-shaped bf16 decode, batch 16", "layers": cfg.n_layers,
                             "batch": cfg.batch, "prompt": n_prompt, "positions": [pos0, pos0 + args.steps - 1],
                             "parallelism": f"tp{ctx.world}"},
                     roofline={"bound": "hbm", "kernel": "whole decode step", "achieved": round(achieved, 1),
                               "peak": round(hbm * ctx.world, 1), "unit": "GB/s",
                               "frac": round(achieved / (hbm * ctx.world), 4), "traffic": None, "peak_source": kind,
                               "bytes_per_step": byts // args.steps},
                     gpu_launches=per_step * args.steps, clocks=clk.summary())
    line["metric"] = "decode tok/s (GPT-2 XL bf16 b16, tensor-parallel)"
    pf_tflops = pf_flops / (pf_ms / 1e3) / 1e12
    line["prefill"] = {"ms": round(pf_ms, 3), "prompt_tok_s": round(cfg.batch * n_prompt / (pf_ms / 1e3), 1),
                       "flops": pf_flops, "tflops": round(pf_tflops, 1),
                       "frac": round(pf_tflops / (bf16_peak * ctx.world), 4), "peak_source": kind,
                       "what": f"XLModel.prefill_run of [{cfg.batch}, {n_prompt}] ids, "
                               + ("one CUDA graph replay" if ctx.world == 1 else "eager launches")}
    return line


# ============================================================================
# config 4 over N GPUs: the (batch, head) pairs split over the ranks
# ============================================================================

def pair_range(n_pairs: int, rank: int, world: int) -> tuple[int, int]:
    """The contiguous (batch, head) pairs [p0, p1) of a rank: an even split."""
    return n_pairs * rank // world, n_pairs * (rank + 1) // world


def prefill_run(args, ctx):
    import torch
    from thvm_b200 import _lib as L
    ctx.init_cuda()
    B, H, S, D = 4, 16, 2048, 128
    lib = L.lib()
    L.check(lib.sm100_init(), "init")
    p0, p1 = pair_range(B * H, ctx.rank, ctx.world)
    n = p1 - p0
    g = torch.Generator(device="cuda")
    g.manual_seed(1000 + ctx.rank)
    copies = max(1, -(-2 * L2_BYTES // max(3 * n * S * D * 2, 1)))
    sets = [[torch.randn(n, S, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3)]
            for _ in range(copies)]
    o = torch.empty(n, S, D, dtype=torch.float32, device="cuda")

    def launch(i):
        q, k, v = sets[i % copies]
        L.check(lib.sm100_attn_prefill_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), 1, n, S, D,
                                            1.0 / D ** 0.5, 1, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
                "attn_prefill")

    for i in range(args.warmup):
        launch(i)
    torch.cuda.synchronize()
    ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(ctx.local) as clk:
        e0.record()
        for i in range(args.steps):
            launch(i)
        e1.record()
        e1.synchronize()
    ms = ctx.max(e0.elapsed_time(e1))
    if lib.sm100_attn_prefill_status() != 0:
        raise RuntimeError("prefill kernel status word set")
    flops = 2 * B * H * S * S * D
    tf = flops * args.steps / (ms / 1e3) / 1e12
    _, peak, kind = peaks()
    line = base_line(args, ctx.world, round(tf, 1), ms, scaling="strong", dtype="bf16",
                     config={"workload": "config 4: causal attention prefill B4 H16 S2048 D128", "p": "bf16 hi+lo",
                             "pairs_per_rank": n, "parallelism": f"bh{ctx.world}",
                             "l2": f"{copies} input copies rotated per rank (> 2x L2)"},
                     roofline={"bound": "tensor", "kernel": "attn_prefill_kernel", "achieved": round(tf, 1),
                               "peak": round(peak * ctx.world, 1), "unit": "TFLOP/s",
                               "frac": round(tf / (peak * ctx.world), 4), "peak_source": kind},
                     clocks=clk.summary())
    line.update(metric="causal prefill TFLOP/s (B4 H16 S2048 D128 bf16)", unit="TFLOP/s")
    return line


# ============================================================================

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="sm100", choices=["sm100", "reference"])
    ap.add_argument("--workload", default="moe", choices=["moe", "spec", "gpt2", "xl", "prefill", "kernels"])
    ap.add_argument("--layers", type=int, default=0, help="moe / xl: fewer layers (0 = the full model)")
    ap.add_argument("--no-extras", action="store_true", help="moe at N = 1: skip the config-1 and kernel lines")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    ctx = Ctx()
    if args.impl == "reference":
        if ctx.rank != 0:
            return
        arms = {"moe": moe_reference, "xl": xl_reference, "prefill": prefill_reference, "gpt2": gpt2_reference}
        if args.workload not in arms:
            why = {"spec": "no reference arm for the speculative workload (the reference's DSV2_SPEC mode is its "
                           "batch-1 decode bench; the default workload's arm runs that bench)",
                   "kernels": "the kernel cases are single launches with no reference CPU metric of their own"}
            print(json.dumps({"impl": "reference", "unavailable": why.get(args.workload, args.workload)}), flush=True)
            return
        return arms[args.workload](args, ctx)
    args.warmup = max(args.warmup, 3)
    cpu = not args.no_cpu_baseline and ctx.rank == 0 and ctx.world == 1
    try:
        if args.workload == "moe":
            line = moe_run(args, ctx)
            if cpu:
                line["cpu_baseline"] = moe_cpu_baseline(32)
            if ctx.world == 1 and not args.no_extras:
                line["gpt2_small"] = gpt2_run(args, ctx, cpu)
                line["kernels"] = kernel_cases()
        elif args.workload == "spec":
            line = spec_run(args, ctx)
        elif args.workload == "gpt2":
            line = gpt2_run(args, ctx, cpu)
        elif args.workload == "xl":
            line = xl_run(args, ctx)
            if cpu:
                import oracle as O
                v, text, _ = xl_cpu_sample()
                line["cpu_baseline"] = {"value": round(v, 3), "unit": "tok/s", "cores": O.num_threads(), "kind": "port",
                                        "sample": text}
        elif args.workload == "prefill":
            line = prefill_run(args, ctx)
        else:
            for r in kernel_cases(skinny=True):
                print(json.dumps(r), flush=True)
            return
        if ctx.rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        ctx.close()


if __name__ == "__main__":
    main()
