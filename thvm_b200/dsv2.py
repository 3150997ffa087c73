"""Batched decode of a DeepSeek-V2-Lite-shaped MoE decoder
on the sm_100a kernels, tensor- and expert-parallel over the GPUs of one box.

Shapes (bench/dsv2_decode_bench.c cfg :97-124): 27 layers, d 2048, 16 heads,
multi-head latent attention (kv_lora 512, rope 64, nope 128, v 128), layer 0
a dense SiLU MLP (10944), layers 1-26 64 routed experts (1408) with top-6
routing over the router logits (softmax weights, no renormalisation, ties to
the lowest id) plus 2 shared experts, vocab 102400, batch 32.  Precision:
routed and shared expert weights fp8-e4m3 with one f32 scale per 128 x 128
block; attention, router, dense layer 0, embedding and lm_head bf16; f32
residual stream, bf16 matmul operands (the oracle's orc_ds_step states the op
order).  The two shared experts are one SiLU MLP of 2816 units, taken as two
halves of 1408 whose outputs add (exact), so they ride the routed-expert
kernel with weight 1.

Per layer: RMSNorm -> fused q | kv_a projection (skinny tcgen05 GEMM) ->
q / latent post-processing (bf16, RMSNorm of the latent, YaRN rotary, cache
append) and the absorbed MLA over the compressed cache (one launch at the
model's shapes) -> o projection into the residual -> RMSNorm -> dense MLP (layer 0) or the router product and the
routing (one launch), fp8 experts (gate / up + SiLU, then down weighted into
the residual).

Parallelism over R ranks (rank r), every weight byte read by one rank:
  * attention by heads: heads split_even(16, R, r); the q rows of those
    heads and the whole kv_a block (the latent every head reads) in the
    fused projection, their W_uk / W_uv, and their columns of W_o (a
    row-split product whose partial sums meet in one all-reduce);
  * dense layer 0 by hidden units: gate / up rows and down columns of
    split_even(10944, R, r), one all-reduce;
  * experts by expert: routed experts split_even(64, R, r) and the shared
    halves k with k % R == r; every rank routes every token (the router is
    replicated, 256 KB) and keeps the slots of its experts; one all-reduce;
  * lm_head by vocabulary rows split_even(102400, R, r); each rank's (max,
    index) per row are all-gathered and the smallest index of the largest
    value wins.
The residual stream h is replicated: after each all-reduce every rank holds
the same h.  Rank 0 adds its partial sums into h; the other ranks overwrite
h with theirs (or zero it before the experts add into it), so the all-reduce
sum is h + sum of the partials.  Each all-reduce is the library's
peer-memory kernel fused with the RMSNorm that consumes h (thvm_b200/comm.py,
sm100_comm_allreduce_rmsnorm: the ranks' rows summed in rank order, the same
h on every rank), and the argmax candidates meet in sm100_comm_pick, so a
step issues no library collective; torch.distributed only exchanges the IPC
handles at set-up.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np

from . import _lib as L
from .gpt2_xl import split_even


@dataclass(frozen=True)
class DSConfig:
    n_layers: int = 27
    dim: int = 2048
    heads: int = 16
    kv_lora: int = 512
    d_nope: int = 128
    d_rope: int = 64
    d_v: int = 128
    n_exp: int = 64
    top_k: int = 6
    moe_inter: int = 1408
    dense_inter: int = 10944
    n_dense: int = 1
    n_shared: int = 2
    vocab: int = 102400
    max_ctx: int = 1024
    batch: int = 32
    eps: float = 1e-6

    @property
    def q_cols(self) -> int:   # q rows of the fused projection
        return self.heads * (self.d_nope + self.d_rope)

    @property
    def n_qkva(self) -> int:
        return self.q_cols + self.kv_lora + self.d_rope

    @property
    def scale(self) -> float:
        """(d_nope + d_rope)^-0.5 * mscale^2, mscale = 0.1 * 0.707 * ln(40) + 1 (YaRN)."""
        mscale = 0.1 * 0.707 * math.log(40.0) + 1.0
        return float((self.d_nope + self.d_rope) ** -0.5 * mscale * mscale)


DSV2_LITE = DSConfig()


def yarn_tables(d_rope: int, max_ctx: int, theta: float = 10000.0, factor: float = 40.0, orig: float = 4096.0,
                beta_fast: float = 32.0, beta_slow: float = 1.0) -> tuple[np.ndarray, np.ndarray]:
    """cos / sin [max_ctx, d_rope] f32 of YaRN-scaled rotary frequencies (Peng et al. 2023,
    "YaRN"): dims below the beta_fast correction keep the base frequency theta^(-2j/d),
    dims above beta_slow are divided by `factor`, a linear ramp between; halves duplicated."""
    half = d_rope // 2
    lo = math.floor(d_rope * math.log(orig / (beta_fast * 2 * math.pi)) / (2 * math.log(theta)))
    hi = math.ceil(d_rope * math.log(orig / (beta_slow * 2 * math.pi)) / (2 * math.log(theta)))
    lo, hi = max(lo, 0), min(hi, d_rope - 1)
    j = np.arange(half, dtype=np.float64)
    pf = theta ** (2 * j / d_rope)
    ramp = np.clip((j - lo) / max(hi - lo, 1e-3), 0.0, 1.0)
    freqs = (1.0 / (factor * pf)) * ramp + (1.0 / pf) * (1.0 - ramp)
    ang = np.arange(max_ctx, dtype=np.float64)[:, None] * freqs[None, :]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    return np.concatenate([cos, cos], 1), np.concatenate([sin, sin], 1)


def _bf16(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _fp8(a: np.ndarray) -> np.ndarray:
    """f32 (|a| < 448) -> e4m3 codes, round to nearest even."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def ds_weights(cfg: DSConfig, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Synthetic weights: bf16 matrices N(0, std); fp8 expert codes of N(0, 1)
    draws with block scales U[0.5, 2] * std (weights ~ N(0, std) per block);
    RMSNorm gains 1."""
    rng = np.random.default_rng(seed)
    D, H, KV, DN, DR, DV = cfg.dim, cfg.heads, cfg.kv_lora, cfg.d_nope, cfg.d_rope, cfg.d_v
    E, I, NS, DI = cfg.n_exp, cfg.moe_inter, cfg.n_shared, cfg.dense_inter

    def mat(*shape):
        return _bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))

    def fp8_blocks(n, rows, cols):
        codes = _fp8(rng.standard_normal((n, rows, cols), dtype=np.float32))
        sc = (rng.uniform(0.5, 2.0, (n, -(-rows // 128), -(-cols // 128))) * std).astype(np.float32)
        return codes, sc

    w = {"embed": mat(cfg.vocab, D), "lm_head": mat(cfg.vocab, D), "norm_f": np.ones(D, np.float32)}
    for l in range(cfg.n_layers):
        p = f"l{l}."
        w[p + "attn_norm"], w[p + "ffn_norm"] = np.ones(D, np.float32), np.ones(D, np.float32)
        w[p + "kv_norm"] = np.ones(KV, np.float32)
        w[p + "w_qkva"] = mat(cfg.n_qkva, D)
        w[p + "w_uk"], w[p + "w_uv"] = mat(H, DN, KV), mat(H, DV, KV)
        w[p + "w_o"] = mat(D, H * DV)
        if l < cfg.n_dense:
            w[p + "d_gu"], w[p + "d_down"] = mat(2 * DI, D), mat(D, DI)
        else:
            w[p + "router"] = mat(E, D)
            w[p + "e_gu"], w[p + "e_gu_s"] = fp8_blocks(E + NS, 2 * I, D)
            w[p + "e_d"], w[p + "e_d_s"] = fp8_blocks(E + NS, D, I)
    return w


@dataclass(frozen=True)
class DSShard:
    """What rank r of R holds: heads [h0, h1), dense hidden units [f0, f1),
    routed experts [e0, e1) and the shared halves `shared`, vocab rows
    [v0, v1)."""
    rank: int
    world: int
    h0: int
    h1: int
    f0: int
    f1: int
    e0: int
    e1: int
    shared: tuple
    v0: int
    v1: int

    @property
    def heads(self) -> int:
        return self.h1 - self.h0


def ds_shard(cfg: DSConfig, rank: int, world: int) -> DSShard:
    if not 0 <= rank < world or world > cfg.heads or world > cfg.n_exp:
        raise ValueError(f"rank {rank} of {world} (heads {cfg.heads}, experts {cfg.n_exp})")
    return DSShard(rank, world, *split_even(cfg.heads, world, rank), *split_even(cfg.dense_inter, world, rank),
                   *split_even(cfg.n_exp, world, rank), tuple(k for k in range(cfg.n_shared) if k % world == rank),
                   *split_even(cfg.vocab, world, rank))


def shard_ds_weights(w: dict[str, np.ndarray], cfg: DSConfig, sh: DSShard) -> dict[str, np.ndarray]:
    """This rank's slices (contiguous copies) of the full weights."""
    QS, DV, DI = cfg.d_nope + cfg.d_rope, cfg.d_v, cfg.dense_inter
    keep = list(range(sh.e0, sh.e1)) + [cfg.n_exp + k for k in sh.shared]
    c = np.ascontiguousarray
    out = {"embed": w["embed"], "norm_f": w["norm_f"], "lm_head": c(w["lm_head"][sh.v0:sh.v1])}
    for l in range(cfg.n_layers):
        p = f"l{l}."
        for k in ("attn_norm", "ffn_norm", "kv_norm", "router"):
            if p + k in w:
                out[p + k] = w[p + k]
        wq = w[p + "w_qkva"]
        out[p + "w_qkva"] = c(np.concatenate([wq[sh.h0 * QS:sh.h1 * QS], wq[cfg.q_cols:]]))
        out[p + "w_uk"], out[p + "w_uv"] = c(w[p + "w_uk"][sh.h0:sh.h1]), c(w[p + "w_uv"][sh.h0:sh.h1])
        out[p + "w_o"] = c(w[p + "w_o"][:, sh.h0 * DV:sh.h1 * DV])
        if l < cfg.n_dense:
            gu = w[p + "d_gu"]
            out[p + "d_gu"] = c(np.concatenate([gu[sh.f0:sh.f1], gu[DI + sh.f0:DI + sh.f1]]))
            out[p + "d_down"] = c(w[p + "d_down"][:, sh.f0:sh.f1])
        else:
            for k in ("e_gu", "e_gu_s", "e_d", "e_d_s"):
                out[p + k] = c(w[p + k][keep])
    return out


class DSModel:
    """One rank's part of the model on the current CUDA device (torch.distributed
    group over the R ranks, None when R = 1); `weights` are this rank's slices
    (shard_ds_weights)."""

    def __init__(self, cfg: DSConfig, weights: dict[str, np.ndarray], shard: DSShard, group=None,
                 n_slots: int | None = None):
        import torch
        self.torch, self.cfg, self.sh, self.group = torch, cfg, shard, group
        self.lib = L.lib()
        dev = torch.device("cuda", torch.cuda.current_device())
        B, D, ctx, Hl = cfg.batch, cfg.dim, cfg.max_ctx, shard.heads
        QS = cfg.d_nope + cfg.d_rope
        self.n_q = Hl * QS                               # local q columns of the fused projection
        self.n_qkva = self.n_q + cfg.kv_lora + cfg.d_rope
        DIl, Vl = shard.f1 - shard.f0, shard.v1 - shard.v0

        def put(a):
            t = torch.from_numpy(np.ascontiguousarray(a))
            if t.dtype == torch.uint16:
                t = t.view(torch.int16)
            return t.to(dev)

        self.w = {k: put(v) for k, v in weights.items()}
        cos, sin = yarn_tables(cfg.d_rope, ctx)
        self.cos, self.sin = put(cos), put(sin)
        z = lambda *s, dt=torch.float32: torch.zeros(*s, dtype=dt, device=dev)
        self.h = z(B, D)
        self.xn = z(B, max(D, DIl), dt=torch.int16)
        self.qkva = z(B, self.n_qkva)
        self.qo = z(B, max(self.n_q, 1), dt=torch.int16)
        self.o = z(B, max(Hl * cfg.d_v, 1), dt=torch.int16)
        self.gu = z(B, 2 * DIl)
        self.rl = z(B, cfg.n_exp)
        self.logits = z(B, Vl)
        self.n_slots = n_slots or B   # cache slots: one per row unless rows share them (use_rows)
        self.cache_c = [z(self.n_slots, ctx, cfg.kv_lora, dt=torch.int16) for _ in range(cfg.n_layers)]
        self.cache_pe = [z(self.n_slots, ctx, cfg.d_rope, dt=torch.int16) for _ in range(cfg.n_layers)]
        self.rows = None   # L.Sm100DsRows when rows carry their own slots and positions
        self.tok = z(B, dt=torch.int32)
        self.pos = z(1, dt=torch.int32)
        K = cfg.top_k
        self.sel, self.wsel = z(B * K, dt=torch.int32), z(B * K)
        self.route_counter = z(1, dt=torch.int32)   # the fused router + routing launch's CTA count
        n_local, ns = shard.e1 - shard.e0, len(shard.shared)
        # slot lists of the local routed experts, then the local shared halves (every token, weight 1)
        self.slot_off = z(n_local + ns + 1, dt=torch.int32)
        self.slot_tok, self.slot_w = z(B * (K + ns), dt=torch.int32), z(B * (K + ns))
        self.a = z(B * (K + ns), cfg.moe_inter, dt=torch.int16)
        self.vals, self.idxs = z(shard.world, B), z(shard.world, B, dt=torch.int32)
        # this rank's (max, index) per row; with one rank it is the gathered row itself
        self.val_me = self.vals[0] if shard.world == 1 else z(B)
        self.idx_me = self.idxs[0] if shard.world == 1 else z(B, dt=torch.int32)
        self.ws = z(int(self.lib.sm100_skinny_ws_bytes(B)) // 4)
        self.counters = z(max(Vl, self.n_qkva, 2 * DIl, D) // 128 + 2, dt=torch.int32)
        self._args = L.Sm100SkinnyArgs()
        self.launches = 0
        self.comm = None
        if shard.world > 1:
            from .comm import PeerComm
            self.comm = PeerComm(shard.rank, shard.world, D, group)
        self._pending = False   # h holds this rank's partial sums until the next norm's all-reduce

    def _stream(self):
        return ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)

    def _skinny(self, x, w, y, K, N, residual=False):
        a = self._args
        a.x, a.w, a.y = x.data_ptr(), w.data_ptr(), y.data_ptr()
        a.bias = None
        a.residual = y.data_ptr() if residual else None
        a.ws, a.counters, a.kv_cache, a.pos = self.ws.data_ptr(), self.counters.data_ptr(), None, None
        a.M, a.N, a.K = self.cfg.batch, N, K
        a.ld_x = a.ld_w = a.ld_res = a.ld_y = 0
        a.flags, a.kv_ctx = L.SK_RESIDUAL if residual else 0, 0
        a.ln_g = a.ln_b = None
        L.check(self.lib.sm100_skinny_bf16(ctypes.byref(a), self._stream()), "skinny")
        self.launches += 1

    def _rms(self, g, D, zero_rest=False):
        """xn = bf16(rms(h) * g); when h holds partial sums, the all-reduce
        over the ranks is fused into the same kernel (zero_rest: ranks other
        than 0 keep zeros in h, for partial sums that accumulate into it)."""
        if self._pending:
            self.comm.allreduce_rmsnorm(self.h.data_ptr(), g.data_ptr(), self.xn.data_ptr(), self.cfg.batch, D,
                                        self.cfg.eps, self._stream(), zero_rest)
            self._pending = False
        else:
            L.check(self.lib.sm100_ds_rmsnorm(self.h.data_ptr(), g.data_ptr(), self.xn.data_ptr(), self.cfg.batch, D,
                                              self.cfg.eps, self._stream()), "ds_rmsnorm")
        self.launches += 1

    def _all_reduce(self):
        self._pending = self.sh.world > 1

    def use_rows(self, row_pos, row_seq, shared_slots: bool):
        """From now on row b reads and appends cache slot row_seq[b] at
        position row_pos[b] (int32 device tensors [batch], kept by the
        caller, read by every step); the step leaves the positions alone.
        shared_slots: rows may share a slot (speculative verify rows)."""
        self._row_bufs = (row_pos, row_seq)
        r = L.Sm100DsRows()
        r.pos, r.seq, r.n_seq, r.shared_slots = row_pos.data_ptr(), row_seq.data_ptr(), self.n_slots, int(shared_slots)
        self.rows = r

    def status(self) -> int:
        """The kernels' sticky status words (non-zero: a bounded wait gave up or an
        expert met more than 32 slots); synchronises the device and clears them."""
        s = int(self.lib.sm100_ds_status())
        return s | (int(self.comm.status()) << 8 if self.comm is not None else 0)

    def close(self):
        if self.comm is not None:
            self.comm.close()
            self.comm = None

    def step(self):
        """One decode step: ids in self.tok at row self.pos -> next ids, pos + 1
        (after use_rows: each row at its own slot and position, which the step
        leaves unchanged)."""
        cfg, sh, w, lib, st = self.cfg, self.sh, self.w, self.lib, self._stream
        B, D, KV, DN, DR, DV = cfg.batch, cfg.dim, cfg.kv_lora, cfg.d_nope, cfg.d_rope, cfg.d_v
        E, K, I, Hl = cfg.n_exp, cfg.top_k, cfg.moe_inter, sh.heads
        DIl, Vl, first = sh.f1 - sh.f0, sh.v1 - sh.v0, sh.rank == 0
        L.check(lib.sm100_ds_embed(w["embed"].data_ptr(), self.tok.data_ptr(), self.h.data_ptr(), B, cfg.vocab, D,
                                   st()), "ds_embed")
        self.launches += 1
        for l in range(cfg.n_layers):
            p = f"l{l}."
            self._rms(w[p + "attn_norm"], D)
            self._skinny(self.xn, w[p + "w_qkva"], self.qkva, D, self.n_qkva)
            # q / latent post-processing (rotary, latent norm, cache append) and the absorbed MLA:
            # one launch for the DeepSeek-V2-Lite shapes, two otherwise
            mla_args = (self.qo.data_ptr(), w[p + "w_uk"].data_ptr(), w[p + "w_uv"].data_ptr(),
                        self.cache_c[l].data_ptr(), self.cache_pe[l].data_ptr(), self.o.data_ptr(), B, Hl, DN, DR, DV,
                        KV, cfg.max_ctx, cfg.eps, cfg.scale, st())
            if self.rows is None:
                L.check(lib.sm100_ds_mla_post(self.qkva.data_ptr(), self.n_qkva, self.n_q, w[p + "kv_norm"].data_ptr(),
                                              self.cos.data_ptr(), self.sin.data_ptr(), self.pos.data_ptr(), *mla_args),
                        "ds_mla_post")
            else:
                L.check(lib.sm100_ds_mla_post_rows(self.qkva.data_ptr(), self.n_qkva, self.n_q,
                                                   w[p + "kv_norm"].data_ptr(), self.cos.data_ptr(), self.sin.data_ptr(),
                                                   ctypes.byref(self.rows), *mla_args), "ds_mla_post_rows")
            fused = KV == 512 and DR == 64 and DN <= 128 and DV <= 128 and not (self.rows and self.rows.shared_slots)
            self.launches += 1 if fused else 2
            # the o projection's partial sums: rank 0 into the residual, the others over it
            self._skinny(self.o, w[p + "w_o"], self.h, Hl * DV, D, residual=first)
            self._all_reduce()
            # the experts add into h: on ranks other than 0 it must start from zero
            self._rms(w[p + "ffn_norm"], D, zero_rest=l >= cfg.n_dense)
            if l < cfg.n_dense:
                self._skinny(self.xn, w[p + "d_gu"], self.gu, D, 2 * DIl)
                L.check(lib.sm100_ds_silu_mul(self.gu.data_ptr(), self.xn.data_ptr(), B, DIl, st()), "ds_silu_mul")
                self.launches += 1
                self._skinny(self.xn, w[p + "d_down"], self.h, DIl, D, residual=first)
                self._all_reduce()
                continue
            ns = len(sh.shared)
            # the router product and the routing in one launch
            L.check(lib.sm100_ds_router_route(self.xn.data_ptr(), w[p + "router"].data_ptr(), self.rl.data_ptr(),
                                              self.route_counter.data_ptr(), D, E, K, B, sh.e0, sh.e1, ns,
                                              self.sel.data_ptr(), self.wsel.data_ptr(), self.slot_off.data_ptr(),
                                              self.slot_tok.data_ptr(), self.slot_w.data_ptr(), st()),
                    "ds_router_route")
            self.launches += 1
            # one launch pair over the local routed experts and shared halves (contiguous in this rank's
            # arrays), adding into the residual on rank 0 and into the zeros the all-reduce left in h on
            # the others
            L.check(lib.sm100_ds_experts(self.xn.data_ptr(), w[p + "e_gu"].data_ptr(), w[p + "e_gu_s"].data_ptr(),
                                         w[p + "e_d"].data_ptr(), w[p + "e_d_s"].data_ptr(), self.slot_off.data_ptr(),
                                         self.slot_tok.data_ptr(), self.slot_w.data_ptr(), self.a.data_ptr(),
                                         self.h.data_ptr(), sh.e1 - sh.e0 + ns, D, I, st()), "ds_experts")
            self.launches += 2
            self._all_reduce()
        self._rms(w["norm_f"], D)
        self._skinny(self.xn, w["lm_head"], self.logits, D, Vl)
        L.check(lib.sm100_xl_argmax(self.logits.data_ptr(), Vl, B, Vl, self.val_me.data_ptr(), self.idx_me.data_ptr(),
                                    sh.v0, 0, st()), "xl_argmax")
        self.launches += 1
        if sh.world > 1:
            self.comm.pick(self.val_me.data_ptr(), self.idx_me.data_ptr(), B, self.tok.data_ptr(), st())
        else:
            L.check(lib.sm100_xl_pick(self.vals.data_ptr(), self.idxs.data_ptr(), 1, B, self.tok.data_ptr(), st()),
                    "xl_pick")
        self.launches += 1
        if self.rows is None:
            L.check(lib.sm100_pos_add(self.pos.data_ptr(), 1, st()), "pos_add")
            self.launches += 1
