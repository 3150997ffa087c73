"""Batched bf16 decode of a GPT-2-XL-shaped model on the
sm_100a kernels, tensor-parallel over the GPUs of one box.

The model is bench/gpt2/thvm_gpt2.py:27-128 (Transformer / TransformerBlock /
Attention / FeedForward) with bf16 weights and a batch of B sequences decoded
in lockstep: per step, per layer

    x = bf16(ln_1(h)); qkv = x W_attn^T + b   (k, v -> the bf16 cache row pos)
    a = bf16(attention(q, cache[0..pos]));  h += a W_proj^T + b
    x = bf16(ln_2(h)); g = bf16(gelu(x W_fc^T + b));  h += g W_p2^T + b

then logits = bf16(ln_f(h)) W_lm^T and the next ids = row argmax.  The
numerics are those of oracle.XLModel (oracle.c orc_xl_step).

Tensor parallelism (Megatron): rank r of R holds a contiguous group of heads
(25 heads split as evenly as possible: c_attn column rows of its q, k and v,
c_proj the matching input columns), a slice of the MLP hidden units (c_fc
rows, mlp c_proj columns) and a slice of the vocabulary (lm_head rows).  The
row-split projections leave partial sums: rank 0 adds bias and residual in
its GEMM epilogue, the others overwrite their copy of h with their partial,
and one all-reduce (sum) per block restores the same h everywhere: the
library's peer-memory kernel fused with the LayerNorm that consumes h
(thvm_b200/comm.py, sm100_comm_allreduce_layernorm: the ranks' rows summed
in rank order).  The token pick gathers each rank's (max, index) pair over
peer memory and takes the largest (ties: smaller index).  PyTorch provides
device memory, the stream and CUDA graphs, and torch.distributed exchanges
the IPC handles at set-up; every kernel and collective of a step is the
library's.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib as L

HEAD_DIM = 64


@dataclass(frozen=True)
class XLConfig:
    n_layers: int = 48
    dim: int = 1600
    heads: int = 25
    vocab: int = 50257
    max_ctx: int = 1024
    batch: int = 16
    norm_eps: float = 1e-5

    @property
    def hidden(self) -> int:
        return 4 * self.dim


GPT2_XL = XLConfig()


def split_even(n: int, parts: int, r: int) -> tuple[int, int]:
    """Contiguous range [lo, hi) of part r when n items are split as evenly as
    possible (the first n % parts parts get one more)."""
    base, rem = divmod(n, parts)
    lo = r * base + min(r, rem)
    return lo, lo + base + (1 if r < rem else 0)


def _bf16(a: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bits, round to nearest even (finite values)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def xl_weights(cfg: XLConfig, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Synthetic weights in get_state_dict order: matrices and embeddings
    N(0, std) stored as bf16 bits, biases N(0, std) f32, LayerNorm gamma 1 /
    beta 0."""
    rng = np.random.default_rng(seed)
    D, F, V = cfg.dim, cfg.hidden, cfg.vocab

    def mat(*shape):
        return _bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))

    def vec(n):
        return rng.standard_normal(n, dtype=np.float32) * np.float32(std)

    w = {"wte": mat(V, D), "wpe": mat(cfg.max_ctx, D)}
    for i in range(cfg.n_layers):
        p = f"h.{i}."
        w[p + "ln_1.w"], w[p + "ln_1.b"] = np.ones(D, np.float32), np.zeros(D, np.float32)
        w[p + "attn.w"], w[p + "attn.b"] = mat(3 * D, D), vec(3 * D)
        w[p + "proj.w"], w[p + "proj.b"] = mat(D, D), vec(D)
        w[p + "ln_2.w"], w[p + "ln_2.b"] = np.ones(D, np.float32), np.zeros(D, np.float32)
        w[p + "fc.w"], w[p + "fc.b"] = mat(F, D), vec(F)
        w[p + "p2.w"], w[p + "p2.b"] = mat(D, F), vec(D)
    w["ln_f.w"], w["ln_f.b"] = np.ones(D, np.float32), np.zeros(D, np.float32)
    w["lm_head"] = mat(V, D)
    return w


@dataclass(frozen=True)
class Shard:
    """What rank r of R holds: heads [h0, h1), hidden units [f0, f1), vocab [v0, v1)."""
    rank: int
    world: int
    h0: int
    h1: int
    f0: int
    f1: int
    v0: int
    v1: int

    @property
    def cols(self) -> int:   # this rank's attention width (heads * 64)
        return (self.h1 - self.h0) * HEAD_DIM


def shard_of(cfg: XLConfig, rank: int, world: int) -> Shard:
    if not 0 <= rank < world or cfg.heads < world:
        raise ValueError(f"rank {rank} of {world} (heads {cfg.heads})")
    return Shard(rank, world, *split_even(cfg.heads, world, rank), *split_even(cfg.hidden, world, rank),
                 *split_even(cfg.vocab, world, rank))


def shard_weights(w: dict[str, np.ndarray], cfg: XLConfig, sh: Shard) -> dict[str, np.ndarray]:
    """This rank's slices (contiguous copies) of the full weights."""
    D = cfg.dim
    c = slice(sh.h0 * HEAD_DIM, sh.h1 * HEAD_DIM)
    f = slice(sh.f0, sh.f1)
    out = {"wte": w["wte"], "wpe": w["wpe"], "ln_f.w": w["ln_f.w"], "ln_f.b": w["ln_f.b"],
           "lm_head": np.ascontiguousarray(w["lm_head"][sh.v0:sh.v1])}
    for i in range(cfg.n_layers):
        p = f"h.{i}."
        wa, ba = w[p + "attn.w"], w[p + "attn.b"]
        out[p + "attn.w"] = np.ascontiguousarray(np.concatenate([wa[c], wa[D:][c], wa[2 * D:][c]]))
        out[p + "attn.b"] = np.ascontiguousarray(np.concatenate([ba[c], ba[D:][c], ba[2 * D:][c]]))
        out[p + "proj.w"] = np.ascontiguousarray(w[p + "proj.w"][:, c])
        out[p + "fc.w"] = np.ascontiguousarray(w[p + "fc.w"][f])
        out[p + "fc.b"] = np.ascontiguousarray(w[p + "fc.b"][f])
        out[p + "p2.w"] = np.ascontiguousarray(w[p + "p2.w"][:, f])
        for k in ("ln_1.w", "ln_1.b", "ln_2.w", "ln_2.b", "proj.b", "p2.b"):
            out[p + k] = w[p + k]
    return out


class XLModel:
    """One rank's part of the model on the current CUDA device.  `group` is a
    torch.distributed process group over the R ranks (None when R = 1)."""

    def __init__(self, cfg: XLConfig, weights: dict[str, np.ndarray], shard: Shard, group=None):
        import torch
        self.torch, self.cfg, self.sh, self.group = torch, cfg, shard, group
        self.lib = L.lib()
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        B, D, ctx = cfg.batch, cfg.dim, cfg.max_ctx
        C, Fl, Vl = shard.cols, shard.f1 - shard.f0, shard.v1 - shard.v0

        def put(a):
            t = torch.from_numpy(np.ascontiguousarray(a))
            if t.dtype == torch.uint16:
                t = t.view(torch.int16)
            return t.to(dev)

        self.w = {k: put(v) for k, v in weights.items()}
        z = lambda *s, dt=torch.float32: torch.zeros(*s, dtype=dt, device=dev)
        self.h = z(B, D)
        self.xa = z(B, D, dt=torch.int16)          # bf16 LayerNorm outputs
        self.qkv = z(B, 3 * C)
        self.att = z(B, C, dt=torch.int16)
        self.g = z(B, Fl, dt=torch.int16)            # bf16 gelu(c_fc)
        self.logits = z(B, Vl)
        self.kv = [z(2, B, ctx, C, dt=torch.int16) for _ in range(cfg.n_layers)]
        self.tok = z(B, dt=torch.int32)
        self.pos = z(1, dt=torch.int32)
        self.vals = z(shard.world, B)
        self.idxs = z(shard.world, B, dt=torch.int32)
        # this rank's (max, index) per row; with one rank it is the gathered row itself
        self.val_me = self.vals[0] if shard.world == 1 else z(B)
        self.idx_me = self.idxs[0] if shard.world == 1 else z(B, dt=torch.int32)
        self.ws = z(int(self.lib.sm100_skinny_ws_bytes(B)) // 4)
        self.counters = z(max(3 * C, Fl, D, Vl) // 128 + 1, dt=torch.int32)
        self._args = L.Sm100SkinnyArgs()
        self.launches = 0
        self.comm = None
        if shard.world > 1:
            from .comm import PeerComm
            self.comm = PeerComm(shard.rank, shard.world, D, group)
        self._pending = False   # h holds this rank's partial sums until the next LayerNorm's all-reduce
        self._pf = None         # the prompt pass's buffers (for one prompt length)

    # -- one launcher per kernel ------------------------------------------------
    def _stream(self):
        return ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)

    def _skinny(self, x, w, y, K, N, bias=None, residual=None, flags=0, kv=None, ln=None):
        a = self._args
        a.x, a.w, a.y = x.data_ptr(), w.data_ptr(), y.data_ptr()
        a.bias = bias.data_ptr() if bias is not None else None
        a.residual = residual.data_ptr() if residual is not None else None
        a.ws, a.counters = self.ws.data_ptr(), self.counters.data_ptr()
        a.kv_cache = kv.data_ptr() if kv is not None else None
        a.pos = self.pos.data_ptr() if kv is not None else None
        a.M, a.N, a.K = self.cfg.batch, N, K
        a.ld_x = a.ld_w = a.ld_res = a.ld_y = 0
        a.flags, a.kv_ctx = flags, self.cfg.max_ctx
        if ln is not None:   # the operand is bf16(LayerNorm(x)), computed inside the GEMM
            a.flags |= L.SK_X_LN
            a.ln_g, a.ln_b, a.eps = ln[0].data_ptr(), ln[1].data_ptr(), self.cfg.norm_eps
        else:
            a.ln_g = a.ln_b = None
        L.check(self.lib.sm100_skinny_bf16(ctypes.byref(a), self._stream()), "skinny")
        self.launches += 1

    def _ln(self, g, b, zero_h=False, zero_buf=None):
        """xa = bf16(LayerNorm(h) * g + b); when h holds partial sums, the
        all-reduce over the ranks is fused into the same kernel (peer memory)."""
        if self._pending:
            self.comm.allreduce_layernorm(self.h.data_ptr(), g.data_ptr(), b.data_ptr(), self.xa.data_ptr(),
                                          self.cfg.batch, self.cfg.dim, self.cfg.norm_eps, self._stream())
            self._pending = False
            self.launches += 1
            return
        zp, zn = (zero_buf.data_ptr(), zero_buf.numel()) if zero_buf is not None else (None, 0)
        L.check(self.lib.sm100_xl_layernorm(self.h.data_ptr(), g.data_ptr(), b.data_ptr(), self.xa.data_ptr(),
                                            self.cfg.batch, self.cfg.dim, self.cfg.norm_eps, 1 if zero_h else 0,
                                            zp, zn, self._stream()),
                "xl_layernorm")
        self.launches += 1

    def _all_reduce(self, t):
        self._pending = self.sh.world > 1

    def close(self):
        if self.comm is not None:
            self.comm.close()
            self.comm = None

    def step(self):
        """One decode step: ids in self.tok at row self.pos -> next ids in self.tok, pos + 1."""
        cfg, sh, w, lib = self.cfg, self.sh, self.w, self.lib
        B, D, C, Fl = cfg.batch, cfg.dim, sh.cols, sh.f1 - sh.f0
        first = sh.rank == 0
        res = L.SK_RESIDUAL if first else 0
        L.check(lib.sm100_xl_embed(w["wte"].data_ptr(), w["wpe"].data_ptr(), self.tok.data_ptr(), self.pos.data_ptr(),
                                   self.h.data_ptr(), B, cfg.vocab, D, self._stream()), "xl_embed")
        self.launches += 1
        scale = 1.0 / np.sqrt(HEAD_DIM)
        for i in range(cfg.n_layers):
            p = f"h.{i}."
            self._ln(w[p + "ln_1.w"], w[p + "ln_1.b"])
            self._skinny(self.xa, w[p + "attn.w"], self.qkv, D, 3 * C, bias=w[p + "attn.b"], flags=L.SK_KV,
                         kv=self.kv[i])
            L.check(lib.sm100_xl_attention(self.qkv.data_ptr(), 3 * C, self.kv[i].data_ptr(), self.pos.data_ptr(),
                                           self.att.data_ptr(), B, sh.h1 - sh.h0, HEAD_DIM, cfg.max_ctx, scale, 0,
                                           self._stream()), "xl_attention")
            self.launches += 1
            # row-split: rank 0 adds bias + residual, the others leave their partial in h
            self._skinny(self.att, w[p + "proj.w"], self.h, C, D, bias=w[p + "proj.b"] if first else None,
                         residual=self.h if first else None, flags=res)
            self._all_reduce(self.h)
            self._ln(w[p + "ln_2.w"], w[p + "ln_2.b"])
            self._skinny(self.xa, w[p + "fc.w"], self.g, D, Fl, bias=w[p + "fc.b"], flags=L.SK_GELU | L.SK_OUT_BF16)
            self._skinny(self.g, w[p + "p2.w"], self.h, Fl, D, bias=w[p + "p2.b"] if first else None,
                         residual=self.h if first else None, flags=res)
            self._all_reduce(self.h)
        self._head()
        L.check(lib.sm100_pos_add(self.pos.data_ptr(), 1, self._stream()), "pos_add")
        self.launches += 1

    def _head(self):
        """ln_f, lm_head and the token pick of the B rows in self.h -> self.tok."""
        cfg, sh, w, lib = self.cfg, self.sh, self.w, self.lib
        B, D = cfg.batch, cfg.dim
        self._ln(w["ln_f.w"], w["ln_f.b"])
        Vl = sh.v1 - sh.v0
        self._skinny(self.xa, w["lm_head"], self.logits, D, Vl)
        L.check(lib.sm100_xl_argmax(self.logits.data_ptr(), Vl, B, Vl, self.val_me.data_ptr(),
                                    self.idx_me.data_ptr(), sh.v0, 0, self._stream()), "xl_argmax")
        self.launches += 1
        if sh.world > 1:
            self.comm.pick(self.val_me.data_ptr(), self.idx_me.data_ptr(), B, self.tok.data_ptr(), self._stream())
        else:
            L.check(lib.sm100_xl_pick(self.vals.data_ptr(), self.idxs.data_ptr(), 1, B, self.tok.data_ptr(),
                                      self._stream()), "xl_pick")
        self.launches += 1

    # -- the prompt pass ----------------------------------------------------------
    def _gemm(self, a, wt, c, M, N, K, bias=None, residual=None, flags=0):
        L.check(self.lib.sm100_gemm_bf16_ep(a.data_ptr(), wt.data_ptr(), c.data_ptr(), M, N, K,
                                            bias.data_ptr() if bias is not None else None,
                                            residual.data_ptr() if residual is not None else None, flags,
                                            self._stream()), "gemm_bf16_ep")
        self.launches += 1

    def _prefill_bufs(self, P: int) -> dict:
        if self._pf is not None and self._pf["P"] == P:
            return self._pf
        torch, cfg, sh = self.torch, self.cfg, self.sh
        B, D, C, Fl, H, M = cfg.batch, cfg.dim, sh.cols, sh.f1 - sh.f0, sh.h1 - sh.h0, cfg.batch * P
        z = lambda *s, dt=torch.int16: torch.zeros(*s, dtype=dt, device=self.dev)
        self._pf = dict(P=P, tok=z(M, dt=torch.int32), h=z(M, D, dt=torch.float32), x=z(M, D), qkv=z(M, 3 * C),
                        q=z(B, H, P, 128), k=z(B, H, P, 128), v=z(B, H, P, 128),   # columns 64.. stay zero
                        o=z(B, H, P, 128, dt=torch.float32), att=z(M, C), g=z(M, Fl))
        return self._pf

    def prefill(self, prompts: np.ndarray):
        """The prompt pass (thvm_gpt2.py:98-128 with start_pos 0): prompts
        [B, P] ids, all P positions of every sequence through each layer at
        once (the projections on the tcgen05 GEMM with fused epilogues, the
        causal attention on the tcgen05 prefill kernel).  Afterwards the cache
        holds rows 0..P-1, self.tok the ids picked from each sequence's last
        position and pos = P: the state P decode steps fed the prompt leave.
        Same numerics as step() up to f32 summation order, except that q is
        rounded to bf16 for the attention product."""
        self.prefill_ids(prompts)
        self.prefill_run(prompts.shape[1])

    def prefill_ids(self, prompts: np.ndarray):
        """Copies prompts [B, P] into the prompt pass's id buffer."""
        cfg = self.cfg
        prompts = np.ascontiguousarray(prompts, np.int32)
        if prompts.ndim != 2 or prompts.shape[0] != cfg.batch or not 1 <= prompts.shape[1] < cfg.max_ctx:
            raise ValueError(f"prompts of shape {prompts.shape}: want [{cfg.batch}, P] with 1 <= P < {cfg.max_ctx}")
        self._prefill_bufs(prompts.shape[1])["tok"].copy_(self.torch.from_numpy(prompts.reshape(-1)))

    def prefill_run(self, P: int):
        """The launches of the prompt pass over the ids prefill_ids() copied
        (device work only: a CUDA graph can capture it)."""
        torch, cfg, sh, w, lib = self.torch, self.cfg, self.sh, self.w, self.lib
        B, D, C, Fl, H = cfg.batch, cfg.dim, sh.cols, sh.f1 - sh.f0, sh.h1 - sh.h0
        M = B * P
        f = self._pf
        if f is None or f["P"] != P:
            raise ValueError(f"prefill_run({P}) without prefill_ids of P = {P} ids")
        first = sh.rank == 0
        st = self._stream
        L.check(lib.sm100_xl_prefill_embed(w["wte"].data_ptr(), w["wpe"].data_ptr(), f["tok"].data_ptr(),
                                           f["h"].data_ptr(), B, P, cfg.vocab, D, st()), "xl_prefill_embed")
        self.launches += 1
        h, x = f["h"], f["x"]

        def ln(g, b):
            L.check(lib.sm100_xl_prefill_layernorm(h.data_ptr(), g.data_ptr(), b.data_ptr(), x.data_ptr(), M, D,
                                                   cfg.norm_eps, st()), "xl_prefill_layernorm")
            self.launches += 1

        def reduce_rows():   # row-split partial sums -> the full sums on every rank
            if sh.world > 1:
                torch.distributed.all_reduce(h, group=self.group)

        for i in range(cfg.n_layers):
            p = f"h.{i}."
            ln(w[p + "ln_1.w"], w[p + "ln_1.b"])
            self._gemm(x, w[p + "attn.w"], f["qkv"], M, 3 * C, D, bias=w[p + "attn.b"], flags=L.GEMM_OUT_BF16)
            L.check(lib.sm100_xl_prefill_split(f["qkv"].data_ptr(), f["q"].data_ptr(), f["k"].data_ptr(),
                                               f["v"].data_ptr(), self.kv[i].data_ptr(), B, P, H, cfg.max_ctx, st()),
                    "xl_prefill_split")
            L.check(lib.sm100_attn_prefill_bf16(f["q"].data_ptr(), f["k"].data_ptr(), f["v"].data_ptr(),
                                                f["o"].data_ptr(), B, H, P, 128, 1.0 / np.sqrt(HEAD_DIM), 1, st()),
                    "attn_prefill")
            L.check(lib.sm100_xl_prefill_merge(f["o"].data_ptr(), f["att"].data_ptr(), B, P, H, st()),
                    "xl_prefill_merge")
            self.launches += 3
            # row-split: rank 0 adds bias + residual, the others leave their partial in h
            self._gemm(f["att"], w[p + "proj.w"], h, M, D, C, bias=w[p + "proj.b"] if first else None,
                       residual=h if first else None)
            reduce_rows()
            ln(w[p + "ln_2.w"], w[p + "ln_2.b"])
            self._gemm(x, w[p + "fc.w"], f["g"], M, Fl, D, bias=w[p + "fc.b"], flags=L.GEMM_GELU | L.GEMM_OUT_BF16)
            self._gemm(f["g"], w[p + "p2.w"], h, M, D, Fl, bias=w[p + "p2.b"] if first else None,
                       residual=h if first else None)
            reduce_rows()
        L.check(lib.sm100_xl_prefill_last(h.data_ptr(), self.h.data_ptr(), self.pos.data_ptr(), B, P, D, st()),
                "xl_prefill_last")
        self.launches += 1
        self._head()
