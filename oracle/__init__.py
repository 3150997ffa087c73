"""CPU oracle (test infrastructure only).

ctypes bindings over oracle/liboracle.so (our C restatement of the reference's
CPU arithmetic, oracle.c) and, for the timed reference arm, oracle/_ref (the
reference's own CPU path compiled from its sources).  Only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
import this package; the product (thvm_b200/) never does.
"""
from __future__ import annotations

import ctypes
import math
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64 = ctypes.c_int64
_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.orc_linear_f32.argtypes = [_f32p, _f32p, ctypes.c_void_p, _f32p, _i64, _i64, _i64]
        L.orc_layernorm_f32.argtypes = [_f32p, ctypes.c_void_p, ctypes.c_void_p, _f32p, _i64,
                                        _i64, ctypes.c_float]
        L.orc_rmsnorm_f32.argtypes = [_f32p, ctypes.c_void_p, _f32p, _i64, _i64, ctypes.c_float]
        L.orc_softmax_f32.argtypes = [_f32p, _f32p, _i64, _i64]
        L.orc_gelu_f32.argtypes = [_f32p, _f32p, _i64]
        L.orc_sdpa_f32.argtypes = [_f32p, _f32p, _f32p, ctypes.c_void_p, _f32p, _i64, _i64, _i64,
                                   _i64, ctypes.c_int]
        L.orc_argmax_f32.argtypes = [_f32p, _i32p, _i64, _i64]
        L.orc_embedding_f32.argtypes = [_f32p, _i32p, _f32p, _i64, _i64, _i64]
        L.orc_gpt2_state_new.restype = ctypes.c_void_p
        L.orc_gpt2_state_new.argtypes = [ctypes.c_void_p]
        L.orc_gpt2_state_free.argtypes = [ctypes.c_void_p]
        L.orc_gpt2_forward.restype = ctypes.c_int32
        L.orc_gpt2_forward.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_void_p]
        L.orc_gpt2_generate.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int32, ctypes.c_int32,
                                        _i32p]
        L.orc_num_threads.restype = ctypes.c_int
        _u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
        _u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
        L.orc_f32_to_bf16_n.argtypes = [_f32p, _u16p, _i64]
        L.orc_f32_to_fp8e4m3_n.argtypes = [_f32p, _u8p, _i64]
        L.orc_fp8e4m3_to_f32.restype = ctypes.c_float
        L.orc_fp8e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.orc_linear_bf16.argtypes = [_f32p, _u16p, _f32p, _i64, _i64, _i64]
        L.orc_linear_fp8bs.argtypes = [_f32p, _u8p, _f32p, _f32p, _i64, _i64, _i64]
        L.orc_gemm_bf16.argtypes = [_u16p, _u16p, _f32p, _i64, _i64, _i64]
        L.orc_ds_route.argtypes = [_f32p, _i64, _i64, _i64, _i32p, _f32p]
        _lib = L
    return _lib


def _c(a, dt=np.float32):
    return np.ascontiguousarray(a, dtype=dt)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def linear(x, w, b=None):
    x, w = _c(x), _c(w)
    b = None if b is None else _c(b)
    K = x.shape[-1]
    N = w.shape[0]
    M = x.size // K
    y = np.empty(x.shape[:-1] + (N,), np.float32)
    lib().orc_linear_f32(x, w, _ptr(b), y, M, K, N)
    return y


def layernorm(x, g=None, b=None, eps=1e-5):
    x = _c(x)
    g = None if g is None else _c(g)
    b = None if b is None else _c(b)
    y = np.empty_like(x)
    D = x.shape[-1]
    lib().orc_layernorm_f32(x, _ptr(g), _ptr(b), y, x.size // D, D, eps)
    return y


def rmsnorm(x, g=None, eps=1e-6):
    x = _c(x)
    g = None if g is None else _c(g)
    y = np.empty_like(x)
    D = x.shape[-1]
    lib().orc_rmsnorm_f32(x, _ptr(g), y, x.size // D, D, eps)
    return y


def softmax(x):
    x = _c(x)
    y = np.empty_like(x)
    lib().orc_softmax_f32(x, y, x.size // x.shape[-1], x.shape[-1])
    return y


def gelu(x):
    x = _c(x)
    y = np.empty_like(x)
    lib().orc_gelu_f32(x, y, x.size)
    return y


def sdpa(q, k, v, mask=None, causal=False):
    q, k, v = _c(q), _c(k), _c(v)
    Lq, D = q.shape[-2:]
    Lk = k.shape[-2]
    BH = q.size // (Lq * D)
    m = None if mask is None else _c(np.broadcast_to(mask, mask.shape[:-2] + (Lq, Lk)).reshape(-1, Lq, Lk)[0])
    y = np.empty_like(q)
    lib().orc_sdpa_f32(q, k, v, _ptr(m), y, BH, Lq, Lk, D, 1 if causal else 0)
    return y


def argmax(x):
    x = _c(x)
    N = x.shape[-1]
    out = np.empty(x.shape[:-1], np.int32)
    lib().orc_argmax_f32(x, out, x.size // N, N)
    return out


def embedding(w, idx):
    w, idx = _c(w), _c(idx, np.int32)
    y = np.empty(idx.shape + (w.shape[1],), np.float32)
    lib().orc_embedding_f32(w, idx, y, idx.size, w.shape[0], w.shape[1])
    return y


def to_bf16(x):
    """f32 -> bf16 bits (uint16), the reference's f32_to_bf16."""
    x = _c(x)
    y = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_bf16_n(x.reshape(-1), y.reshape(-1), x.size)
    return y


def bf16_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def to_fp8e4m3(x):
    """f32 -> e4m3 codes (uint8), the reference's saturating kernel store."""
    x = _c(x)
    y = np.empty(x.shape, np.uint8)
    lib().orc_f32_to_fp8e4m3_n(x.reshape(-1), y.reshape(-1), x.size)
    return y


FP8E4M3_TABLE = None


def fp8e4m3_to_f32(b):
    global FP8E4M3_TABLE
    if FP8E4M3_TABLE is None:
        FP8E4M3_TABLE = np.array([lib().orc_fp8e4m3_to_f32(i) for i in range(256)], np.float32)
    return FP8E4M3_TABLE[np.asarray(b, np.uint8)]


def linear_bf16(x, w_bits):
    """y = x @ bf16(W)^T, W bits [N, K]."""
    x, w = _c(x), _c(w_bits, np.uint16)
    K, N = x.shape[-1], w.shape[0]
    y = np.empty(x.shape[:-1] + (N,), np.float32)
    lib().orc_linear_bf16(x, w, y, x.size // K, K, N)
    return y


def linear_fp8bs(x, w_codes, scale):
    """y = x @ (e4m3(W) * scale.repeat(128, 128))^T, W codes [N, K], scale [ceil(N/128), ceil(K/128)]."""
    x, w, s = _c(x), _c(w_codes, np.uint8), _c(scale)
    K, N = x.shape[-1], w.shape[0]
    y = np.empty(x.shape[:-1] + (N,), np.float32)
    lib().orc_linear_fp8bs(x, w, s, y, x.size // K, K, N)
    return y


def gemm_bf16(a_bits, b_bits):
    """C[M, N] = bf16(A)[M, K] @ bf16(B)[N, K]^T with f32 accumulate."""
    a, b = _c(a_bits, np.uint16), _c(b_bits, np.uint16)
    M, K = a.shape
    N = b.shape[0]
    c = np.empty((M, N), np.float32)
    lib().orc_gemm_bf16(a, b, c, M, N, K)
    return c


class _OrcGPT2(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("n_layers", "n_heads", "dim", "vocab", "max_ctx")] + [
        ("norm_eps", ctypes.c_float)] + [
        (n, ctypes.c_void_p) for n in ("wte", "wpe", "ln_f_w", "ln_f_b", "lm_head")] + [
        (n, ctypes.POINTER(ctypes.c_void_p)) for n in (
            "c_attn_w", "c_attn_b", "c_proj_w", "c_proj_b", "c_fc_w", "c_fc_b",
            "mlp_proj_w", "mlp_proj_b", "ln_1_w", "ln_1_b", "ln_2_w", "ln_2_b")]


class GPT2:
    """The oracle GPT-2 decoder over a synthetic state dict (numpy float32)."""

    _per_layer = {"c_attn_w": "attn.c_attn.weight", "c_attn_b": "attn.c_attn.bias",
                  "c_proj_w": "attn.c_proj.weight", "c_proj_b": "attn.c_proj.bias",
                  "c_fc_w": "mlp.c_fc.weight", "c_fc_b": "mlp.c_fc.bias",
                  "mlp_proj_w": "mlp.c_proj.weight", "mlp_proj_b": "mlp.c_proj.bias",
                  "ln_1_w": "ln_1.weight", "ln_1_b": "ln_1.bias",
                  "ln_2_w": "ln_2.weight", "ln_2_b": "ln_2.bias"}

    def __init__(self, cfg, weights: dict):
        self.cfg = cfg
        self._keep = {k: _c(v) for k, v in weights.items()}
        s = _OrcGPT2(n_layers=cfg.n_layers, n_heads=cfg.n_heads, dim=cfg.dim, vocab=cfg.vocab,
                     max_ctx=cfg.max_ctx, norm_eps=cfg.norm_eps)
        w = self._keep
        s.wte, s.wpe = _ptr(w["wte.weight"]), _ptr(w["wpe.weight"])
        s.ln_f_w, s.ln_f_b = _ptr(w["ln_f.weight"]), _ptr(w["ln_f.bias"])
        s.lm_head = _ptr(w["lm_head.weight"])
        self._arrays = []
        for field, suffix in self._per_layer.items():
            arr = (ctypes.c_void_p * cfg.n_layers)(
                *[w[f"h.{i}.{suffix}"].ctypes.data for i in range(cfg.n_layers)])
            self._arrays.append(arr)
            setattr(s, field, ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)))
        self._s = s
        self._state = lib().orc_gpt2_state_new(ctypes.byref(s))

    def forward(self, tokens, start_pos: int, want_logits: bool = False):
        t = _c(tokens, np.int32)
        lg = np.empty(self.cfg.vocab, np.float32) if want_logits else None
        tok = lib().orc_gpt2_forward(self._state, t, t.size, start_pos, _ptr(lg))
        if tok < 0:
            raise RuntimeError("orc_gpt2_forward failed")
        return (tok, lg) if want_logits else tok

    def generate(self, prompt, n_new: int):
        p = _c(prompt, np.int32)
        out = np.empty(n_new, np.int32)
        if lib().orc_gpt2_generate(ctypes.byref(self._s), p, p.size, n_new, out) != 0:
            raise RuntimeError("orc_gpt2_generate failed")
        return out

    def __del__(self):
        st = getattr(self, "_state", None)
        if st and _lib is not None:
            _lib.orc_gpt2_state_free(st)
            self._state = None


class _OrcXL(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("n_layers", "dim", "heads", "vocab", "max_ctx", "batch")] + [
        ("norm_eps", ctypes.c_float)] + [
        (n, ctypes.c_void_p) for n in ("wte", "wpe", "lm_head", "ln_f_w", "ln_f_b")] + [
        (n, ctypes.POINTER(ctypes.c_void_p)) for n in (
            "ln_1_w", "ln_1_b", "ln_2_w", "ln_2_b", "c_attn_w", "c_proj_w", "c_fc_w", "mlp_proj_w",
            "c_attn_b", "c_proj_b", "c_fc_b", "mlp_proj_b")] + [("exact", ctypes.c_int32)]


class XLModel:
    """The oracle's batched bf16 decode step (orc_xl_step) over the weight
    dict of thvm_b200.gpt2_xl.xl_weights (bf16 bits as uint16, f32 vectors)."""

    _per_layer = {"ln_1_w": "ln_1.w", "ln_1_b": "ln_1.b", "ln_2_w": "ln_2.w", "ln_2_b": "ln_2.b",
                  "c_attn_w": "attn.w", "c_proj_w": "proj.w", "c_fc_w": "fc.w", "mlp_proj_w": "p2.w",
                  "c_attn_b": "attn.b", "c_proj_b": "proj.b", "c_fc_b": "fc.b", "mlp_proj_b": "p2.b"}

    def __init__(self, cfg, weights: dict, exact: bool = False):
        """exact: no bf16 rounding of activations or cache rows (an f32 cache):
        the pinned f32 GPT-2 forward on the bf16-valued weights."""
        self.cfg = cfg
        self._keep = {k: np.ascontiguousarray(v) for k, v in weights.items()}
        w = self._keep
        s = _OrcXL(n_layers=cfg.n_layers, dim=cfg.dim, heads=cfg.heads, vocab=cfg.vocab, max_ctx=cfg.max_ctx,
                   batch=cfg.batch, norm_eps=cfg.norm_eps, exact=int(exact))
        s.wte, s.wpe, s.lm_head = w["wte"].ctypes.data, w["wpe"].ctypes.data, w["lm_head"].ctypes.data
        s.ln_f_w, s.ln_f_b = w["ln_f.w"].ctypes.data, w["ln_f.b"].ctypes.data
        self._arrays = []
        for field, suffix in self._per_layer.items():
            arr = (ctypes.c_void_p * cfg.n_layers)(*[w[f"h.{i}.{suffix}"].ctypes.data for i in range(cfg.n_layers)])
            self._arrays.append(arr)
            setattr(s, field, ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)))
        self._s = s
        self.kv = np.zeros((cfg.n_layers, 2, cfg.batch, cfg.max_ctx, cfg.dim), np.float32 if exact else np.uint16)
        L = lib()
        if not getattr(L, "_xl_bound", False):
            L.orc_xl_step.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                      ctypes.c_void_p, ctypes.c_void_p]
            L.orc_xl_step.restype = None
            L._xl_bound = True

    def step(self, tok, pos: int):
        """(logits [B, V], next ids [B]) of one decode step at row pos."""
        t = np.ascontiguousarray(tok, np.int32)
        lg = np.empty((self.cfg.batch, self.cfg.vocab), np.float32)
        nxt = np.empty(self.cfg.batch, np.int32)
        lib().orc_xl_step(ctypes.byref(self._s), self.kv.ctypes.data, t.ctypes.data, pos, lg.ctypes.data,
                          nxt.ctypes.data)
        return lg, nxt


class _OrcDS(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "dim", "n_layers", "heads", "kv_lora", "d_nope", "d_rope", "d_v", "n_exp", "top_k", "moe_inter",
        "dense_inter", "n_dense", "n_shared", "vocab", "max_ctx", "batch")] + [
        ("eps", ctypes.c_float), ("scale", ctypes.c_float)] + [
        (n, ctypes.c_void_p) for n in ("embed", "lm_head", "norm_f", "cos_t", "sin_t")] + [
        (n, ctypes.POINTER(ctypes.c_void_p)) for n in (
            "attn_norm", "kv_norm", "ffn_norm", "w_qkva", "w_uk", "w_uv", "w_o", "d_gu", "d_down", "router",
            "e_gu", "e_d", "e_gu_s", "e_d_s")]


class DSModel:
    """The oracle's batched MoE decode step (orc_ds_step) over the weight dict
    of thvm_b200.dsv2.ds_weights (bf16 bits uint16, fp8 codes uint8, f32)."""

    _per_layer = {"attn_norm": "attn_norm", "kv_norm": "kv_norm", "ffn_norm": "ffn_norm", "w_qkva": "w_qkva",
                  "w_uk": "w_uk", "w_uv": "w_uv", "w_o": "w_o", "d_gu": "d_gu", "d_down": "d_down",
                  "router": "router", "e_gu": "e_gu", "e_d": "e_d", "e_gu_s": "e_gu_s", "e_d_s": "e_d_s"}

    def __init__(self, cfg, weights: dict, cos_t, sin_t):
        self.cfg = cfg
        self._keep = {k: np.ascontiguousarray(v) for k, v in weights.items()}
        self._keep["cos"], self._keep["sin"] = np.ascontiguousarray(cos_t), np.ascontiguousarray(sin_t)
        w = self._keep
        s = _OrcDS(dim=cfg.dim, n_layers=cfg.n_layers, heads=cfg.heads, kv_lora=cfg.kv_lora, d_nope=cfg.d_nope,
                   d_rope=cfg.d_rope, d_v=cfg.d_v, n_exp=cfg.n_exp, top_k=cfg.top_k, moe_inter=cfg.moe_inter,
                   dense_inter=cfg.dense_inter, n_dense=cfg.n_dense, n_shared=cfg.n_shared, vocab=cfg.vocab,
                   max_ctx=cfg.max_ctx, batch=cfg.batch, eps=cfg.eps, scale=cfg.scale)
        s.embed, s.lm_head, s.norm_f = w["embed"].ctypes.data, w["lm_head"].ctypes.data, w["norm_f"].ctypes.data
        s.cos_t, s.sin_t = w["cos"].ctypes.data, w["sin"].ctypes.data
        self._arrays = []
        for field, suffix in self._per_layer.items():
            ptrs = [w[f"l{i}.{suffix}"].ctypes.data if f"l{i}.{suffix}" in w else None for i in range(cfg.n_layers)]
            arr = (ctypes.c_void_p * cfg.n_layers)(*ptrs)
            self._arrays.append(arr)
            setattr(s, field, ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)))
        self._s = s
        self.cache_c = np.zeros((cfg.n_layers, cfg.batch, cfg.max_ctx, cfg.kv_lora), np.uint16)
        self.cache_pe = np.zeros((cfg.n_layers, cfg.batch, cfg.max_ctx, cfg.d_rope), np.uint16)
        L = lib()
        if not getattr(L, "_ds_bound", False):
            L.orc_ds_step.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
            L.orc_ds_step.restype = None
            L._ds_bound = True

    def step(self, tok, pos: int):
        t = np.ascontiguousarray(tok, np.int32)
        lg = np.empty((self.cfg.batch, self.cfg.vocab), np.float32)
        nxt = np.empty(self.cfg.batch, np.int32)
        lib().orc_ds_step(ctypes.byref(self._s), self.cache_c.ctypes.data, self.cache_pe.ctypes.data, t.ctypes.data,
                          pos, lg.ctypes.data, nxt.ctypes.data)
        return lg, nxt


def ds_route(logits, k: int):
    """(sel [B, k], probs [B, k]) of orc_ds_route: the reference's top-k-of-logits rule."""
    g = _c(np.atleast_2d(logits))
    B, E = g.shape
    sel, pr = np.empty((B, k), np.int32), np.empty((B, k), np.float32)
    lib().orc_ds_route(g, B, E, k, sel, pr)
    return sel, pr


class _OrcDSRef(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "dim", "n_layers", "heads", "kv_lora", "d_nope", "d_rope", "d_v", "n_exp", "n_shared", "top_k", "moe_inter",
        "dense_inter", "first_dense", "vocab", "max_seq")] + [
        ("eps", ctypes.c_float), ("scale", ctypes.c_float)] + [
        (n, ctypes.c_void_p) for n in ("embed", "lm_head", "norm", "cos_t", "sin_t")] + [
        (n, ctypes.POINTER(ctypes.c_void_p)) for n in (
            "win", "wkvn", "wpost", "gate", "wqkv", "wuk", "wuv", "wo", "wg1", "wu1", "wd1", "wg", "wu", "wd",
            "swg", "swu", "swd")]


class _OrcDSRefTrace(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("ql", "sm", "ol", "ob", "g1o", "u1o")]


@dataclass(frozen=True)
class DSRefConfig:
    """Shape knobs of the reference's DeepSeek-V2 decode bench
    (bench/dsv2_decode_bench.c cfg_init :106-131; DSV2_* environment names)."""
    dim: int = 2048
    n_layers: int = 27
    heads: int = 16
    kv_lora: int = 512
    d_nope: int = 128
    d_rope: int = 64
    d_v: int = 128
    n_exp: int = 64
    n_shared: int = 2
    top_k: int = 6
    moe_inter: int = 1408
    dense_inter: int = 10944
    first_dense: int = 1
    vocab: int = 102400
    max_seq: int = 1024
    eps: float = 1e-6

    @property
    def scale(self) -> float:
        """(dn + dr)^-0.5 * mscale^2, mscale = 0.1 * 0.707 * ln(40) + 1, as a float (cfg_init :125-129)."""
        ms = 0.1 * 0.707 * math.log(40.0) + 1.0
        return float(np.float32(math.pow(self.d_nope + self.d_rope, -0.5) * ms * ms))

    def env(self) -> dict:
        names = {"dim": "DIM", "n_layers": "LAYERS", "heads": "HEADS", "kv_lora": "KVLORA", "d_nope": "DNOPE",
                 "d_rope": "DROPE", "d_v": "DV", "n_exp": "EXPERTS", "n_shared": "NSHARED", "top_k": "TOPK",
                 "moe_inter": "MOEINTER", "dense_inter": "DENSEINTER", "first_dense": "FIRSTDENSE",
                 "vocab": "VOCAB", "max_seq": "MAXSEQ"}
        return {f"DSV2_{v}": str(getattr(self, k)) for k, v in names.items()}


# the shape the reference run in tests/golden/dsv2.npz used
DSREF_SMALL = DSRefConfig(dim=256, n_layers=3, heads=4, kv_lora=128, d_nope=32, d_rope=16, d_v=32, n_exp=16,
                          n_shared=2, top_k=4, moe_inter=64, dense_inter=512, first_dense=1, vocab=2048, max_seq=64)


def ds_rope_tables(d_rope: int, max_seq: int):
    """YaRN cos / sin [max_seq, d_rope] f32, halves duplicated: the reference's
    rope_tables (bench/dsv2_decode_bench.c:312-343) in doubles through libm,
    rounded to float once."""
    half = d_rope // 2
    theta, factor, orig, bfast, bslow = 10000.0, 40.0, 4096.0, 32.0, 1.0
    lo = math.floor((d_rope * math.log(orig / (bfast * 2.0 * math.pi))) / (2.0 * math.log(theta)))
    hi = math.ceil((d_rope * math.log(orig / (bslow * 2.0 * math.pi))) / (2.0 * math.log(theta)))
    lo, hi = max(lo, 0), min(hi, d_rope - 1)
    freqs = []
    for j in range(half):
        pf = math.pow(theta, (2 * j) / d_rope)
        ramp = min(max((j - lo) / ((hi - lo) if (hi - lo) > 1e-3 else 1e-3), 0.0), 1.0)
        freqs.append((1.0 / (factor * pf)) * ramp + (1.0 / pf) * (1.0 - ramp))
    cs = np.empty((max_seq, d_rope), np.float32)
    sn = np.empty((max_seq, d_rope), np.float32)
    for p_ in range(max_seq):
        for j in range(half):
            a = p_ * freqs[j]
            cs[p_, j] = cs[p_, half + j] = math.cos(a)
            sn[p_, j] = sn[p_, half + j] = math.sin(a)
    return cs, sn


def _bf16_bits(a: np.ndarray) -> np.ndarray:
    out = np.empty(a.size, np.uint16)
    lib().orc_f32_to_bf16_n(np.ascontiguousarray(a, np.float32).ravel(), out, a.size)
    return out.reshape(a.shape)


def ds_ref_weights(cfg: DSRefConfig, seed: int = 0, std: float = 0.02, fp8_experts: bool = False) -> dict:
    """Seeded weights in the DSV2PK01 pack's names and layouts
    (bench/dsv2_decode_bench.c model_init :2130-2254): bf16 matrices N(0, std);
    norm gains 1 + U(-0.1, 0.1) (f32); router f32 N(0, 0.05).  fp8_experts:
    the routed and shared expert matrices are e4m3 values of N(0, 1) draws
    times 2^-6, which bf16 holds exactly, so the same experts can be stated as
    fp8 codes with a block scale of 2^-6."""
    rng = np.random.default_rng(seed)
    D, H, KV, DN, DR, DV = cfg.dim, cfg.heads, cfg.kv_lora, cfg.d_nope, cfg.d_rope, cfg.d_v
    E, MI, SI, DI = cfg.n_exp, cfg.moe_inter, cfg.moe_inter * cfg.n_shared, cfg.dense_inter

    def bf(*shape):
        return _bf16_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))

    def ex(*shape):
        if not fp8_experts:
            return bf(*shape)
        codes = np.empty(int(np.prod(shape)), np.uint8)
        lib().orc_f32_to_fp8e4m3_n(rng.standard_normal(codes.size, dtype=np.float32), codes, codes.size)
        vals = np.array([lib().orc_fp8e4m3_to_f32(int(c)) for c in range(256)], np.float32)[codes]
        return _bf16_bits(vals * np.float32(2.0 ** -6)).reshape(shape)

    def gain(n):
        return (1.0 + rng.uniform(-0.1, 0.1, n)).astype(np.float32)

    w = {"embed": bf(cfg.vocab, D), "norm": gain(D), "lm_head": bf(D, cfg.vocab)}
    for l in range(cfg.n_layers):
        p = f"l{l}."
        w[p + "win"] = gain(D)
        w[p + "wq"] = bf(D, H * (DN + DR))
        w[p + "wkv"] = bf(D, KV + DR)
        w[p + "wkvn"] = gain(KV)
        w[p + "wuk"] = bf(H * DN * KV)
        w[p + "wuv"] = bf(H * DV * KV)
        w[p + "wo"] = bf(H * DV, D)
        w[p + "wpost"] = gain(D)
        if l < cfg.first_dense:
            w[p + "wg1"], w[p + "wu1"], w[p + "wd1"] = bf(D, DI), bf(D, DI), bf(DI, D)
        else:
            w[p + "gate"] = (rng.standard_normal((D, E)) * 0.05).astype(np.float32)
            w[p + "wg"], w[p + "wu"], w[p + "wd"] = ex(E * MI, D), ex(E * MI, D), ex(E * D, MI)
            w[p + "swg"], w[p + "swu"], w[p + "swd"] = ex(SI, D), ex(SI, D), ex(D, SI)
    return w


def write_dsv2_pack(path, weights: dict) -> None:
    """The DSV2PK01 weight pack the reference's bench loads (DSV2_WEIGHTS,
    bench/dsv2_decode_bench.c:229-262): magic, u64 count, count x {char
    name[48]; u32 dtype (0 bf16, 1 f32); u32 pad; u64 offset; u64 nbytes},
    64-byte-aligned payloads."""
    import struct
    names = list(weights)
    off = 16 + 72 * len(names)
    table, blobs = [], []
    for n in names:
        a = np.ascontiguousarray(weights[n])
        dt = 0 if a.dtype == np.uint16 else 1
        if dt == 1:
            a = a.astype(np.float32)
        off = (off + 63) // 64 * 64
        table.append(struct.pack("<48sIIQQ", n.encode(), dt, 0, off, a.nbytes))
        blobs.append((off, a.tobytes()))
        off += a.nbytes
    with open(path, "wb") as f:
        f.write(b"DSV2PK01" + struct.pack("<Q", len(names)) + b"".join(table))
        for o, b in blobs:
            f.write(b"\0" * (o - f.tell()))
            f.write(b)


def ds_from_ref(cfg: DSRefConfig, w: dict, batch: int = 1):
    """(config, weights) for DSModel (orc_ds_step, the batched config-5
    composition) holding the same model as a ds_ref_weights(fp8_experts=True)
    dict: projections transposed to (out, in); gate | up and the shared halves
    regrouped per expert; expert matrices as e4m3 codes with block scale 2^-6
    (exact); the f32 router rounded to bf16 (the one lossy change)."""
    from types import SimpleNamespace
    D, E, MI, NS = cfg.dim, cfg.n_exp, cfg.moe_inter, cfg.n_shared
    c = SimpleNamespace(dim=D, n_layers=cfg.n_layers, heads=cfg.heads, kv_lora=cfg.kv_lora, d_nope=cfg.d_nope,
                        d_rope=cfg.d_rope, d_v=cfg.d_v, n_exp=E, top_k=cfg.top_k, moe_inter=MI,
                        dense_inter=cfg.dense_inter, n_dense=cfg.first_dense, n_shared=NS, vocab=cfg.vocab,
                        max_ctx=cfg.max_seq, batch=batch, eps=cfg.eps, scale=cfg.scale)

    def codes(bits):
        v = np.ascontiguousarray(bf16_to_f32(bits) * np.float32(64.0))
        out = np.empty(v.size, np.uint8)
        lib().orc_f32_to_fp8e4m3_n(v.ravel(), out, v.size)
        return out.reshape(v.shape)

    T = lambda a: np.ascontiguousarray(a.T)
    o = {"embed": w["embed"], "lm_head": T(w["lm_head"]), "norm_f": w["norm"]}
    for l in range(cfg.n_layers):
        p = f"l{l}."
        o[p + "attn_norm"], o[p + "kv_norm"], o[p + "ffn_norm"] = w[p + "win"], w[p + "wkvn"], w[p + "wpost"]
        o[p + "w_qkva"] = T(np.concatenate([w[p + "wq"], w[p + "wkv"]], 1))
        o[p + "w_uk"], o[p + "w_uv"], o[p + "w_o"] = w[p + "wuk"], w[p + "wuv"], T(w[p + "wo"])
        if l < cfg.first_dense:
            o[p + "d_gu"] = np.ascontiguousarray(np.concatenate([w[p + "wg1"].T, w[p + "wu1"].T], 0))
            o[p + "d_down"] = T(w[p + "wd1"])
            continue
        o[p + "router"] = to_bf16(T(w[p + "gate"]))
        rows = lambda a, i: a[i * MI:(i + 1) * MI]
        gu = [np.concatenate([rows(w[p + "wg"], e), rows(w[p + "wu"], e)]) for e in range(E)]
        gu += [np.concatenate([rows(w[p + "swg"], k), rows(w[p + "swu"], k)]) for k in range(NS)]
        dn = [w[p + "wd"][e * D:(e + 1) * D] for e in range(E)] + [w[p + "swd"][:, k * MI:(k + 1) * MI]
                                                                  for k in range(NS)]
        o[p + "e_gu"], o[p + "e_d"] = codes(np.stack(gu)), codes(np.stack(dn))
        o[p + "e_gu_s"] = np.full((E + NS, -(-2 * MI // 128), -(-D // 128)), 2.0 ** -6, np.float32)
        o[p + "e_d_s"] = np.full((E + NS, -(-D // 128), -(-MI // 128)), 2.0 ** -6, np.float32)
    return c, o


class DSRef:
    """orc_ds_ref_step over a ds_ref_weights dict: the reference's batch-1 step."""

    _layer = ("win", "wkvn", "wpost", "gate", "wqkv", "wuk", "wuv", "wo", "wg1", "wu1", "wd1", "wg", "wu", "wd",
              "swg", "swu", "swd")

    def __init__(self, cfg: DSRefConfig, weights: dict):
        self.cfg = cfg
        w = {k: np.ascontiguousarray(v) for k, v in weights.items()}
        for l in range(cfg.n_layers):   # the q | kv row concatenation of model_init :2162-2170
            w[f"l{l}.wqkv"] = np.ascontiguousarray(np.concatenate([w[f"l{l}.wq"], w[f"l{l}.wkv"]], axis=1))
        w["cos"], w["sin"] = ds_rope_tables(cfg.d_rope, cfg.max_seq)
        self._keep = w
        s = _OrcDSRef(**{f: getattr(cfg, f) for f in (
            "dim", "n_layers", "heads", "kv_lora", "d_nope", "d_rope", "d_v", "n_exp", "n_shared", "top_k",
            "moe_inter", "dense_inter", "first_dense", "vocab", "max_seq")}, eps=cfg.eps, scale=cfg.scale)
        s.embed, s.lm_head, s.norm = w["embed"].ctypes.data, w["lm_head"].ctypes.data, w["norm"].ctypes.data
        s.cos_t, s.sin_t = w["cos"].ctypes.data, w["sin"].ctypes.data
        self._arrays = []
        for f in self._layer:
            ptrs = [w[f"l{i}.{f}"].ctypes.data if f"l{i}.{f}" in w else None for i in range(cfg.n_layers)]
            arr = (ctypes.c_void_p * cfg.n_layers)(*ptrs)
            self._arrays.append(arr)
            setattr(s, f, ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)))
        self._s = s
        self.ckv = np.zeros((cfg.n_layers, cfg.max_seq, cfg.kv_lora), np.uint16)
        self.kpe = np.zeros((cfg.n_layers, cfg.max_seq, cfg.d_rope), np.uint16)
        H, KV = cfg.heads, cfg.kv_lora
        self.trace = {"ql": np.zeros(H * KV, np.float32), "sm": np.zeros(H * cfg.max_seq, np.float32),
                      "ol": np.zeros(H * KV, np.float32), "ob": np.zeros(H * cfg.d_v, np.uint16),
                      "g1o": np.zeros(cfg.dense_inter, np.uint16), "u1o": np.zeros(cfg.dense_inter, np.uint16)}
        self._tr = _OrcDSRefTrace(**{k: v.ctypes.data for k, v in self.trace.items()})
        L = lib()
        if not getattr(L, "_dsref_bound", False):
            L.orc_ds_ref_step.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                                                  ctypes.c_void_p]
            L.orc_ds_ref_step.restype = ctypes.c_int32
            L._dsref_bound = True

    def step(self, tok: int, length: int):
        """(logits [V], argmax) of one step of `tok` with `length` positions (row length - 1 written)."""
        lg = np.empty(self.cfg.vocab, np.float32)
        nxt = lib().orc_ds_ref_step(ctypes.byref(self._s), self.ckv.ctypes.data, self.kpe.ctypes.data, int(tok),
                                    int(length), lg.ctypes.data, ctypes.byref(self._tr))
        return lg, int(nxt)


def num_threads() -> int:
    return int(lib().orc_num_threads())
