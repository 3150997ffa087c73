"""CPU oracle (test infrastructure only).

ctypes bindings over oracle/liboracle.so (our C restatement of the reference's
CPU arithmetic, oracle.c) and, for the timed reference arm, oracle/_ref (the
reference's own CPU path compiled from its sources).  Only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
import this package; the product (thvm_b200/) never does.
"""
from __future__ import annotations

import ctypes
import subprocess
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
            "c_attn_b", "c_proj_b", "c_fc_b", "mlp_proj_b")]


class XLModel:
    """The oracle's batched bf16 decode step (orc_xl_step) over the weight
    dict of thvm_b200.gpt2_xl.xl_weights (bf16 bits as uint16, f32 vectors)."""

    _per_layer = {"ln_1_w": "ln_1.w", "ln_1_b": "ln_1.b", "ln_2_w": "ln_2.w", "ln_2_b": "ln_2.b",
                  "c_attn_w": "attn.w", "c_proj_w": "proj.w", "c_fc_w": "fc.w", "mlp_proj_w": "p2.w",
                  "c_attn_b": "attn.b", "c_proj_b": "proj.b", "c_fc_b": "fc.b", "mlp_proj_b": "p2.b"}

    def __init__(self, cfg, weights: dict):
        self.cfg = cfg
        self._keep = {k: np.ascontiguousarray(v) for k, v in weights.items()}
        w = self._keep
        s = _OrcXL(n_layers=cfg.n_layers, dim=cfg.dim, heads=cfg.heads, vocab=cfg.vocab, max_ctx=cfg.max_ctx,
                   batch=cfg.batch, norm_eps=cfg.norm_eps)
        s.wte, s.wpe, s.lm_head = w["wte"].ctypes.data, w["wpe"].ctypes.data, w["lm_head"].ctypes.data
        s.ln_f_w, s.ln_f_b = w["ln_f.w"].ctypes.data, w["ln_f.b"].ctypes.data
        self._arrays = []
        for field, suffix in self._per_layer.items():
            arr = (ctypes.c_void_p * cfg.n_layers)(*[w[f"h.{i}.{suffix}"].ctypes.data for i in range(cfg.n_layers)])
            self._arrays.append(arr)
            setattr(s, field, ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)))
        self._s = s
        self.kv = np.zeros((cfg.n_layers, 2, cfg.batch, cfg.max_ctx, cfg.dim), np.uint16)
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


def num_threads() -> int:
    return int(lib().orc_num_threads())
