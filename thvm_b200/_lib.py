"""ctypes bindings over libthvm_sm100.so (include/thvm_sm100.h).

The library is the product: there is no CPU fallback.  Loading fails with an
ImportError when the in-tree build is missing (build it with
`python -m thvm_b200.build`).
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int, c_int32, c_int64, c_uint32, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(os.environ.get("THVM_SM100_LIB") or Path(__file__).resolve().parent / "libthvm_sm100.so")

OK = 0
ERR_ARG, ERR_CUDA, ERR_UNSUPPORTED, ERR_OOM, ERR_STATE, ERR_TIMEOUT = -1, -2, -3, -4, -5, -6
DT_F32, DT_BF16, DT_FP8E4M3, DT_I32 = 0, 1, 2, 3

(K_LINEAR, K_LAYERNORM, K_RMSNORM, K_SOFTMAX, K_GELU, K_ADD, K_ATTENTION, K_EMBEDDING, K_ARGMAX,
 K_SCATTER, K_KV_APPEND, K_POS_ADD, K_DECODE_STEP, K_ATTN_PREFILL) = range(1, 15)

DECODE_MAX_LAYERS = 48
DECODE_REPLICAS = 8
DECODE_ERR_STALL, DECODE_ERR_BARRIER, DECODE_ERR_ARG = 1, 2, 4

LIN_LN, LIN_GELU, LIN_RESIDUAL, LIN_KV_APPEND = 1, 2, 4, 8


class Sm100Kernel(ctypes.Structure):
    _fields_ = [
        ("kind", c_uint32), ("dtype", c_uint32), ("flags", c_uint32),
        ("inp", c_int32 * 10),
        ("m", c_int64), ("n", c_int64), ("k", c_int64),
        ("ld_in", c_int64), ("ld_out", c_int64), ("row_off", c_int64),
        ("heads", c_int32), ("head_dim", c_int32), ("max_ctx", c_int32), ("causal", c_int32),
        ("pos", c_int32), ("eps", c_float), ("scale", c_float),
    ]

    @classmethod
    def make(cls, kind, slots=None, **kw):
        k = cls()
        k.kind = kind
        for i in range(10):
            k.inp[i] = -1
        for s, v in (slots or {}).items():
            k.inp[s] = v
        for name, v in kw.items():
            setattr(k, name, v)
        return k


class Sm100View(ctypes.Structure):
    _fields_ = [("ndim", c_uint32), ("elem_bytes", c_uint32), ("offset", c_int64),
                ("dims", c_int64 * 8), ("strides", c_int64 * 8)]


class Sm100LinearArgs(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("x", "w", "w_scale", "bias", "ln_g", "ln_b", "residual", "y",
                                        "kv_cache", "pos")] + [
        (n, c_int64) for n in ("M", "N", "K", "ldx", "ldy")] + [
        (n, c_int32) for n in ("wdtype", "flags", "max_ctx", "host_pos")] + [("eps", c_float)]


class Sm100AttnArgs(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("q", "k_cache", "v_cache", "out", "pos")] + [
        ("ldq", c_int64)] + [(n, c_int32) for n in ("T", "H", "hd", "max_ctx", "host_pos")] + [
        ("scale", c_float)]


SK_GELU, SK_RESIDUAL, SK_OUT_BF16, SK_KV, SK_ACCUM, SK_X_GELU, SK_X_LN = 1, 2, 4, 8, 16, 32, 64
GEMM_GELU, GEMM_OUT_BF16 = 1, 2


class Sm100TensorEntry(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 128), ("dtype", ctypes.c_char * 12), ("ndim", c_int32),
                ("shape", c_int64 * 8), ("nbytes", c_uint64), ("buf_id", c_uint32)]


class Sm100Insn(ctypes.Structure):
    """One instruction of the generic device interpreter (include/thvm_sm100.h)."""
    _fields_ = [("op", ctypes.c_uint8), ("dt", ctypes.c_uint8), ("dst", ctypes.c_uint16), ("a", ctypes.c_uint16),
                ("b", ctypes.c_uint16), ("c", ctypes.c_uint16), ("imm", c_int32)]


class Sm100XlCfg(ctypes.Structure):
    """include/thvm_sm100.h Sm100XlCfg: the config-3 model of the C host."""
    _fields_ = [(f, c_int32) for f in ("n_layers", "dim", "heads", "vocab", "max_ctx", "batch")] + \
        [("norm_eps", c_float)]


class Sm100DsCfg(ctypes.Structure):
    """include/thvm_sm100.h Sm100DsCfg: the config-5 model of the C host."""
    _fields_ = [(n, c_int32) for n in ("n_layers", "dim", "heads", "kv_lora", "d_nope", "d_rope", "d_v", "n_exp",
                                       "top_k", "moe_inter", "dense_inter", "n_dense", "n_shared", "vocab", "max_ctx",
                                       "batch")] + [("eps", c_float), ("scale", c_float)]


class Sm100DsRows(ctypes.Structure):
    """include/thvm_sm100.h Sm100DsRows: per-row cache slots and positions."""
    _fields_ = [("pos", c_void_p), ("seq", c_void_p), ("n_seq", c_int32), ("shared_slots", c_int32)]


class Sm100SkinnyArgs(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("x", "w", "bias", "residual", "y", "ws", "counters", "kv_cache", "pos")] + [
        (n, c_int64) for n in ("M", "N", "K", "ld_x", "ld_w", "ld_res", "ld_y")] + [
        ("flags", c_int32), ("kv_ctx", c_int32), ("ln_g", c_void_p), ("ln_b", c_void_p), ("eps", c_float)]


_PL = ctypes.c_void_p * DECODE_MAX_LAYERS


class Sm100DecodeModel(ctypes.Structure):
    _fields_ = [("kv_map", (ctypes.c_uint8 * 128) * DECODE_MAX_LAYERS)] + [(n, c_int32) for n in ("n_layers", "dim", "hidden", "vocab", "max_ctx", "heads", "head_dim",
                                       "bump")] + [
        ("eps", c_float), ("attn_scale", c_float)] + [
        (n, c_void_p) for n in ("wte", "wpe", "ln_f_g", "ln_f_b", "lm_head_bt")] + [
        (n, _PL) for n in ("ln1_g", "ln1_b", "w_qkv_bt", "b_qkv", "b_o", "ln2_g", "ln2_b", "w_fc_bt", "b_fc",
                           "b_p2", "w_o_h", "w_p2_t", "kv_cache")] + [
        (n, c_void_p) for n in ("io", "qkv_w", "red_w", "part_w", "logits", "trace", "sync")]


# name -> (restype, argtypes): every symbol include/thvm_sm100.h declares.
SIGNATURES = {
    "sm100_init": (c_int, []),
    "sm100_shutdown": (None, []),
    "sm100_last_error": (ctypes.c_char_p, []),
    "sm100_ready": (c_int, []),
    "sm100_debug_host_memory": (None, [c_int]),
    "sm100_buf_alloc": (c_uint32, [c_uint64]),
    "sm100_buf_free": (None, [c_uint32]),
    "sm100_buf_incref": (None, [c_uint32]),
    "sm100_buf_decref": (None, [c_uint32]),
    "sm100_buf_jit_pin": (None, [c_uint32]),
    "sm100_buf_jit_unpin": (None, [c_uint32]),
    "sm100_buf_read": (c_int, [c_uint32, c_void_p, c_uint64]),
    "sm100_buf_write": (c_int, [c_uint32, c_void_p, c_uint64]),
    "sm100_buf_copy": (c_int, [c_uint32, c_uint32, c_uint64]),
    "sm100_buf_write_at": (c_int, [c_uint32, c_uint64, c_void_p, c_uint64]),
    "sm100_buf_copy_at": (c_int, [c_uint32, c_uint64, c_uint32, c_uint64]),
    "sm100_buf_refcount": (c_uint32, [c_uint32]),
    "sm100_buf_freelist_push": (None, [c_uint32]),
    "sm100_buf_freelist_remove": (None, [c_uint32]),
    "sm100_buf_storage_root": (c_uint32, [c_uint32]),
    "sm100_buf_nbytes": (c_uint64, [c_uint32]),
    "sm100_buf_zero": (None, [c_uint32]),
    "sm100_buf_view": (c_uint32, [c_uint32, c_uint64, c_uint64]),
    "sm100_buf_dptr": (c_void_p, [c_uint32]),
    "sm100_mem_live_bytes": (c_uint64, []),
    "sm100_mem_peak_bytes": (c_uint64, []),
    "sm100_buf_live_count": (c_uint32, []),
    "sm100_stream": (c_void_p, []),
    "sm100_set_stream": (c_int, [c_void_p]),
    "sm100_dispatch_begin": (None, []),
    "sm100_dispatch_flush": (None, []),
    "sm100_dispatch_end": (None, []),
    "sm100_dispatch_kernel": (c_int, [POINTER(Sm100Kernel), POINTER(c_uint32), c_uint32, c_uint32]),
    "sm100_gather_strided": (c_int, [c_uint32, c_uint32, POINTER(Sm100View)]),
    "sm100_linear": (c_int, [POINTER(Sm100LinearArgs), c_void_p]),
    "sm100_attention": (c_int, [POINTER(Sm100AttnArgs), c_void_p]),
    "sm100_layernorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p]),
    "sm100_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p]),
    "sm100_softmax": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "sm100_gelu": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "sm100_add": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "sm100_embedding": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                c_void_p]),
    "sm100_argmax": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "sm100_argmax_noalloc": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "sm100_scatter_rows":(c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int32, c_void_p]),
    "sm100_kv_append": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int32, c_int32, c_int32,
                                c_int32, c_void_p]),
    "sm100_pos_add": (c_int, [c_void_p, c_int32, c_void_p]),
    "sm100_decode_sync_bytes": (c_uint64, []),
    "sm100_decode_trace_bytes": (c_uint64, [c_int32]),
    "sm100_decode_part_bytes": (c_uint64, []),
    "sm100_decode_red_bytes": (c_uint64, [c_int32, c_int32]),
    "sm100_decode_grid": (c_int32, [c_int32, c_int32]),
    "sm100_decode_prepare": (c_int, [c_void_p]),
    "sm100_decode_block_transpose": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p]),
    "sm100_decode_regroup": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p]),
    "sm100_decode_steps": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p]),
    "sm100_decode_step": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p]),
    "sm100_gemm_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p]),
    "sm100_gemm_bf16_ep": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int32,
                                   c_void_p]),
    "sm100_gemm_status": (c_uint32, []),
    "sm100_attn_prefill_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
                                        c_float, c_int32, c_void_p]),
    "sm100_attn_prefill_status": (c_uint32, []),
    "sm100_skinny_bf16": (c_int, [c_void_p, c_void_p]),
    "sm100_skinny_ws_bytes": (c_uint64, [c_int32]),
    "sm100_skinny_status": (c_uint32, []),
    "sm100_xl_embed": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p]),
    "sm100_xl_layernorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_float, c_int32,
                                   c_void_p, c_int64, c_void_p]),
    "sm100_xl_attention": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                   c_int32, c_float, c_int32, c_void_p]),
    "sm100_xl_argmax": (c_int, [c_void_p, c_int64, c_int32, c_int32, c_void_p, c_void_p, c_int32, c_int32,
                                c_void_p]),
    "sm100_xl_pick": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p]),
    "sm100_xl_prefill_embed": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
                                       c_void_p]),
    "sm100_xl_prefill_split": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                       c_int32, c_void_p]),
    "sm100_xl_prefill_merge": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p]),
    "sm100_xl_prefill_layernorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_float,
                                           c_void_p]),
    "sm100_xl_prefill_last": (c_int, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p]),
    "sm100_ds_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_float, c_void_p]),
    "sm100_ds_embed": (c_int, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p]),
    "sm100_ds_qkv_post": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_float,
                                  c_void_p]),
    "sm100_ds_mla": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                             c_int32, c_int32, c_int32, c_int32, c_int32, c_float, c_void_p]),
    "sm100_ds_route": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p,
                               c_void_p, c_void_p, c_void_p, c_void_p]),
    "sm100_ds_mla_post": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
                                  c_int32, c_int32, c_int32, c_float, c_float, c_void_p]),
    "sm100_ds_mla_post_rows": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                       c_int32, c_int32, c_int32, c_int32, c_float, c_float, c_void_p]),
    "sm100_spec_draft": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_void_p]),
    "sm100_spec_accept": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p,
                                  c_void_p]),
    "sm100_spec_status": (c_uint32, []),
    "sm100_ds_model_open": (c_int, [c_void_p, ctypes.c_char_p, c_uint32, c_void_p]),
    "sm100_ds_model_open_ptrs": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_uint32, c_void_p]),
    "sm100_ds_model_step": (c_int, [c_void_p, c_void_p, c_void_p]),
    "sm100_ds_model_pos": (c_int32, [c_void_p]),
    "sm100_ds_model_reset": (c_int, [c_void_p]),
    "sm100_ds_model_logits": (c_uint32, [c_void_p]),
    "sm100_ds_model_close": (None, [c_void_p]),
    "sm100_xl_model_open": (c_int, [c_void_p, ctypes.c_char_p, c_uint32, c_void_p]),
    "sm100_xl_model_open_ptrs": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_uint32, c_void_p]),
    "sm100_xl_model_prefill": (c_int, [c_void_p, c_void_p, c_int32, c_void_p]),
    "sm100_xl_model_step": (c_int, [c_void_p, c_void_p, c_void_p]),
    "sm100_xl_model_pos": (c_int32, [c_void_p]),
    "sm100_xl_model_logits": (c_uint32, [c_void_p]),
    "sm100_xl_model_close": (None, [c_void_p]),
    "sm100_serve_advance": (c_int, [c_void_p] * 10 + [c_int32, c_int32, c_void_p]),
    "sm100_ds_router_route": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
                                      c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_void_p]),
    "sm100_ds_experts": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p]),
    "sm100_ds_silu_mul": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_void_p]),
    "sm100_ds_status": (c_uint32, []),
    "sm100_comm_bytes": (c_uint64, [c_int32]),
    "sm100_peer_alloc": (c_int, [c_uint64, POINTER(c_void_p), c_void_p]),
    "sm100_peer_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "sm100_peer_close": (c_int, [c_void_p]),
    "sm100_peer_free": (c_int, [c_void_p]),
    "sm100_comm_set_peers": (c_int, [c_void_p, POINTER(c_void_p), c_int32]),
    "sm100_comm_allreduce_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                             c_int32, c_float, c_int32, c_void_p]),
    "sm100_comm_allreduce_layernorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                                               c_int32, c_int32, c_float, c_void_p]),
    "sm100_comm_pick": (c_int, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p]),
    "sm100_comm_status": (c_uint32, []),
    "sm100_safetensors_load": (c_int, [ctypes.c_char_p, POINTER(Sm100TensorEntry), c_int32, POINTER(c_int32)]),
    "sm100_dsv2pack_load": (c_int, [ctypes.c_char_p, POINTER(Sm100TensorEntry), c_int32, POINTER(c_int32)]),
    "sm100_torch_load": (c_int, [ctypes.c_char_p, POINTER(Sm100TensorEntry), c_int32, POINTER(c_int32)]),
    "sm100_custom_program": (c_int32, [ctypes.c_char_p, ctypes.c_char_p, POINTER(c_uint32), POINTER(c_uint32),
                                       c_uint32]),
    "sm100_custom_dispatch": (c_int, [c_int32, POINTER(c_uint32), c_uint32, c_uint32, c_uint32]),
    "sm100_custom_launch": (c_int, [c_int32, POINTER(c_void_p), c_uint32, c_void_p]),
    "sm100_interp_run": (c_int, [POINTER(Sm100Insn), c_uint32, c_uint32, c_uint32, c_uint32, POINTER(c_int64),
                                 POINTER(c_void_p), POINTER(c_int64), c_uint32, POINTER(c_int64), c_uint32,
                                 c_void_p]),
    "sm100_interp_status": (c_int, []),
    "sm100_graph_capture_begin": (c_int, [c_uint32]),
    "sm100_graph_capture_end": (c_int, [c_uint32]),
    "sm100_graph_replay": (c_int, [c_uint32]),
    "sm100_graph_drop": (None, [c_uint32]),
    "sm100_graph_capturing": (c_int, []),
    "sm100_launch_count": (c_uint64, []),
}

_lib = None


def lib():
    """The loaded library with every declared signature bound."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m thvm_b200.build` "
                              "(the sm_100a device has no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class Sm100Error(RuntimeError):
    def __init__(self, code: int, what: str):
        msg = lib().sm100_last_error()
        super().__init__(f"{what} failed ({code}): {msg.decode() if msg else ''}")
        self.code = code


def check(code: int, what: str) -> int:
    if code != OK:
        raise Sm100Error(code, what)
    return code
