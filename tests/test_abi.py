"""The C ABI library on the CPU: it loads, exports every function that
include/*.h declares, and its Python bindings cover exactly those.  No compute
call is made here (no GPU)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(sm100_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    from thvm_b200 import _lib
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in sorted(_declared()) if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_match_header():
    from thvm_b200 import _lib
    assert set(_lib.SIGNATURES) == _declared()
    _lib.lib()  # binds every signature


def test_kernel_descriptor_layout():
    """Sm100Kernel in Python has the C struct's size and field offsets."""
    from thvm_b200._lib import Sm100Kernel
    # 3 u32 + 10 i32 (52 B), pad to 56, 6 i64, 5 i32 + 2 f32, padded to 8
    assert ctypes.sizeof(Sm100Kernel) == 136
    assert Sm100Kernel.m.offset == 56


def test_init_without_gpu_reports_error():
    """On a host with no CUDA device sm100_init fails with a message (and no
    CPU fallback is offered)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from thvm_b200 import _lib
    rc = _lib.lib().sm100_init()
    assert rc != 0
    assert _lib.lib().sm100_last_error()


def test_custom_program_compiles_for_sm100a_without_a_gpu():
    """The custom-kernel ABI compiles with NVRTC before it needs the device:
    a broken program fails with the compiler's log, a good one compiles for
    sm_100a and then reports that the device is not initialised."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from ctypes import c_uint32
    from thvm_b200 import _lib
    lib = _lib.lib()
    g, b = (c_uint32 * 3)(1, 1, 1), (c_uint32 * 3)(32, 1, 1)
    bad = b'extern "C" __global__ void broken(float *y) { y[0] = undefined_name; }\n'
    assert lib.sm100_custom_program(b"broken", bad, g, b, 0) == _lib.ERR_UNSUPPORTED
    assert b"undefined_name" in lib.sm100_last_error()
    good = b'extern "C" __global__ void fine(float *y) { y[threadIdx.x] = 1.0f; }\n'
    assert lib.sm100_custom_program(b"fine", good, g, b, 0) == _lib.ERR_STATE
    assert b"compiled" in lib.sm100_last_error()
    assert lib.sm100_custom_program(b"fine", good, g, (c_uint32 * 3)(2048, 1, 1), 0) == _lib.ERR_ARG


def test_prompt_pass_entry_points_reject_bad_arguments_without_a_gpu():
    """The fused-epilogue GEMM, the prompt-pass glue and the config-3 C host
    check their arguments before anything touches a device: shapes outside
    their contracts come back as SM100_ERR_ARG with a message."""
    from thvm_b200 import _lib
    lib = _lib.lib()
    p = ctypes.c_void_p(1 << 20)   # an aligned stand-in address; never dereferenced
    ERR = _lib.ERR_ARG
    assert lib.sm100_gemm_bf16_ep(None, p, p, 128, 256, 64, None, None, 0, None) == ERR
    assert lib.sm100_gemm_bf16_ep(p, p, p, 128, 100, 64, None, None, 0, None) == ERR            # N % 8
    assert lib.sm100_gemm_bf16_ep(p, p, p, 128, 256, 60, None, None, 0, None) == ERR            # K % 8
    assert lib.sm100_gemm_bf16_ep(p, p, p, 128, 256, 64, None, p, _lib.GEMM_OUT_BF16, None) == ERR  # bf16 in place
    assert lib.sm100_gemm_bf16_ep(p, p, p, 128, 256, 64, None, None, 8, None) == ERR            # unknown flag
    assert lib.sm100_xl_prefill_split(p, p, p, p, p, 16, 65, 4, 64, None) == ERR               # P > ctx
    assert lib.sm100_xl_prefill_layernorm(p, p, p, p, 16, 4096, 1e-5, None) == ERR             # D > 2048
    assert lib.sm100_xl_prefill_merge(None, p, 16, 8, 4, None) == ERR
    assert lib.sm100_xl_prefill_embed(p, p, p, p, 0, 8, 1000, 256, None) == ERR
    assert lib.sm100_xl_prefill_last(p, p, None, 16, 8, 256, None) == ERR
    cfg = _lib.Sm100XlCfg(n_layers=2, dim=320, heads=4, vocab=1000, max_ctx=64, batch=16, norm_eps=1e-5)  # dim != 64 heads
    out = ctypes.c_void_p()
    assert lib.sm100_xl_model_open(ctypes.byref(cfg), b"missing.safetensors", 0, ctypes.byref(out)) == ERR
    assert not out.value
    assert b"configuration" in lib.sm100_last_error()
    assert ctypes.sizeof(_lib.Sm100XlCfg) == 28
