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
