"""The router on the device.  (1) The generic interpreter's C ABI on a small
hand-written program: a row sum with a select and a loop, against numpy.
(2) The reference's own GPT-2 example (2 layers, 8 greedy ids) through the
reference's own `thvm` package with DEV=cuda, on a build of its runtime
whose dispatch_kernel is routed to this library (thvm_b200/refside,
`make cuda`): the ids equal the golden the reference's CPU path produced,
and every kernel ran on this library (hand-written matvec or interpreter),
none on the reference's rendered path."""
import ctypes
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from thvm_b200 import _lib as L

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
REFLIB = ROOT / "thvm_b200" / "refside" / "_build" / "cuda" / "thvm" / "libthvm_py.so"

I = {n: i + 1 for i, n in enumerate(
    "CONST RANGE VAR LOAD STORE FADD FMUL FNEG FRECIP FEXP2 FLOG2 FSQRT FSIN FLT FEQ IADD ISUB IMUL INEG IDIV IMOD "
    "ILT ULT IEQ IAND IOR IXOR ISHL ISHR WRAP I2F F2I NARROW SEL LOOP ENDLOOP ACCF ACCI THREEFRY".split())}


def _prog(code):
    return (L.Sm100Insn * len(code))(*[L.Sm100Insn(*c) for c in code])


def test_interp_row_sum_with_select(device):
    """y[i] = sum_j (0 < x[i, j] ? x[i, j] : 0) * 0.5 over a 37 x 53 f32
    block, then + x[rows * cols], a load past the end that reads 0."""
    import torch
    rows, cols = 37, 53
    x = torch.randn(rows, cols, device="cuda")
    y = torch.full((rows,), 7.0, device="cuda")
    code = [
        (I["CONST"], 2, 10, 0, 0, 0, 0),           # 0  r10 = 0.0f
        (I["CONST"], 2, 12, 0, 0, 0, 0x3F000000),  # 1  r12 = 0.5f
        (I["CONST"], 2, 2, 0, 0, 0, 0),            # 2  r2 = acc = 0.0f
        (I["CONST"], 1, 1, 0, 0, 0, cols),         # 3  r1 = cols
        (I["RANGE"], 0, 0, 0, 0, 0, 0),            # 4  r0 = i (output slot 0)
        (I["LOOP"], 0, 0, 1, 1, 0, 14),            # 5  slot 1 over [0, r1), ENDLOOP at 14
        (I["RANGE"], 0, 4, 1, 0, 0, 0),            # 6  r4 = j
        (I["IMUL"], 0, 5, 0, 1, 0, 0),             # 7  r5 = i * cols
        (I["IADD"], 0, 6, 5, 4, 0, 0),             # 8  r6 = i * cols + j
        (I["LOAD"], 13, 7, 1, 6, 0, 0),            # 9  r7 = x[r6]
        (I["FLT"], 0, 8, 10, 7, 0, 0),             # 10 r8 = 0 < x
        (I["SEL"], 0, 9, 8, 7, 10, 0),             # 11 r9 = r8 ? x : 0
        (I["FMUL"], 0, 11, 9, 12, 0, 0),           # 12 r11 = r9 * 0.5
        (I["ACCF"], 0, 2, 11, 0, 0, 0),            # 13 acc += r11
        (I["ENDLOOP"], 0, 0, 1, 1, 0, 5),          # 14
        (I["CONST"], 1, 13, 0, 0, 0, rows * cols), # 15 r13 = one past the end
        (I["LOAD"], 13, 14, 1, 13, 0, 0),          # 16 r14 = x[r13] -> 0
        (I["FADD"], 0, 15, 2, 14, 0, 0),           # 17 r15 = acc + r14
        (I["STORE"], 13, 0, 0, 0, 15, 1),          # 18 y[i] = r15
    ]
    ext = (ctypes.c_int64 * 1)(rows)
    bufs = (ctypes.c_void_p * 2)(y.data_ptr(), x.data_ptr())
    nbytes = (ctypes.c_int64 * 2)(rows * 4, rows * cols * 4)
    L.check(device.lib.sm100_interp_run(_prog(code), len(code), 16, 2, 1, ext, bufs, nbytes, 2, None, 0, None),
            "interp_run")
    torch.cuda.synchronize()
    assert device.lib.sm100_interp_status() == 0
    xs = x.cpu().numpy()
    ref = np.zeros(rows, np.float32)
    for i in range(rows):
        for j in range(cols):
            ref[i] = np.float32(ref[i] + np.float32(np.float32(max(xs[i, j], 0.0)) * np.float32(0.5)))
    np.testing.assert_array_equal(y.cpu().numpy(), ref)


def test_interp_rejects_a_malformed_loop(device):
    code = [(I["LOOP"], 0, 0, 0, 0, 0, 0)]  # names itself as its ENDLOOP
    ext = (ctypes.c_int64 * 1)(4)
    rc = device.lib.sm100_interp_run(_prog(code), 1, 4, 1, 1, ext, None, None, 0, None, 0, None)
    assert rc != 0 and b"loops" in device.lib.sm100_last_error()


@pytest.mark.skipif(not REFLIB.exists(), reason="reference-side build absent (make -C thvm_b200/refside cuda)")
@pytest.mark.parametrize("jit", ["0", "1"])
def test_reference_gpt2_runs_on_this_device(jit):
    env = dict(os.environ, JIT=jit)
    r = subprocess.run([sys.executable, str(ROOT / "tests" / "refside_gpt2.py"), "cuda", "2", "8"], env=env,
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    res = json.loads(r.stdout.strip().splitlines()[-1])
    golden = np.load(ROOT / "tests" / "golden" / "gpt2_l2.npz")
    assert res["ids"] == golden["tokens"].tolist(), res
    assert res["declined"] == 0 and res["linear"] > 0 and res["interp"] > 0, res
    assert res["interp_status"] == 0, res
