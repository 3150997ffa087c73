"""The reference-side router on the CPU.  The reference's own GPT-2 example
(2 layers, the golden's 16 prompt ids, 8 greedy ids) runs through the
reference's own `thvm` package on a build of its runtime that carries the
router in checking mode (thvm_b200/refside, `make cpu`): every kernel the
CPU backend dispatches is planned (hand-written matvec, or the generic
interpreter), re-run by the interpreter core on the host over the buffers
the CPU backend read, and compared with the output it wrote."""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "thvm_b200" / "refside" / "_build" / "cpu" / "thvm" / "libthvm_py.so"


@pytest.mark.skipif(not LIB.exists(), reason="reference-side build absent (make -C thvm_b200/refside cpu)")
@pytest.mark.parametrize("prepass", ["0", "1"])
def test_every_gpt2_kernel_is_routed_and_rechecks(prepass):
    """prepass 0: every reduce runs inline, in the walker's order, so every
    interpreted kernel is bit-exact.  prepass 1 (the default): reduces that
    every output element would recompute move to chunked pre-pass programs;
    a chunked sum rounds differently, so those kernels are checked within the
    tolerance (1e-4 relative) and the rest stay bit-exact."""
    env = dict(os.environ, THVM_SM100_CHECK="1", JIT="0", THVM_SM100_PREPASS=prepass)
    r = subprocess.run([sys.executable, str(ROOT / "tests" / "refside_gpt2.py"), "cpu", "2", "8"], env=env,
                       capture_output=True, text=True, timeout=1200)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    golden = np.load(ROOT / "tests" / "golden" / "gpt2_l2.npz")
    assert res["ids"] == golden["tokens"].tolist()
    # nothing is left to the reference's rendered path
    assert res["declined"] == 0, res
    assert res["linear"] > 0 and res["interp"] > 0, res
    assert res["checked"] == res["dispatch"] and res["mismatch"] == 0, res
    if prepass == "0":
        # the interpreter computes in the walker's order: its outputs are bit-exact
        assert res["exact"] == res["interp"], res
    else:
        assert res["exact"] >= 0.9 * res["interp"], res
