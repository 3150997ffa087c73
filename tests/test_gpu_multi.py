"""The sharded decode steps on two GPUs against the CPU oracle
(tests/tp_parity.py under torch.distributed.run, one process per GPU):
the peer-memory collectives alone, config 5 split over heads, dense units,
experts and vocabulary rows (its all-reduces fused into RMSNorm kernels over
peer memory), its speculative decode and serve loop, and config 3 split
Megatron-style (decode steps, and the prompt pass followed by decode steps).  Skipped when fewer than two GPUs are visible."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _gpus():
    import torch
    return torch.cuda.device_count()


@pytest.mark.parametrize("which", ["comm", "ds", "xl", "spec"])
def test_two_rank_decode_matches_oracle(which):
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(29530 + ["comm", "ds", "xl", "spec"].index(which)),
           str(ROOT / "tests" / "tp_parity.py"), which]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
