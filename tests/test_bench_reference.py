"""bench.py's reference arms that run on the host cores alone (no GPU): the
config-3 and config-4 CPU paths print one JSON line each with the contract's
keys, the workload's metric and unit, and a positive value."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("workload,metric,unit", [
    ("xl", "decode tok/s (GPT-2 XL bf16 b16, tensor-parallel)", "tok/s"),
    ("prefill", "causal prefill TFLOP/s (B4 H16 S2048 D128 bf16)", "TFLOP/s"),
])
def test_reference_arm_prints_one_contract_line(workload, metric, unit):
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--workload", workload, "--impl", "reference",
                        "--steps", "1", "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == metric and d["unit"] == unit and d["value"] > 0
    for k in ("n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
