"""bench.py's host logic, on the CPU: the reference arm's JSON line and the
choice between sequence sharding and the tensor-parallel hybrid for the ragged
9B batch (benchmark config 5).

The reference arm times the reference's CPU path (the C restatement of its
shader math in oracle/) and must print one JSON line with the same metric
keys as the GPU arm plus its cpu_baseline and an e2e record with no host/device
copies; the driver reads exactly these keys.
"""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


@pytest.mark.parametrize("world,sizes,tp,no_tp,want", [
    (1, [64], False, False, False),          # one GPU: never the hybrid
    (1, [64], True, False, False),           # --tp has nothing to split on one GPU
    (2, [32, 32], False, False, False),      # 16+ sequences per rank: sequence sharding
    (4, [16, 16, 16, 16], False, False, False),
    (8, [8] * 8, False, False, True),        # below 16 per rank: the hybrid
    (3, [22, 21, 15], False, False, True),   # the smallest shard decides
    (2, [32, 32], True, False, True),        # --tp forces the hybrid
    (8, [8] * 8, False, True, False),        # --no-tp forces sequence sharding
])
def test_ragged_mode_choice(world, sizes, tp, no_tp, want):
    assert bench.ragged_uses_hybrid(world, sizes, tp, no_tp) is want


def test_reference_arm_json_line():
    """`bench.py --impl reference` on config 1 (the MLP): one JSON line with
    the contract's keys, a positive rate, the CPU sample described, and an e2e
    record that moves no bytes between host and device."""
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "mlp",
           "--steps", "2", "--warmup", "1", "--cpu-budget", "0.5"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "dtype", "data",
                "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["steps"] == 2 and line["n_gpus"] == 1
    assert line["warmup"] == 3  # warm-ups are raised to the timing rules' minimum of 3
    assert line["config"]["workload"] == "config1_swiglu_mlp_b1"
    base = line["cpu_baseline"]
    assert base["kind"] in ("port", "reference") and base["cores"] >= 1 and base["sample"]
    assert base["value"] == line["value"] and base["unit"] == line["unit"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
