"""bench.py's reference arm on CPU: the reference's own AnchoredExact + OpenMP kernels (baseline/_ref and
oracle/_ref) on a small window, printing the contract's JSON line."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_contract_line():
    if not (ROOT / "baseline" / "_ref" / "atl").is_dir() or not list((ROOT / "oracle" / "_ref").glob("*.so")):
        pytest.skip("reference install / its compiled CPU kernels not present")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--events", "3000", "--steps",
                        "2", "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    if "unavailable" in line:
        pytest.skip(line["unavailable"])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "config",
              "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["value"] > 0 and line["unit"] == "events/s"
    assert line["cpu_baseline"]["kind"] == "reference" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0
