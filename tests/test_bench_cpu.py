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


def test_candidate_pairs_counts_the_3x3_neighbourhoods():
    """bench.candidate_pairs: per anchor, the plan entries of the 3x3 cells around its cell, clipped."""
    import types
    import numpy as np
    import torch
    sys.path.insert(0, str(ROOT))
    import bench
    rng = np.random.default_rng(4)
    G, GH, GW = 3, 5, 7
    cnt = torch.as_tensor(rng.integers(0, 9, G * GH * GW))
    cs = torch.cat([torch.zeros(1, dtype=torch.long), cnt.cumsum(0)])
    ac = torch.as_tensor(np.stack([rng.integers(0, G, 50), rng.integers(0, GW, 50), rng.integers(0, GH, 50)], 1))
    plan = types.SimpleNamespace(cell_start=cs, GH=GH, GW=GW, anc_cell=ac)
    c = cnt.view(G, GH, GW).numpy()
    want = sum(int(c[g, max(cy - 1, 0):cy + 2, max(cx - 1, 0):cx + 2].sum()) for g, cx, cy in ac.tolist())
    assert bench.candidate_pairs(plan) == want


def test_compute_roofline_picks_the_binding_term():
    sys.path.insert(0, str(ROOT))
    import bench
    rates = {"fp32_lane_ops": 3.5e13, "fp32x2_lane_ops": 3.7e13, "ex2": 4.6e12, "red_f32": 1.9e11, "red_v4": 1.9e11,
             "smem_atomic": 9.8e11}
    r = bench.compute_roofline("k_pair_bwd", 4e8, 1.6e7, 4.1e8, 0.5, rates)
    assert r["bound"] == "fp32"
    assert abs(r["terms_ms"]["fp32"] - 4e8 * 16 / 3.7e13 * 1e3) < 1e-9
    assert abs(r["frac"] - r["t_roof_ms"] / 0.5) < 1e-12
    slow_red = dict(rates, red_v4=1e10)  # 1.6e7 reductions at 1e10/s = 1.6 ms binds
    assert bench.compute_roofline("k_pair_bwd", 4e8, 1.6e7, 4.1e8, 0.5, slow_red)["bound"] == "red"
    assert "red" not in bench.compute_roofline("k_pair_fwd", 4e8, 1.6e7, 2.9e8, 0.5, rates)["terms_ms"]
