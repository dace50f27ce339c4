"""Pin the plain-C oracle against the reference's own outputs (tests/golden/*.npz).

Integer outputs (plan keys, CSR offsets, anchor cells, window counts, slice ranges) must match
bit-for-bit; float outputs within the tolerances stated per test."""
import math

import numpy as np
import pytest

from oracle import oracle as O
from tests.goldens import load, plan_of, sort_within_cells

PLANS = ["plan_tau1_s8", "plan_tau02_s16", "plan_tau005_s4", "plan_smooth_fast"]


def test_ops_match_reference():
    g = load("ops")
    B, H, W = g["splat_bilinear"].shape
    sig, R = float(g["sigma"]), int(g["R"])
    np.testing.assert_allclose(O.splat_bilinear_fwd(g["pos"], g["w"], g["b"], B, H, W), g["splat_bilinear"],
                               rtol=1e-6, atol=1e-6)
    gp, gw = O.splat_bilinear_bwd(g["gimg"], g["pos"], g["w"], g["b"])
    np.testing.assert_array_equal(gp, g["splat_bilinear_gpos"]); np.testing.assert_array_equal(gw, g["splat_bilinear_gw"])
    np.testing.assert_allclose(O.splat_gauss_fwd(g["pos"], g["w"], g["b"], B, H, W, sig, R), g["splat_gauss"],
                               rtol=1e-6, atol=1e-6)
    gp, gw = O.splat_gauss_bwd(g["gimg"], g["pos"], g["w"], g["b"], sig, R)
    np.testing.assert_array_equal(gp, g["splat_gauss_gpos"]); np.testing.assert_array_equal(gw, g["splat_gauss_gw"])
    np.testing.assert_array_equal(O.gather_fwd(g["img"], g["pos"], g["b"]), g["gather"])
    gi, gp = O.gather_bwd(g["gval"], g["img"], g["pos"], g["b"])
    np.testing.assert_allclose(gi, g["gather_gimg"], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(gp, g["gather_gpos"])
    np.testing.assert_allclose(O.voxel_grid(g["pos"], g["t"], g["p"], g["b"], B, 5, H, W), g["voxel"],
                               rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name", PLANS)
def test_plan_bit_exact(name):
    g = load(name)
    axy = g["anchor_xy"] if g["anchor_xy"].shape[0] else None
    p = O.build_pair_plan(g["pos"], g["t"], g["v"], g["b"], int(g["B"]), int(g["H"]), int(g["W"]), g["anchors"],
                          float(g["h"]), float(g["tau"]), 3.0, int(g["S"]), anchor_xy=axy)
    assert (p["GH"], p["GW"]) == (int(g["GH"]), int(g["GW"]))
    np.testing.assert_array_equal(p["cell_start"], g["cell_start"])
    ours, ref = sort_within_cells(p), sort_within_cells(plan_of(g))
    for a, b in zip(ours, ref):
        np.testing.assert_array_equal(a, b)
    for k in ("anc_x", "anc_t", "anc_cell", "anc_id", "slice_c"):
        np.testing.assert_array_equal(p[k], g[k], err_msg=k)


@pytest.mark.parametrize("name", PLANS)
def test_pair_fwd_bwd_match_reference(name):
    g = load(name)
    p = plan_of(g)
    h, tau = float(g["h"]), float(g["tau"])
    S, hits = O.pair_fwd(p, h, tau, 3.0)
    np.testing.assert_array_equal(S, g["pair_S"])              # same double accumulation order per anchor
    np.testing.assert_allclose(S, g["brute_S"], rtol=1e-5, atol=1e-5)
    assert hits > 0
    gv = O.pair_bwd(p, g["gS"], h, tau, 3.0, g["pos"].shape[0])
    np.testing.assert_allclose(gv, g["pair_gv"], rtol=1e-5, atol=1e-5)


def test_window_counts_match_reference():
    g = load("window")
    np.testing.assert_array_equal(O.window_counts(g["kat_t"], g["kat_b"], np.arange(6), 0.15), g["kat"])
    assert g["kat"].tolist() == [1, 2, 1, 0, 0, 0]
    for k, tau in enumerate(g["taus"]):
        np.testing.assert_array_equal(O.window_counts(g["t"], g["b"], g["idx"], float(tau)), g[f"tau{k}"])
    np.testing.assert_array_equal(O.window_counts(g["unsorted_t"], g["unsorted_b"], g["unsorted_idx"], 0.1),
                                  g["unsorted"])


@pytest.mark.parametrize("kind", ["translation", "affine", "dense"])
def test_motion_velocity_and_visibility_bit_exact(kind):
    g = load("motion")
    H, W, B = int(g["H"]), int(g["W"]), int(g["B"])
    v = O.velocity(kind, g[f"{kind}_theta"], g["xy"], g["b"], H, W)
    np.testing.assert_array_equal(v, g[f"{kind}_v"])
    ia = g["vis_idx"]
    for tau, key in ((0.3, "tau03"), (1.0, "tau1")):
        vis = O.visible_fraction(kind, g[f"{kind}_theta"], g["xy"][ia], g["t"][ia], g["b"][ia], g["t"], g["b"], B, H,
                                 W, tau)
        np.testing.assert_array_equal(vis, g[f"{kind}_vis_{key}"])


@pytest.mark.parametrize("kind", ["translation", "affine", "dense"])
def test_anchored_exact_objective_matches_reference(kind):
    g = load(f"exact_{kind}")
    B, H, W = int(g["B"]), int(g["H"]), int(g["W"])
    np.testing.assert_array_equal((g["xy"] + (g["u"] - np.float32(0.5))).astype(np.float32), g["xs"])
    r = O.anchored_exact(kind, g["theta"], g["xs"], g["t"], g["b"], B, H, W, g["anchors"], g["xa"], h=float(g["h"]),
                         tau=float(g["tau"]), n_slices=int(g["S"]), visibility=bool(g["visibility"]))
    np.testing.assert_array_equal(r["v"], g["v"])
    np.testing.assert_array_equal(r["S"], g["pair_S"])
    np.testing.assert_array_equal(r["vis"], g["vis"])
    np.testing.assert_allclose(r["ls"], g["ls"], rtol=1e-6, atol=1e-6)
    assert math.isclose(r["loss"], float(g["loss"]), rel_tol=1e-6)
    # the reference's fp32 gradient against the oracle's: both are fp32 sums in different orders (the
    # reference's omp atomics), so norm-wise within the north star's 1e-5
    d = r["grad_theta"].astype(np.float64) - g["grad_theta"]
    assert np.linalg.norm(d) <= 1e-5 * np.linalg.norm(g["grad_theta"].astype(np.float64))
    assert np.abs(d).max() <= 1e-5 * np.abs(g["grad_theta"]).max()
