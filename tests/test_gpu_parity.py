"""Parity of the CUDA path (through the C ABI) with the reference's outputs (golden fixtures) and the
C oracle.  Integer outputs bit-exact; float outputs within the stated tolerances (the reference
north-star tolerance is 1e-5 relative; fp32 atomic accumulation order is not deterministic)."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.goldens import load, plan_of, sort_within_cells
from tests.parity import assert_grad_parity, grad_errors

pytestmark = pytest.mark.gpu

DEV = "cuda"
RTOL = 1e-5


def T(a, dtype=None):
    t = torch.as_tensor(np.asarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(DEV).contiguous()


def np_(t):
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def ext():
    from x_b200 import get_ext
    return get_ext()


# ------------------------------------------------------------------------------------------- splat / gather
def test_ops_match_reference_goldens(ext):
    g = load("ops")
    B, H, W = g["splat_bilinear"].shape
    pos, w, b, t, p = T(g["pos"]), T(g["w"]), T(g["b"]), T(g["t"]), T(g["p"])
    sig, R = float(g["sigma"]), int(g["R"])
    np.testing.assert_allclose(np_(ext.splat_bilinear_fwd(pos, w, b, B, H, W)), g["splat_bilinear"], rtol=RTOL, atol=1e-6)
    gp, gw = ext.splat_bilinear_bwd(T(g["gimg"]), pos, w, b)
    np.testing.assert_array_equal(np_(gp), g["splat_bilinear_gpos"])   # same per-thread rounding order
    np.testing.assert_array_equal(np_(gw), g["splat_bilinear_gw"])
    np.testing.assert_allclose(np_(ext.splat_gauss_fwd(pos, w, b, B, H, W, sig, R)), g["splat_gauss"], rtol=RTOL,
                               atol=1e-6)
    gp, gw = ext.splat_gauss_bwd(T(g["gimg"]), pos, w, b, sig, R)
    np.testing.assert_allclose(np_(gp), g["splat_gauss_gpos"], rtol=RTOL, atol=1e-6)
    np.testing.assert_allclose(np_(gw), g["splat_gauss_gw"], rtol=RTOL, atol=1e-6)
    np.testing.assert_array_equal(np_(ext.gather_bilinear_fwd(T(g["img"]), pos, b)), g["gather"])
    gi, gp = ext.gather_bilinear_bwd(T(g["gval"]), T(g["img"]), pos, b)
    np.testing.assert_allclose(np_(gi), g["gather_gimg"], rtol=RTOL, atol=1e-6)
    np.testing.assert_array_equal(np_(gp), g["gather_gpos"])
    np.testing.assert_allclose(np_(ext.voxel_grid(pos, t, p, b, B, 5, H, W)), g["voxel"], rtol=RTOL, atol=1e-6)


# sigma sweep of configuration 4 (R = 2, 3, 6, 12), a radius beyond the compiled window sizes (R = 15),
# widths that are not multiples of 4 (scalar flush) and of 32 (partial tiles), window centres outside the image
@pytest.mark.parametrize("n,B,H,W,sigma", [(20000, 3, 64, 80, 1.5), (5000, 1, 30, 40, 0.5), (0, 2, 8, 8, 1.0),
                                           (30000, 2, 70, 101, 1.0), (20000, 1, 96, 128, 2.0),
                                           (12000, 2, 64, 64, 4.0), (4000, 1, 50, 75, 5.0)])
def test_splat_gather_vs_oracle(ext, n, B, H, W, sigma):
    rng = np.random.default_rng(n + B)
    R = int(math.ceil(3 * sigma))
    pos = np.stack([rng.uniform(-R - 3, W + R + 3, n), rng.uniform(-R - 3, H + R + 3, n)], 1).astype(np.float32)
    w = rng.uniform(0.1, 1.1, n).astype(np.float32)
    w[::97] = 0.0  # zero weights are skipped by the forward and still get gw in the backward
    b = rng.integers(0, B, n).astype(np.int64)
    img = ext.splat_gauss_fwd(T(pos), T(w), T(b), B, H, W, sigma, R)
    np.testing.assert_allclose(np_(img), O.splat_gauss_fwd(pos, w, b, B, H, W, sigma, R), rtol=RTOL, atol=1e-5)
    gimg = rng.normal(size=(B, H, W)).astype(np.float32)
    gp, gw = ext.splat_gauss_bwd(T(gimg), T(pos), T(w), T(b), sigma, R)
    ogp, ogw = O.splat_gauss_bwd(gimg, pos, w, b, sigma, R)
    if n:
        for got, ref, what in ((np_(gp), ogp, "d pos"), (np_(gw), ogw, "d w")):
            e = assert_grad_parity(got, ref, what=f"Gaussian splat {what}")
            assert e["max_over_max"] <= 1e-5, e
    val = ext.gather_bilinear_fwd(T(gimg), T(pos), T(b))
    np.testing.assert_array_equal(np_(val), O.gather_fwd(gimg, pos, b))


# ------------------------------------------------------------------------------------------- plan + pairs
PLANS = ["plan_tau1_s8", "plan_tau02_s16", "plan_tau005_s4", "plan_smooth_fast"]


def _plan_from_golden(g):
    from x_b200 import functional as F
    axy = T(g["anchor_xy"]) if g["anchor_xy"].shape[0] else None
    return F.build_pair_plan(T(g["pos"]), T(g["t"]), T(g["v"]), T(g["b"]), int(g["B"]), int(g["H"]), int(g["W"]),
                             T(g["anchors"]), float(g["h"]), float(g["tau"]), 3.0, int(g["S"]), anchor_xy=axy)


def _plan_np(p):
    d = {k: np_(getattr(p, k)) for k in ("src_y", "src_v", "src_t", "src_id", "cell_start", "anc_x", "anc_t",
                                         "anc_cell", "anc_id", "slice_c")}
    d.update(S=p.S, GH=p.GH, GW=p.GW)
    return d


@pytest.mark.parametrize("name", PLANS)
def test_device_plan_bit_exact_vs_reference(name):
    g = load(name)
    p = _plan_np(_plan_from_golden(g))
    assert (p["GH"], p["GW"]) == (int(g["GH"]), int(g["GW"]))
    np.testing.assert_array_equal(p["cell_start"], g["cell_start"])
    for a, r in zip(sort_within_cells(p), sort_within_cells(plan_of(g))):
        np.testing.assert_array_equal(a, r)
    for k in ("anc_x", "anc_t", "anc_cell", "anc_id", "slice_c"):
        np.testing.assert_array_equal(p[k], g[k], err_msg=k)


@pytest.mark.parametrize("name", PLANS)
def test_pair_fwd_bwd_vs_reference(ext, name):
    g = load(name)
    pl = plan_of(g)
    args = [T(pl[k]) for k in ("src_y", "src_v", "src_t", "src_id", "cell_start", "anc_x", "anc_t", "anc_cell",
                               "anc_id", "slice_c")]
    h, tau = float(g["h"]), float(g["tau"])
    S = ext.ats_pair_fwd(*args, pl["S"], pl["GH"], pl["GW"], h, tau, 3.0)
    np.testing.assert_allclose(np_(S), g["pair_S"], rtol=RTOL, atol=1e-6)
    n = g["pos"].shape[0]
    gv = np_(ext.ats_pair_bwd(T(g["gS"]), *args, pl["S"], pl["GH"], pl["GW"], h, tau, 3.0, n))
    assert_grad_parity(gv, g["pair_gv"], what="pair gradient vs the reference")
    gv64, gabs, cnt = O.pair_bwd_f64(pl, g["gS"], h, tau, 3.0, n)
    assert_grad_parity(gv, gv64, A=gabs, n=cnt[:, None], what="pair gradient vs the double-accumulated oracle")


def test_ats_pair_sums_autograd_matches_bruteforce_reference():
    """Mirror of the reference's test_ats_pair_matches_bruteforce (tests/test_ops.py:62-77)."""
    from x_b200 import functional as F
    for name in PLANS[:3]:
        g = load(name)
        v = T(g["v"]).requires_grad_(True)
        s = F.ats_pair_sums(T(g["pos"]), T(g["t"]), v, T(g["b"]), int(g["B"]), int(g["H"]), int(g["W"]),
                            T(g["anchors"]), float(g["h"]), float(g["tau"]), 3.0, int(g["S"]))
        np.testing.assert_allclose(np_(s), g["brute_S"], rtol=1e-4, atol=1e-4)
        (s * T(g["gS"])).sum().backward()
        assert_grad_parity(np_(v.grad), g["pair_gv"], what=f"ats_pair_sums autograd ({name})")


@pytest.mark.parametrize("n,tau,S,vs", [(60000, 1.0, 16, 20.0), (40000, 0.1, 8, 5.0), (30000, 0.3, 24, 40.0)])
def test_plan_and_pairs_vs_oracle_larger(ext, n, tau, S, vs):
    from x_b200 import functional as F
    rng = np.random.default_rng(n)
    H, W, B = 96, 128, 2
    xy = np.stack([rng.integers(0, W, n), rng.integers(0, H, n)], 1).astype(np.float32)
    xy += rng.uniform(-0.5, 0.5, xy.shape).astype(np.float32)
    b = np.sort(rng.integers(0, B, n)).astype(np.int64)
    t = np.concatenate([np.sort(rng.uniform(0, 1, (b == k).sum())) for k in range(B)]).astype(np.float32)
    v = (rng.normal(size=(n, 2)) * vs / 3).astype(np.float32)
    anchors = np.sort(rng.choice(n, n // 2, replace=False)).astype(np.int64)
    axy = (xy[anchors] + rng.normal(size=(anchors.size, 2))).astype(np.float32)
    ref = O.build_pair_plan(xy, t, v, b, B, H, W, anchors, 1.0, tau, 3.0, S, anchor_xy=axy)
    p = F.build_pair_plan(T(xy), T(t), T(v), T(b), B, H, W, T(anchors), 1.0, tau, 3.0, S, anchor_xy=T(axy))
    pn = _plan_np(p)
    np.testing.assert_array_equal(pn["cell_start"], ref["cell_start"])
    for a, r in zip(sort_within_cells(pn), sort_within_cells(ref)):
        np.testing.assert_array_equal(a, r)
    np.testing.assert_array_equal(pn["anc_cell"], ref["anc_cell"])
    Sg = ext.ats_pair_fwd(p.src_y, p.src_v, p.src_t, p.src_id, p.cell_start, p.anc_x, p.anc_t, p.anc_cell, p.anc_id,
                          p.slice_c, p.S, p.GH, p.GW, 1.0, tau, 3.0)
    So, hits = O.pair_fwd(ref, 1.0, tau, 3.0)
    assert hits > 0
    np.testing.assert_allclose(np_(Sg), So, rtol=RTOL, atol=1e-6)
    gS = rng.normal(size=anchors.size).astype(np.float32)
    gv = ext.ats_pair_bwd(T(gS), p.src_y, p.src_v, p.src_t, p.src_id, p.cell_start, p.anc_x, p.anc_t, p.anc_cell,
                          p.anc_id, p.slice_c, p.S, p.GH, p.GW, 1.0, tau, 3.0, n)
    gv64, gabs, cnt = O.pair_bwd_f64(ref, gS, 1.0, tau, 3.0, n)
    assert_grad_parity(np_(gv), gv64, A=gabs, n=cnt[:, None], what="pair gradient vs the double-accumulated oracle")


def test_plan_edge_cases():
    """Empty anchors (grid from the image box), no events, a single event, sources outside the grid."""
    from x_b200 import functional as F
    x = T(np.array([[1.0, 2.0], [300.0, -400.0], [5.0, 5.0]], np.float32))
    t = T(np.array([0.1, 0.5, 0.9], np.float32))
    v = T(np.zeros((3, 2), np.float32))
    b = T(np.zeros(3, np.int64))
    for anchors in (np.zeros(0, np.int64), np.array([0], np.int64), np.array([0, 2], np.int64)):
        p = F.build_pair_plan(x, t, v, b, 1, 8, 8, T(anchors), 1.0, 1.0, 3.0, 4)
        ref = O.build_pair_plan(np_(x), np_(t), np_(v), np_(b), 1, 8, 8, anchors, 1.0, 1.0, 3.0, 4)
        np.testing.assert_array_equal(np_(p.cell_start), ref["cell_start"])
        np.testing.assert_array_equal(np_(p.anc_cell), ref["anc_cell"])
    e = F.build_pair_plan(T(np.zeros((0, 2), np.float32)), T(np.zeros(0, np.float32)), T(np.zeros((0, 2), np.float32)),
                          T(np.zeros(0, np.int64)), 1, 8, 8, T(np.zeros(0, np.int64)), 1.0, 1.0, 3.0, 4)
    assert e.src_y.shape[0] == 0 and int(e.cell_start[-1]) == 0


# ------------------------------------------------------------------------------------------- window / motion
def test_window_counts_vs_reference():
    from x_b200 import functional as F
    g = load("window")
    assert F.window_counts(T(g["kat_t"]), T(g["kat_b"]), T(np.arange(6)), 0.15).tolist() == [1, 2, 1, 0, 0, 0]
    for k, tau in enumerate(g["taus"]):
        np.testing.assert_array_equal(np_(F.window_counts(T(g["t"]), T(g["b"]), T(g["idx"]), float(tau))), g[f"tau{k}"])
    out = F.window_counts(T(g["unsorted_t"]), T(g["unsorted_b"]), T(g["unsorted_idx"]), 0.1)
    np.testing.assert_array_equal(np_(out), g["unsorted"])


@pytest.mark.parametrize("kind", ["translation", "affine", "dense"])
def test_velocity_and_visibility_bit_exact(kind):
    from x_b200 import motion as Mo
    from x_b200.events import EventPacket
    from x_b200.objectives import visible_fraction
    g = load("motion")
    B, H, W = int(g["B"]), int(g["H"]), int(g["W"])
    th = T(g[f"{kind}_theta"])
    m = {"translation": lambda: Mo.Translation(B, H, W, init=th), "affine": lambda: Mo.Affine(B, H, W, init=th),
         "dense": lambda: Mo.DenseLinearFlow(B, H, W, grid=(H, W), init=th)}[kind]().to(DEV)
    xy, t, b = T(g["xy"]), T(g["t"]), T(g["b"])
    np.testing.assert_array_equal(np_(m.velocity(xy, t, b)), g[f"{kind}_v"])
    ev = EventPacket(xy, t, torch.ones_like(t), b, B, H, W)
    ia = T(g["vis_idx"])
    for tau, key in ((0.3, "tau03"), (1.0, "tau1")):
        vis = visible_fraction(m, xy[ia], t[ia], b[ia], ev, tau)
        np.testing.assert_array_equal(np_(vis), g[f"{kind}_vis_{key}"])


@pytest.mark.parametrize("kind", ["translation", "affine", "dense"])
def test_velocity_backward_vs_oracle(kind):
    from x_b200 import motion as Mo
    g = load("motion")
    B, H, W = int(g["B"]), int(g["H"]), int(g["W"])
    th = T(g[f"{kind}_theta"])
    m = {"translation": lambda: Mo.Translation(B, H, W, init=th), "affine": lambda: Mo.Affine(B, H, W, init=th),
         "dense": lambda: Mo.DenseLinearFlow(B, H, W, grid=(H, W), init=th)}[kind]().to(DEV)
    gv = np.random.default_rng(1).normal(size=g["xy"].shape).astype(np.float32)
    (m.velocity(T(g["xy"]), T(g["t"]), T(g["b"])) * T(gv)).sum().backward()
    ref = O.velocity_backward(kind, g[f"{kind}_theta"], g["xy"], g["b"], H, W, gv)  # double accumulation
    e = assert_grad_parity(np_(m.theta.grad), ref, what=f"{kind} velocity backward")
    assert e["max_over_max"] <= 1e-5, e


# ------------------------------------------------------------------------------------------- objective
@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("kind", ["translation", "affine", "dense"])
def test_anchored_exact_objective_vs_reference(kind, fused):
    """Mirror of the reference's test_anchored_exact_gradient_matches_reference (tests/test_objectives.py:166-183),
    against the reference's own AnchoredExact outputs on identical seeded inputs."""
    from x_b200 import motion as Mo
    from x_b200.events import EventPacket
    from x_b200.objectives import AnchoredExact
    g = load(f"exact_{kind}")
    B, H, W = int(g["B"]), int(g["H"]), int(g["W"])
    th = T(g["theta"])
    m = {"translation": lambda: Mo.Translation(B, H, W, init=th), "affine": lambda: Mo.Affine(B, H, W, init=th),
         "dense": lambda: Mo.DenseLinearFlow(B, H, W, grid=(H, W), init=th)}[kind]().to(DEV)
    ev = EventPacket(T(g["xy"]), T(g["t"]), torch.ones(g["t"].shape[0], device=DEV), T(g["b"]), B, H, W)
    n_anchors = None if g["anchors"].shape[0] == g["t"].shape[0] else int(g["anchors"].shape[0])
    obj = AnchoredExact(h=float(g["h"]), tau=float(g["tau"]), n_anchors=n_anchors, n_slices=int(g["S"]),
                        seed=int({"translation": 42, "affine": 52, "dense": 62}[kind]),
                        visibility=bool(g["visibility"]), fused=fused)
    anchors, u, z = obj.draw(ev)
    np.testing.assert_array_equal(np_(anchors), g["anchors"])
    np.testing.assert_array_equal(np_(u), g["u"])
    np.testing.assert_array_equal(np_(z), g["z"])
    ls, anc = obj.log_scores(ev, m, noise=(anchors, u, z))
    np.testing.assert_allclose(np_(ls), g["ls"], rtol=RTOL, atol=RTOL)
    loss = -ls.mean()
    loss.backward()
    assert math.isclose(float(loss.detach()), float(g["loss"]), rel_tol=RTOL)
    gr = np_(m.theta.grad)
    assert_grad_parity(gr, g["grad_theta"], what=f"{kind} motion gradient vs the reference")
    # and against the oracle's double-accumulated gradient on the same draws, element by element
    h = np.float32(g["h"])
    xs = (g["xy"] + (np_(u) - np.float32(0.5))).astype(np.float32)
    xa = (xs[np_(anchors)] + h * np_(z)).astype(np.float32)
    ref = O.anchored_exact(kind, g["theta"], xs, g["t"], g["b"], B, H, W, np_(anchors), xa, h=float(g["h"]),
                           tau=float(g["tau"]), n_slices=int(g["S"]), visibility=bool(g["visibility"]), exact_grad=True)
    assert_grad_parity(gr, ref["grad_theta64"], A=ref["grad_theta_abs"], n=ref["grad_theta_terms"],
                       what=f"{kind} motion gradient vs the double-accumulated oracle")


def test_fused_matches_stagewise_unsorted_fallback():
    """Unsorted events: the fused pipeline declines and the stage-by-stage path (which sorts the window
    keys like the reference) gives the same scores as the oracle."""
    from x_b200 import motion as Mo
    from x_b200.events import EventPacket
    from x_b200.objectives import AnchoredExact
    g = load("exact_translation")
    B, H, W = int(g["B"]), int(g["H"]), int(g["W"])
    n = g["t"].shape[0]
    perm = np.random.default_rng(0).permutation(n)
    ev = EventPacket(T(g["xy"][perm]), T(g["t"][perm]), torch.ones(n, device=DEV), T(g["b"][perm]), B, H, W)
    m = Mo.Translation(B, H, W, init=T(g["theta"])).to(DEV)
    obj = AnchoredExact(h=1.0, n_anchors=None, seed=3)
    anchors, u, z = obj.draw(ev)
    ls, _ = obj.log_scores(ev, m, noise=(anchors, u, z))
    xs = (g["xy"][perm] + (np_(u) - np.float32(0.5))).astype(np.float32)
    xa = (xs[np_(anchors)] + np_(z)).astype(np.float32)
    ref = O.anchored_exact("translation", g["theta"], xs, g["t"][perm], g["b"][perm], B, H, W, np_(anchors), xa,
                           with_grad=False)
    np.testing.assert_allclose(np_(ls), ref["ls"], rtol=RTOL, atol=RTOL)


@pytest.mark.parametrize("n,box", [(20000, 6.0), (6000, 40.0)])
def test_fused_dense_clusters_vs_oracle(n, box):
    """Events packed into a few pixels: tiles overflow their shared-memory staging (global-memory paths of
    the tiled forward/backward and the overflow pass) and still match the oracle."""
    from x_b200 import motion as Mo
    from x_b200.events import EventPacket
    from x_b200.objectives import AnchoredExact
    rng = np.random.default_rng(5)
    H, W = 64, 96
    xy = np.stack([rng.integers(40, 40 + int(box), n), rng.integers(20, 20 + int(box), n)], 1).astype(np.float32)
    t = np.sort(rng.uniform(0, 1, n)).astype(np.float32)
    b = np.zeros(n, np.int64)
    th = np.array([[3.0, -2.0]], np.float32)
    ev = EventPacket(T(xy), T(t), torch.ones(n, device=DEV), T(b), 1, H, W)
    m = Mo.Translation(1, H, W, init=T(th)).to(DEV)
    obj = AnchoredExact(h=1.0, n_anchors=None, seed=9)
    anchors, u, z = obj.draw(ev)
    ls, _ = obj.log_scores(ev, m, noise=(anchors, u, z))
    (-ls.mean()).backward()
    xs = (xy + (np_(u) - np.float32(0.5))).astype(np.float32)
    xa = (xs[np_(anchors)] + np_(z)).astype(np.float32)
    ref = O.anchored_exact("translation", th, xs, t, b, 1, H, W, np_(anchors), xa, exact_grad=True)
    np.testing.assert_allclose(np_(ls), ref["ls"], rtol=RTOL, atol=RTOL)
    assert_grad_parity(np_(m.theta.grad), ref["grad_theta64"], A=ref["grad_theta_abs"], n=ref["grad_theta_terms"],
                       what="dense-cluster translation gradient")
