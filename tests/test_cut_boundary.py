"""Pairs at the cut: the acceptance test d^2 <= (cut h)^2 must use the reference's separately rounded
residual r = x_i - (y_j + v_j dt_i) (csrc/atl_cpu.cpp:192-195), not a fused multiply-add.

The plan is crafted: every anchor has one source whose squared distance lies within a few ulps of the cut
and whose acceptance differs between the exact rounding sequence and a contracted fl(y + v dt) -- so any
contraction anywhere in the pair kernels changes S by a whole kernel value (~0.011).  Anchors sit 40 px
apart, further than any transported source can move (|v dt| <= 10 px), so each S_i holds exactly its own
boundary pair.  The CPU test pins the oracle to the exact sequence; the GPU tests run the drop-in forward
(tiled and untiled kernels) and backward against it."""
import numpy as np
import pytest

from tests.parity import assert_grad_parity

f32 = np.float32


def craft(n_slots, seed):
    """Anchor slots on a 40 px lattice and, per slot, one boundary pair whose acceptance flips under a
    contracted y + v dt.  Returns dict(x, y, v, dt, accept) in float32 (accept: exact-sequence verdict)."""
    rng = np.random.default_rng(seed)
    cols = 40
    slot_xy = np.stack([100 + 40 * (np.arange(n_slots) % cols), 100 + 40 * (np.arange(n_slots) // cols)], 1).astype(f32)
    n = 2000 * n_slots
    slot = rng.integers(0, n_slots, n)
    x = slot_xy[slot]
    v = rng.uniform(-20, 20, (n, 2)).astype(f32)
    dt = (rng.integers(-2 ** 19, 2 ** 19, n) * 2.0 ** -20).astype(f32)[:, None]
    ang = rng.uniform(0, 2 * np.pi, n)
    rad = 3.0 + rng.uniform(-3e-7, 3e-7, n)  # d^2 within a few ulps of 9
    off = np.stack([np.cos(ang), np.sin(ang)], 1) * rad[:, None]
    y = (x.astype(np.float64) - v.astype(np.float64) * dt.astype(np.float64) - off).astype(f32)
    # exact: fl(x - fl(y + fl(v dt))); contracted: fl(x - RN(y + v dt)) (the sum is exact in long double)
    r_ex = (x - (y + (v * dt).astype(f32)).astype(f32)).astype(f32)
    ld = np.longdouble
    inner = (y.astype(ld) + v.astype(ld) * dt.astype(ld)).astype(f32)
    r_fm = (x - inner).astype(f32)
    d2 = lambda r: ((r[:, 0] * r[:, 0]).astype(f32) + (r[:, 1] * r[:, 1]).astype(f32)).astype(f32)
    cut2 = f32(9.0)
    acc_ex, acc_fm = d2(r_ex) <= cut2, d2(r_fm) <= cut2
    flip = np.flatnonzero(acc_ex != acc_fm)
    first = {}
    for i in flip:  # first flipping sample of each slot
        first.setdefault(int(slot[i]), int(i))
    keep = np.array([first[k] for k in sorted(first)])
    return {"x": slot_xy[sorted(first)], "y": y[keep], "v": v[keep], "dt": dt[keep, 0], "accept": acc_ex[keep],
            "d2": d2(r_ex)[keep]}


def plan_of(c, batches=1):
    """The reference plan layout for the crafted pairs: one cell per batch grid (GH = GW = S = 1), the pairs
    split evenly over `batches` grids, every source at the slice centre 0.5."""
    K = c["x"].shape[0]
    g = np.arange(K) * batches // K
    order = np.argsort(g, kind="stable")
    counts = np.bincount(g, minlength=batches)
    return {
        "src_y": c["y"][order], "src_v": c["v"][order], "src_t": np.full(K, 0.5, f32),
        "src_id": (K + order).astype(np.int64),
        "cell_start": np.concatenate([[0], np.cumsum(counts)]).astype(np.int64),
        "anc_x": c["x"], "anc_t": (f32(0.5) + c["dt"]).astype(f32),
        "anc_cell": np.stack([g, np.zeros(K, np.int64), np.zeros(K, np.int64)], 1).astype(np.int64),
        "anc_id": np.arange(K, dtype=np.int64), "slice_c": np.array([0.5], f32), "S": 1, "GH": 1, "GW": 1,
    }


def test_oracle_uses_the_exact_rounding_at_the_cut():
    from oracle import oracle as O
    c = craft(300, seed=3)
    assert c["x"].shape[0] >= 250 and c["accept"].any() and (~c["accept"]).any()
    p = plan_of(c)
    S, hits = O.pair_fwd(p, 1.0, 1.0, 3.0)
    assert hits == int(c["accept"].sum())
    expect = np.where(c["accept"], np.exp(-c["d2"].astype(np.float64) / 2.0), 0.0)
    np.testing.assert_allclose(S, expect, rtol=1e-6, atol=0)


@pytest.mark.gpu
@pytest.mark.parametrize("n_slots,batches", [(1000, 2), (1000, 1)])  # tiled kernel; untiled (> 768 anchors a tile)
def test_pair_kernels_exact_at_the_cut(n_slots, batches):
    import torch
    from oracle import oracle as O
    from x_b200 import get_ext
    ext = get_ext()
    c = craft(n_slots, seed=5 + batches)
    p = plan_of(c, batches)
    T = lambda a: torch.as_tensor(np.ascontiguousarray(a)).cuda()
    args = [T(p[k]) for k in ("src_y", "src_v", "src_t", "src_id", "cell_start", "anc_x", "anc_t", "anc_cell",
                              "anc_id", "slice_c")]
    S = ext.ats_pair_fwd(*args, 1, 1, 1, 1.0, 1.0, 3.0).cpu().numpy()
    So, hits = O.pair_fwd(p, 1.0, 1.0, 3.0)
    assert hits == int(c["accept"].sum())
    # a flipped pair moves S_i by exp(-4.5) ~ 0.011; the kernel values themselves agree to ~1e-6
    np.testing.assert_allclose(S, So, rtol=2e-6, atol=1e-7)
    K = c["x"].shape[0]
    gS = np.linspace(0.5, 1.5, K).astype(f32)
    gv = ext.ats_pair_bwd(T(gS), *args, 1, 1, 1, 1.0, 1.0, 3.0, 2 * K).cpu().numpy()
    gvo, gabs, cnt = O.pair_bwd_f64(p, gS, 1.0, 1.0, 3.0, 2 * K)
    assert_grad_parity(gv, gvo, A=gabs, n=cnt[:, None], what="pair gradient at the cut")


@pytest.mark.gpu
def test_pair_fwd_with_ids_beyond_32_bits():
    """Ids outside [0, 2^32) (the reference compares int64 ids): the count pass flags them and every cell
    takes the untiled kernel, which compares all 64 bits.  Source ids that share their low 32 bits with an
    anchor's id must still count; the anchor's own source (same 64-bit id) must not."""
    import torch
    from oracle import oracle as O
    from x_b200 import get_ext
    ext = get_ext()
    c = craft(400, seed=11)
    p = plan_of(c, 2)
    K = c["x"].shape[0]
    base = np.int64(1) << np.int64(33)
    # each anchor's own crafted source keeps the anchor's id (excluded); the others alias in the low 32 bits
    p["anc_id"] = base + np.arange(K, dtype=np.int64)
    order = p["src_id"] - K
    p["src_id"] = np.where(order % 2 == 0, base + order, (np.int64(1) << np.int64(34)) + order).astype(np.int64)
    T = lambda a: torch.as_tensor(np.ascontiguousarray(a)).cuda()
    args = [T(p[k]) for k in ("src_y", "src_v", "src_t", "src_id", "cell_start", "anc_x", "anc_t", "anc_cell",
                              "anc_id", "slice_c")]
    S = ext.ats_pair_fwd(*args, 1, 1, 1, 1.0, 1.0, 3.0).cpu().numpy()
    So, _ = O.pair_fwd(p, 1.0, 1.0, 3.0)
    np.testing.assert_allclose(S, So, rtol=2e-6, atol=1e-7)
    even = (np.arange(K) % 2 == 0)
    assert np.all(So[even] == 0.0)          # own source (same id) excluded
    assert np.any(So[~even] > 0.0)          # low-32-bit aliases counted


@pytest.mark.gpu
def test_pair_ops_fallback_grid():
    """A cell count that is not a whole number of S x GH x GW grids cannot be indexed by the tiled kernels:
    the drop-in ops take the per-cell-warp kernels, with the same results as the oracle."""
    import torch
    from oracle import oracle as O
    from x_b200 import get_ext
    ext = get_ext()
    c = craft(300, seed=13)
    p = plan_of(c, 3)   # 3 one-cell grids ...
    p["S"] = 2          # ... declared as slices of 2: ncell = 3 is not a multiple of S * GH * GW = 2
    T = lambda a: torch.as_tensor(np.ascontiguousarray(a)).cuda()
    args = [T(p[k]) for k in ("src_y", "src_v", "src_t", "src_id", "cell_start", "anc_x", "anc_t", "anc_cell",
                              "anc_id", "slice_c")]
    args[-1] = T(np.array([0.5, 0.5], f32))  # one centre per declared slice
    p["slice_c"] = np.array([0.5, 0.5], f32)
    S = ext.ats_pair_fwd(*args, 2, 1, 1, 1.0, 1.0, 3.0).cpu().numpy()
    So, hits = O.pair_fwd(p, 1.0, 1.0, 3.0)
    assert hits == int(c["accept"].sum())
    np.testing.assert_allclose(S, So, rtol=2e-6, atol=1e-7)
    K = c["x"].shape[0]
    gS = np.linspace(0.5, 1.5, K).astype(f32)
    gv = ext.ats_pair_bwd(T(gS), *args, 2, 1, 1, 1.0, 1.0, 3.0, 2 * K).cpu().numpy()
    gvo, gabs, cnt = O.pair_bwd_f64(p, gS, 1.0, 1.0, 3.0, 2 * K)
    assert_grad_parity(gv, gvo, A=gabs, n=cnt[:, None], what="pair gradient at the cut")
