"""AnchoredSliced (atl/objectives/ats.py:108-183) on the library's tiled Gaussian splat and bilinear gather,
against the reference's own outputs on identical seeded inputs (tests/golden/sliced_*.npz): the
continuous-time Bezier PixelTrajectories of configuration 3, the exact (matrix-exponential) Affine flow
and a linear dense flow.  Both sides draw the dequantisation / smoothing noise from the same seeded CPU
generator, so the per-anchor scores compare one to one."""
import ast
import math

import numpy as np
import pytest
import torch

from tests.goldens import load
from tests.parity import assert_grad_parity

pytestmark = pytest.mark.gpu

DEV = "cuda"


def T(a):
    return torch.as_tensor(np.asarray(a)).to(DEV).contiguous()


def np_(t):
    return t.detach().cpu().numpy()


# sliced_affine_exact_f64exp: the reference's objective with torch.linalg.matrix_exp evaluated in float64
# (tests/golden/gen_golden.py); sliced_affine_exact: as the reference runs, with its fp32 matrix_exp, whose
# own error (up to ~1e-4 px here) moves the reference's scores by up to 2.4e-4 and its gradient by 1.9e-4
# norm-wise (measured between the two goldens, both made by the reference)
# sliced_traj_subsets: slices_per_step, n_anchors_per_slice and tau < 1 (sources a subset of the window);
# sliced_affine_plain: no smoothing (self term), no log-determinant, no jitter, no exposure correction;
# sliced_dense_heldout: the held-out split of heldout_score (anchor and source masks, ats.py:204-213)
@pytest.mark.parametrize("name", ["sliced_trajectories", "sliced_affine_exact_f64exp", "sliced_affine_exact",
                                  "sliced_dense", "sliced_traj_subsets", "sliced_affine_plain",
                                  "sliced_dense_heldout"])
def test_anchored_sliced_vs_reference(name):
    from x_b200 import motion as Mo
    from x_b200.events import EventPacket
    from x_b200.objectives import AnchoredSliced
    g = load(name)
    kind = str(g["kind"])
    B, H, W = int(g["B"]), int(g["H"]), int(g["W"])
    if kind == "trajectories":
        param = T(g["param"]).requires_grad_(True)
        m = Mo.PixelTrajectories(param, int(g["K"]), basis_kind="bezier", tile=4)
    elif kind in ("affine_exact", "affine_linear"):
        m = Mo.Affine(B, H, W, mode="exact" if kind == "affine_exact" else "linear", init=T(g["param"])).to(DEV)
        param = m.theta
    else:
        m = Mo.DenseLinearFlow(B, H, W, grid=(H, W), mode="linear", init=T(g["param"])).to(DEV)
        param = m.grid
    n = g["t"].shape[0]
    ev = EventPacket(T(g["xy"]), T(g["t"]), torch.ones(n, device=DEV), T(g["b"]), B, H, W)
    kw = ast.literal_eval(str(g["obj_kw"])) if "obj_kw" in g else {}
    obj = AnchoredSliced(n_slices=int(g["S"]), sigma=float(g["sigma"]), seed=int(g["seed"]), **kw)
    held = T(g["held"]) if "held" in g else None
    ls, idx = obj.log_scores(ev, m, anchor_mask=held, source_mask=None if held is None else ~held)
    np.testing.assert_array_equal(np_(idx), g["idx"])
    # splat sums in another order and with separable exponentials: scores within 1e-5
    fp32_exp = name == "sliced_affine_exact"
    if fp32_exp:
        # the device flow is within 2e-6 px of float64; the reference's fp32 matrix_exp error enters the
        # finite-difference log-determinant (ats.py:154-157, delta = 0.5) of a few anchors in 1e3
        off = ~np.isclose(np_(ls), g["ls"], rtol=1e-5, atol=2e-5)
        assert off.mean() <= 1e-3, off.sum()
        np.testing.assert_allclose(np_(ls), g["ls"], rtol=1e-4, atol=1e-4)
    else:
        np.testing.assert_allclose(np_(ls), g["ls"], rtol=1e-5, atol=2e-5)
    loss = -ls.mean()
    loss.backward()
    assert math.isclose(float(loss.detach()), float(g["loss"]), rel_tol=1e-5)  # the mean hides single anchors
    # the reference's gradient is an fp32 sum in another order: norm-wise within 1e-5, and no element off by
    # more than 1e-5 of the largest
    tol = 3e-4 if fp32_exp else 1e-5
    e = assert_grad_parity(np_(param.grad), g["grad"], rtol=tol, what=f"{name} parameter gradient")
    assert e["max_over_max"] <= tol, e


def test_count_keys_matches_bincount():
    """atlb_count_keys against torch.bincount: sorted and shuffled keys, keys outside [0, nbins), mask rows."""
    from x_b200.objectives import count_keys
    g = torch.Generator().manual_seed(21)
    n, nbins, R = 300_000, 37, 5
    key = torch.sort(torch.randint(-3, nbins + 3, (n,), generator=g)).values
    mask = (torch.rand(R, n, generator=g) < 0.6).float()
    for k in (key, key[torch.randperm(n, generator=g)]):
        kc, mc = k.to(DEV), mask.to(DEV)
        ok = (k >= 0) & (k < nbins)
        ref = torch.bincount(k[ok], minlength=nbins)
        assert torch.equal(count_keys(kc, nbins).cpu(), ref)
        got = count_keys(kc, nbins, mc).cpu()
        for r in range(R):
            assert torch.equal(got[r], torch.bincount(k[ok], weights=mask[r][ok], minlength=nbins).long())
    assert count_keys(torch.zeros(0, dtype=torch.long, device=DEV), 4).sum() == 0


def test_splat_slices_matches_splat():
    """The stacked splat of T point sets equals T separate splats, and its position gradient (reusing the
    forward's buckets) equals theirs; zero weights add nothing and get zero gradient."""
    from x_b200.functional import splat, splat_slices
    g = torch.Generator().manual_seed(22)
    T_, n, B, H, W, sigma = 3, 20000, 2, 40, 72, 1.5
    pos = torch.stack([torch.rand(T_, n, generator=g) * (W + 10) - 5, torch.rand(T_, n, generator=g) * (H + 10) - 5],
                      2).to(DEV)
    w = (torch.rand(T_, n, generator=g) < 0.7).float().to(DEV)
    b = torch.sort(torch.randint(0, B, (n,), generator=g)).values.to(DEV)
    gimg = torch.randn(T_ * B, H, W, generator=g).to(DEV)
    p1 = pos.clone().requires_grad_(True)
    img1 = splat_slices(p1, w, b, B, H, W, sigma)
    (img1 * gimg).sum().backward()
    p2 = pos.clone().requires_grad_(True)
    img2 = torch.cat([splat(p2[j], w[j], b, B, H, W, kernel="gauss", sigma=sigma) for j in range(T_)])
    (img2 * gimg).sum().backward()
    torch.testing.assert_close(img1, img2, rtol=1e-6, atol=1e-7)  # tile flushes add in any order
    assert torch.equal(p1.grad, p2.grad)
    assert bool((p1.grad[w == 0] == 0).all())
