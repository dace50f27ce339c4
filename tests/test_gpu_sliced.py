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
