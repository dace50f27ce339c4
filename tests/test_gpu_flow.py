"""Exact transport of the affine fields on the device (atlb_flow_exact / _bwd, mode="exact" of Translation and
Affine, atl/motion/parametric.py:60-71) against a torch float64 evaluation of the same formula
(torch.linalg.matrix_exp of the augmented matrix; in fp32, as the reference calls it, matrix_exp itself is off
by up to ~1e-4 px on these inputs): positions within 1e-5 relative, and the gradients w.r.t. theta and the
positions within 1e-5 norm-wise.  Scalar and per-event target times, large and tiny |A dt|, an event
whose batch index is outside [0, B)."""
import numpy as np
import pytest
import torch

from tests.parity import assert_grad_parity

pytestmark = pytest.mark.gpu


def torch_flow(theta, xy, t, t_dst, b, kind, H, W):
    c = torch.tensor([(W - 1) / 2.0, (H - 1) / 2.0], device=xy.device, dtype=xy.dtype)
    th = theta[b]
    n = xy.shape[0]
    Z = torch.zeros(n, 3, 3, device=xy.device, dtype=xy.dtype)
    Z[:, :2, 2] = th[:, :2]
    if kind == "affine":
        Z[:, :2, :2] = th[:, 2:6].view(-1, 2, 2)
    dt = (t_dst if torch.is_tensor(t_dst) else torch.full_like(t, t_dst)) - t
    E = torch.linalg.matrix_exp(Z * dt[:, None, None])
    return c + torch.bmm(E[:, :2, :2], (xy - c)[..., None])[..., 0] + E[:, :2, 2]


@pytest.mark.parametrize("kind,scale,per_event", [("affine", 0.05, False), ("affine", 2.0, True),
                                                  ("translation", 1.0, True), ("affine", 1e-6, False)])
def test_flow_exact_vs_torch(kind, scale, per_event):
    from x_b200 import motion as Mo
    g = torch.Generator().manual_seed(7)
    B, H, W, n = 3, 64, 96, 20000
    np_ = 6 if kind == "affine" else 2
    th0 = torch.cat([torch.randn(B, 2, generator=g) * 20, torch.randn(B, np_ - 2, generator=g) * scale], 1)
    xy = torch.stack([torch.rand(n, generator=g) * W, torch.rand(n, generator=g) * H], 1).cuda()
    t = torch.rand(n, generator=g).cuda()
    b = torch.randint(0, B, (n,), generator=g).cuda()
    t_dst = torch.rand(n, generator=g).cuda() if per_event else 0.3
    gy = torch.randn(n, 2, generator=g).cuda()
    cls = Mo.Affine if kind == "affine" else Mo.Translation
    m = cls(B, H, W, mode="exact", init=th0).cuda()
    xg = xy.clone().requires_grad_(True)
    y = m.transport(xg, t, t_dst, b)
    (y * gy).sum().backward()
    th = th0.clone().cuda().double().requires_grad_(True)
    xr = xy.clone().double().requires_grad_(True)
    td = t_dst.double() if torch.is_tensor(t_dst) else t_dst
    yr = torch_flow(th, xr, t.double(), td, b, kind, H, W)
    (yr * gy.double()).sum().backward()
    # fp32 rounding of terms as large as the largest position (|A dt| up to ~6 in the stress case expands
    # (x - c) e^(A dt)), so the absolute part scales with the output's magnitude
    yn = yr.detach().cpu().numpy()
    np.testing.assert_allclose(y.detach().cpu().numpy(), yn, rtol=1e-5, atol=2e-6 * np.abs(yn).max())
    assert_grad_parity(m.theta.grad.cpu().numpy(), th.grad.cpu().numpy(), what=f"{kind} theta gradient")
    assert_grad_parity(xg.grad.cpu().numpy(), xr.grad.cpu().numpy(), what=f"{kind} position gradient")


def test_flow_exact_bad_batch_index():
    from x_b200 import motion as Mo
    m = Mo.Affine(1, 8, 8, mode="exact", init=torch.zeros(1, 6)).cuda()
    xy = torch.tensor([[1.0, 2.0], [3.0, 4.0]], device="cuda")
    y = m.transport(xy, torch.zeros(2, device="cuda"), 0.5, torch.tensor([0, 1], device="cuda"))
    assert torch.equal(y[0], xy[0]) and torch.isnan(y[1]).all()


def test_dense_rk4_matches_torch():
    """DenseLinearFlow(mode="exact") on the device (atlb_flow_rk4: RK4 of the bilinear grid field) against the
    torch statement of the same integration: positions within 1e-5, the grid gradient within 1e-5
    norm-wise; positions past the border (clamped samples), scalar and per-event target times."""
    from tests.parity import assert_grad_parity
    from tests.torch_reference import dense_rk4
    from x_b200 import motion as Mo
    g = torch.Generator().manual_seed(5)
    B, H, W, n, steps = 2, 40, 56, 20000, 4
    grid0 = torch.nn.functional.avg_pool2d(torch.randn(B, 2, H // 4, W // 4, generator=g), 3, 1, 1) * 25
    xy = torch.stack([torch.rand(n, generator=g) * (W + 10) - 5, torch.rand(n, generator=g) * (H + 10) - 5],
                     1).cuda()
    t = torch.rand(n, generator=g).cuda()
    b = torch.randint(0, B, (n,), generator=g).cuda()
    w = torch.randn(n, 2, generator=g).cuda()
    for t_dst in (0.625, torch.rand(n, generator=g).cuda()):
        m = Mo.DenseLinearFlow(B, H, W, grid=(H // 4, W // 4), mode="exact", init=grid0, rk4_steps=steps).cuda()
        y1 = m.transport(xy, t, t_dst, b)
        (y1 * w).sum().backward()
        g2 = grid0.clone().cuda().requires_grad_(True)
        td = t_dst if torch.is_tensor(t_dst) else torch.full_like(t, t_dst)
        y2 = dense_rk4(g2, H, W, xy, t, td, b, steps)
        (y2 * w).sum().backward()
        np.testing.assert_allclose(y1.detach().cpu().numpy(), y2.detach().cpu().numpy(), rtol=1e-5, atol=1e-4)
        e = assert_grad_parity(m.grid.grad.cpu().numpy(), g2.grad.cpu().numpy(), what="RK4 grid gradient")
        assert e["max_over_max"] <= 1e-5, e
