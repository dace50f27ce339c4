"""PixelTrajectories transport on the device (atlb_traj_transport / _bwd): against the reference's own
transport outputs (tests/golden/traj_*.npz, written by the reference's atl/motion/trajectories.py), and
against the torch restatement of the same module with the kernels bypassed.  Positions and the gradient
w.r.t. the coefficient grid, Bezier and polynomial bases, scalar and per-event target times, border
clamping of the coefficient samples.  Also the trainer's loss (configuration 5b): AnchoredExact with
PixelTrajectories(K=1, polynomial) against the reference's outputs."""
import math

import numpy as np
import pytest
import torch

from tests.goldens import load
from tests.parity import assert_grad_parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["traj_k10_bezier", "traj_k3_poly_pe", "traj_k1_poly", "traj_k4_bezier_pe"])
def test_traj_transport_vs_reference(name):
    """Positions within 1e-5 relative of the reference's (the fixed-point iterates round in another order),
    the coefficient gradient within 1e-5 norm-wise."""
    from x_b200.motion import PixelTrajectories
    g = load(name)
    dev = "cuda"
    T = lambda a: torch.as_tensor(np.asarray(a)).to(dev).contiguous()  # noqa: E731
    K = int(g["K"])
    c = T(g["coeff"]).requires_grad_(True)
    m = PixelTrajectories(c, K, basis_kind=str(g["basis"]), tile=4)
    xy, t, b = T(g["xy"]), T(g["t"]), T(g["b"])
    assert m._device_transport(xy, t)
    t_dst = T(g["t_dst"]) if bool(g["per_event"]) else float(g["t_dst"])
    y = m.transport(xy, t, t_dst, b)
    (y * T(g["w"])).sum().backward()
    np.testing.assert_allclose(y.detach().cpu().numpy(), g["y"], rtol=1e-5, atol=1e-5)
    e = assert_grad_parity(c.grad.cpu().numpy(), g["grad"], what=f"{name} coefficient gradient")
    assert e["max_over_max"] <= 1e-5, e


def test_anchored_exact_pixel_trajectories_k1_vs_reference():
    """Configuration 5b's loss, the trainer's call (atl/train/trainer.py:167): AnchoredExact over a batch of
    windows with PixelTrajectories(K=1, "polynomial") motion (linear at the event), against the reference's
    per-anchor scores, loss and coefficient gradient on identical seeded inputs."""
    from x_b200.events import EventPacket
    from x_b200.motion import PixelTrajectories
    from x_b200.objectives import AnchoredExact
    g = load("exact_traj_k1")
    dev = "cuda"
    T = lambda a: torch.as_tensor(np.asarray(a)).to(dev).contiguous()  # noqa: E731
    B, H, W = int(g["B"]), int(g["H"]), int(g["W"])
    c = T(g["coeff"]).requires_grad_(True)
    m = PixelTrajectories(c, 1, basis_kind="polynomial", tile=4)
    assert m.linear_at_event
    n = g["t"].shape[0]
    ev = EventPacket(T(g["xy"]), T(g["t"]), torch.ones(n, device=dev), T(g["b"]), B, H, W)
    obj = AnchoredExact(h=float(g["h"]), tau=1.0, n_anchors=None, n_slices=16, seed=int(g["seed"]), visibility=True)
    ls, anchors = obj.log_scores(ev, m)
    np.testing.assert_array_equal(anchors.cpu().numpy(), g["anchors"])
    np.testing.assert_allclose(ls.detach().cpu().numpy(), g["ls"], rtol=1e-5, atol=1e-5)
    loss = -ls.mean()
    loss.backward()
    assert math.isclose(float(loss.detach()), float(g["loss"]), rel_tol=1e-5)
    e = assert_grad_parity(c.grad.cpu().numpy(), g["grad"], what="PixelTrajectories(K=1) coefficient gradient")
    assert e["max_over_max"] <= 1e-5, e


def _torch_transport(coeff, K, basis, xy, t, t_dst, b, velocity=False):
    from tests.torch_reference import trajectory_transport
    td = t_dst if torch.is_tensor(t_dst) else torch.full_like(t, float(t_dst))
    return trajectory_transport(coeff, K, basis, 4, 6, xy, t, td, b, velocity=velocity)


@pytest.mark.parametrize("K,basis,per_event", [(10, "bezier", False), (3, "polynomial", True), (1, "polynomial", False),
                                                (4, "bezier", True)])
def test_traj_transport_matches_torch(K, basis, per_event):
    from x_b200.motion import PixelTrajectories
    g = torch.Generator().manual_seed(K * 7 + per_event)
    B, H, W, n = 2, 48, 64, 20000
    coeff = (torch.nn.functional.avg_pool2d(torch.randn(B, 2 * K, H, W, generator=g), 9, 1, 4) * 10).cuda()
    xy = torch.stack([torch.rand(n, generator=g) * (W + 16) - 8, torch.rand(n, generator=g) * (H + 16) - 8], 1).cuda()
    t = torch.rand(n, generator=g).cuda()
    b = torch.randint(0, B, (n,), generator=g).cuda()
    t_dst = torch.rand(n, generator=g).cuda() if per_event else 0.375
    w = torch.randn(n, 2, generator=g).cuda()
    c1 = coeff.clone().requires_grad_(True)
    m1 = PixelTrajectories(c1, K, basis_kind=basis, tile=4)
    assert m1._device_transport(xy, t)
    y1 = m1.transport(xy, t, t_dst, b)
    (y1 * w).sum().backward()
    c2 = coeff.clone().requires_grad_(True)
    y2 = _torch_transport(c2, K, basis, xy, t, t_dst, b)  # the torch statement of tests/torch_reference.py
    (y2 * w).sum().backward()
    np.testing.assert_allclose(y1.detach().cpu().numpy(), y2.detach().cpu().numpy(), rtol=1e-5, atol=1e-5)
    g1, g2 = c1.grad.cpu().numpy(), c2.grad.cpu().numpy()
    e = assert_grad_parity(g1, g2, what="coefficient gradient vs the torch transport")
    assert e["max_over_max"] <= 1e-5, e


def test_traj_visible_fraction_matches_torch():
    """The fused exposure correction (origin solved once per anchor, one coefficient sample for the 16 check
    times) against the generic computation of atl/objectives/ats.py:31-50 over the same trajectories (16
    transports per anchor, torch sums).  The check positions are identical; a tiny share may differ only if
    an anchor sat exactly on the image border."""
    from x_b200 import synth
    from x_b200.motion import PixelTrajectories
    from x_b200.objectives import visible_fraction
    g = torch.Generator().manual_seed(99)
    B, H, W, K = 2, 48, 64, 10
    ev = synth.textured_window(20000, H, W, duration=0.1, seed=98, batch=B).to("cuda")
    coeff = (torch.nn.functional.avg_pool2d(torch.randn(B, 2 * K, H, W, generator=g), 9, 1, 4) * 4).cuda()
    m1 = PixelTrajectories(coeff, K, basis_kind="bezier", tile=4)

    class Moved:  # the same trajectories seen only through transport: visible_fraction's generic path
        def transport(self, xy, t, t_dst, b):
            return m1.transport(xy, t, t_dst, b)
    m2 = Moved()
    xa = ev.xy + torch.randn(ev.xy.shape, generator=g).cuda()
    for tau in (1.0, 0.3):
        v1 = visible_fraction(m1, xa, ev.t, ev.b, ev, tau).cpu().numpy()
        v2 = visible_fraction(m2, xa, ev.t, ev.b, ev, tau).cpu().numpy()
        close = np.isclose(v1, v2, rtol=1e-6, atol=1e-7)
        assert close.mean() > 0.999


def test_traj_origin_then_from_origin_equals_transport():
    """Solving the origins once (mode 1) and moving them to a target time (mode 2) reproduces the transport
    bit for bit, and the gradient through the two steps equals the direct one (up to summation order)."""
    from x_b200.motion import PixelTrajectories
    g = torch.Generator().manual_seed(5)
    B, H, W, K, n = 2, 48, 64, 10, 20000
    coeff = (torch.nn.functional.avg_pool2d(torch.randn(B, 2 * K, H, W, generator=g), 9, 1, 4) * 8).cuda()
    xy = torch.stack([torch.rand(n, generator=g) * W, torch.rand(n, generator=g) * H], 1).cuda()
    t = torch.rand(n, generator=g).cuda()
    b = torch.randint(0, B, (n,), generator=g).cuda()
    w = torch.randn(3, n, 2, generator=g).cuda()
    c1 = coeff.clone().requires_grad_(True)
    m1 = PixelTrajectories(c1, K, basis_kind="bezier", tile=4)
    ys1 = [m1.transport(xy, t, c, b) for c in (0.1, 0.5, 0.9)]
    sum((y * w[i]).sum() for i, y in enumerate(ys1)).backward()
    c2 = coeff.clone().requires_grad_(True)
    m2 = PixelTrajectories(c2, K, basis_kind="bezier", tile=4)
    p = m2.origin_on_device(xy, t, b)
    ys2 = [m2.from_origin(p, t, c, b) for c in (0.1, 0.5, 0.9)]
    sum((y * w[i]).sum() for i, y in enumerate(ys2)).backward()
    for a, c in zip(ys1, ys2):
        assert torch.equal(a, c)
    g1, g2 = c1.grad.cpu().numpy(), c2.grad.cpu().numpy()
    e = assert_grad_parity(g2, g1, what="coefficient gradient through origins")
    assert e["max_over_max"] <= 1e-5, e


@pytest.mark.parametrize("K,basis", [(10, "bezier"), (3, "polynomial"), (1, "polynomial")])
def test_traj_records_and_targets_equal_transport(K, basis):
    """The batched transports of AnchoredSliced: records (R positions per event, one target time per event)
    and targets (every event to each of T shared times) reproduce the per-position transport bit for bit,
    and their coefficient gradients equal the per-position ones up to summation order.  Positions include
    ones past the image border (clamped coefficient samples)."""
    from x_b200.motion import PixelTrajectories
    g = torch.Generator().manual_seed(6 + K)
    B, H, W, n, R = 2, 48, 64, 8000, 6
    coeff = (torch.nn.functional.avg_pool2d(torch.randn(B, 2 * K, H, W, generator=g), 9, 1, 4) * 8).cuda()
    xy = torch.stack([torch.rand(n, R, generator=g) * (W + 8) - 4, torch.rand(n, R, generator=g) * (H + 8) - 4],
                     2).cuda()
    t = torch.rand(n, generator=g).cuda()
    td = torch.rand(n, generator=g).cuda()
    b = torch.randint(0, B, (n,), generator=g).cuda()
    targets = torch.tensor([0.05, 0.15, 0.35, 0.55, 0.75, 0.95]).cuda()
    wr = torch.randn(n, R, 2, generator=g).cuda()
    wt = torch.randn(targets.numel(), n, 2, generator=g).cuda()

    def run(batched):
        c = coeff.clone().requires_grad_(True)
        m = PixelTrajectories(c, K, basis_kind=basis, tile=4)
        if batched:
            yr = m.transport_records(xy, t, td, b)
            yt = m.transport_targets(xy[:, 0].contiguous(), t, targets, b)
        else:
            yr = m.transport(xy.reshape(-1, 2), t.repeat_interleave(R), td.repeat_interleave(R),
                             b.repeat_interleave(R)).view(n, R, 2)
            yt = torch.stack([m.transport(xy[:, 0].contiguous(), t, float(c_), b) for c_ in targets.tolist()])
        ((yr * wr).sum() + (yt * wt).sum()).backward()
        return yr.detach(), yt.detach(), c.grad.cpu().numpy()

    yr1, yt1, g1 = run(False)
    yr2, yt2, g2 = run(True)
    assert torch.equal(yr1, yr2)
    assert torch.equal(yt1, yt2)
    e = assert_grad_parity(g2, g1, what=f"records / targets coefficient gradient (K={K})")
    assert e["max_over_max"] <= 1e-5, e


def test_traj_velocity_matches_torch():
    """PixelTrajectories(K=1, polynomial).velocity on the device (mode 3: c_1 at the trajectory origin) against
    the torch statement, values within 1e-5 and the coefficient gradient within 1e-5 norm-wise."""
    from x_b200.motion import PixelTrajectories
    g = torch.Generator().manual_seed(77)
    B, H, W, n = 2, 48, 64, 20000
    coeff = (torch.nn.functional.avg_pool2d(torch.randn(B, 2, H, W, generator=g), 9, 1, 4) * 30).cuda()
    xy = torch.stack([torch.rand(n, generator=g) * (W + 16) - 8, torch.rand(n, generator=g) * (H + 16) - 8], 1).cuda()
    t = torch.rand(n, generator=g).cuda()
    b = torch.randint(0, B, (n,), generator=g).cuda()
    w = torch.randn(n, 2, generator=g).cuda()
    c1 = coeff.clone().requires_grad_(True)
    v1 = PixelTrajectories(c1, 1, basis_kind="polynomial", tile=4).velocity(xy, t, b)
    (v1 * w).sum().backward()
    c2 = coeff.clone().requires_grad_(True)
    v2 = _torch_transport(c2, 1, "polynomial", xy, t, 0.0, b, velocity=True)
    (v2 * w).sum().backward()
    np.testing.assert_allclose(v1.detach().cpu().numpy(), v2.detach().cpu().numpy(), rtol=1e-5, atol=1e-5)
    e = assert_grad_parity(c1.grad.cpu().numpy(), c2.grad.cpu().numpy(), what="velocity coefficient gradient")
    assert e["max_over_max"] <= 1e-5, e
