"""Parity at the other BASELINE configurations (the fused CUDA pipeline against the C oracle):

* configuration 1 at full size: 100k events (integer pixels uniform over 240x180, times over 50 ms),
  2-DOF Translation at (vx, vy) ~ U(-30, 30) px/s over the window, h = 1, dequantisation, exposure on;
* configuration 4 at reduced size (200k of the 4M events, same 640x480 sensor and densities of scene
  and noise events): 6-DOF Affine with A = I + U(-0.05, 0.05) mapped to the velocity field A - I and
  t ~ U(-20, 20) px, 30 % uniform noise events, kernel widths h in {0.5, 1, 2, 4}.
Seeded synthetic inputs stand in for the datasets (x_b200.synth)."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _check(ev, motion, kind, theta, obj, rtol_grad=1e-3):
    anchors, u, z = obj.draw(ev)
    motion.theta.grad = None
    ls, _ = obj.log_scores(ev, motion, noise=(anchors, u, z))
    loss = -ls.mean()
    loss.backward()
    xs = (ev.xy + (u - 0.5)).cpu().numpy()
    a = anchors.cpu().numpy()
    xa = (xs[a] + obj.h * z.cpu().numpy()).astype(np.float32)
    ref = O.anchored_exact(kind, theta, xs, ev.t.cpu().numpy(), ev.b.cpu().numpy(), ev.batch_size, ev.height,
                           ev.width, a, xa, h=obj.h, tau=obj.tau, n_slices=obj.n_slices)
    assert math.isclose(float(loss.detach()), ref["loss"], rel_tol=1e-5)
    np.testing.assert_allclose(ls.detach().cpu().numpy(), ref["ls"], rtol=1e-5, atol=1e-5)
    g = motion.theta.grad.cpu().numpy()
    np.testing.assert_allclose(g, ref["grad_theta"], rtol=rtol_grad, atol=1e-4 * np.abs(ref["grad_theta"]).max())


def test_config1_translation_full_size():
    from x_b200 import synth
    from x_b200.motion import Translation
    from x_b200.objectives import AnchoredExact
    ev = synth.uniform_window(100_000, 180, 240, duration=0.05, seed=11, device="cuda")
    g = torch.Generator().manual_seed(12)
    v = (torch.rand(1, 2, generator=g) * 60 - 30) * 0.05  # px/s over a 50 ms window -> px per window
    m = Translation(1, 180, 240, init=v).cuda()
    obj = AnchoredExact(h=1.0, tau=1.0, n_anchors=None, n_slices=16, seed=13, visibility=True)
    _check(ev, m, "translation", v.numpy(), obj)


def _config4_window(n, seed):
    from x_b200 import synth
    from x_b200.events import EventPacket
    H, W = 480, 640
    scene = synth.textured_window(int(n * 0.7), H, W, duration=0.1, seed=seed)
    noise = synth.uniform_window(n - int(n * 0.7), H, W, duration=0.1, seed=seed + 1)
    xy = torch.cat([scene.xy, noise.xy])
    t = torch.cat([scene.t, noise.t])
    order = torch.argsort(t)
    p = torch.ones(n)
    return EventPacket(xy[order], t[order], p, torch.zeros(n, dtype=torch.long), 1, H, W).to("cuda")


@pytest.mark.parametrize("h", [0.5, 1.0, 2.0, 4.0])
def test_config4_affine_sigma_sweep(h):
    from x_b200.motion import Affine
    from x_b200.objectives import AnchoredExact
    ev = _config4_window(200_000, 400)
    g = torch.Generator().manual_seed(401)
    th = torch.cat([torch.rand(1, 2, generator=g) * 40 - 20, torch.rand(1, 4, generator=g) * 0.1 - 0.05], 1)
    m = Affine(1, 480, 640, init=th).cuda()
    obj = AnchoredExact(h=h, tau=1.0, n_anchors=None, n_slices=16, seed=402, visibility=True)
    _check(ev, m, "affine", th.numpy(), obj)
