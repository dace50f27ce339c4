"""The tiled bilinear splat, gather and voxel grid (x_b200/csrc/tile_ops.cu) against the C oracle, and the
separable blur against a torch fp32 convolution.  Sizes cover both tile staging paths: image widths that
are a multiple of 4 (TMA tensor-map copies) and widths that are not (plain loads), partial tiles, points on
and beyond the border (floor corner at -1 and at W-1), non-finite positions and batch indices outside
[0, B).  The gather and both backward passes keep the reference's per-point corner order and rounding, so
they are compared bit for bit."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.parity import assert_grad_parity

pytestmark = pytest.mark.gpu
DEV = "cuda"


def T(a):
    return torch.as_tensor(np.ascontiguousarray(a)).to(DEV)


def np_(t):
    return t.detach().cpu().numpy()


def points(n, B, H, W, seed):
    rng = np.random.default_rng(seed)
    pos = np.stack([rng.uniform(-2.5, W + 1.5, n), rng.uniform(-2.5, H + 1.5, n)], 1).astype(np.float32)
    if n > 6:
        pos[:6] = [[-1.0, 3.0], [W - 1.0, 2.0], [W - 0.5, H - 0.5], [0.0, -1.0], [-0.999, -0.999], [5.5, H - 1.0]]
    if n > 10:
        pos[7] = [np.nan, 1.0]
        pos[8] = [np.inf, 2.0]
    b = rng.integers(0, B, n).astype(np.int64)
    if n > 10:
        b[9] = B  # outside [0, B): touches nothing
    w = rng.uniform(0.1, 1.5, n).astype(np.float32)
    w[::50] = 0.0
    return pos, w, b, rng


@pytest.fixture(scope="module")
def ext():
    from x_b200 import get_ext
    return get_ext()


@pytest.mark.parametrize("n,B,H,W", [(40000, 2, 96, 128), (25000, 3, 70, 101), (5000, 1, 33, 66), (0, 1, 8, 8),
                                     (3000, 2, 17, 5)])
def test_tiled_bilinear_ops_vs_oracle(ext, n, B, H, W):
    pos, w, b, rng = points(n, B, H, W, n + W)
    ok = np.isfinite(pos).all(1) & (b < B)  # the oracle reads out of bounds for these, the library skips them
    img = ext.splat_bilinear_fwd(T(pos), T(w), T(b), B, H, W)
    ref = O.splat_bilinear_fwd(pos[ok], w[ok], b[ok], B, H, W)
    np.testing.assert_allclose(np_(img), ref, rtol=1e-5, atol=1e-6)
    g = rng.normal(size=(B, H, W)).astype(np.float32)
    gp, gw = ext.splat_bilinear_bwd(T(g), T(pos), T(w), T(b))
    ogp, ogw = O.splat_bilinear_bwd(g, pos[ok], w[ok], b[ok])
    np.testing.assert_array_equal(np_(gp)[ok], ogp)  # per point: the reference's corner order and rounding
    np.testing.assert_array_equal(np_(gw)[ok], ogw)
    assert (np_(gp)[~ok] == 0).all() and (np_(gw)[~ok] == 0).all()
    val = ext.gather_bilinear_fwd(T(g), T(pos), T(b))
    np.testing.assert_array_equal(np_(val)[ok], O.gather_fwd(g, pos[ok], b[ok]))
    assert (np_(val)[~ok] == 0).all()
    gv = rng.normal(size=n).astype(np.float32)
    gi, gp2 = ext.gather_bilinear_bwd(T(gv), T(g), T(pos), T(b))
    ogi, ogp2 = O.gather_bwd(gv[ok], g, pos[ok], b[ok])
    np.testing.assert_array_equal(np_(gp2)[ok], ogp2)
    if n:
        e = assert_grad_parity(np_(gi), ogi, what="gather image gradient")
        assert e["max_over_max"] <= 1e-5, e
    t = rng.uniform(-0.05, 1.05, n).astype(np.float32)
    p = np.where(rng.uniform(size=n) < 0.5, -1.0, 1.0).astype(np.float32)
    for C in (5, 20):  # shared-memory channels, and the global fallback above 16 channels
        vox = ext.voxel_grid(T(pos), T(t), T(p), T(b), B, C, H, W)
        np.testing.assert_allclose(np_(vox), O.voxel_grid(pos[ok], t[ok], p[ok], b[ok], B, C, H, W), rtol=1e-5,
                                   atol=1e-6)


@pytest.mark.parametrize("shape,sigma", [((2, 48, 64), 1.0), ((1, 3, 37, 53), 2.5), ((4, 20, 24), 0.3),
                                         ((1, 100, 160), 6.0)])
def test_blur_vs_torch_conv(shape, sigma):
    """The device blur against the reference's construction (atl/ops/functional.py:89-110) run in torch fp32:
    forward within 1e-5, and the gradient through the autograd function equals the adjoint convolution."""
    from x_b200.functional import blur
    torch.manual_seed(0)
    img = torch.randn(shape, device=DEV, requires_grad=True)
    out = blur(img, sigma)
    r = max(int(math.ceil(3 * sigma)), 1)
    xk = torch.arange(-r, r + 1, device=DEV, dtype=torch.float32)
    k = torch.exp(-xk * xk / (2 * sigma * sigma))
    k = k / k.sum()
    x0 = img.detach().clone().requires_grad_(True)
    x = x0[:, None] if x0.dim() == 3 else x0
    C = x.shape[1]
    y = torch.nn.functional.conv2d(x, k.view(1, 1, 1, -1).expand(C, 1, 1, -1), padding=(0, r), groups=C)
    y = torch.nn.functional.conv2d(y, k.view(1, 1, -1, 1).expand(C, 1, -1, 1), padding=(r, 0), groups=C)
    y = y[:, 0] if x0.dim() == 3 else y
    assert out.shape == y.shape
    np.testing.assert_allclose(np_(out), np_(y), rtol=1e-5, atol=1e-6)
    gout = torch.randn_like(out)
    (out * gout).sum().backward()
    (y * gout).sum().backward()
    e = assert_grad_parity(np_(img.grad), np_(x0.grad), what="blur gradient")
    assert e["max_over_max"] <= 1e-5, e
