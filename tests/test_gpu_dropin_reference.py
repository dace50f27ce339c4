"""The drop-in claim exercised through the reference's own code: the reference package (``atl``, an
unmodified install) gets this library as its extension for CUDA tensors -- installed where its loader keeps
the module it returns (atl/ops/_ext.py:16-42), with its own OpenMP module still serving CPU tensors -- and
its unchanged AnchoredExact / AnchoredSliced, motion models and autograd functions then run on CUDA tensors
through libatlb200.  Their scores, losses and gradients are compared with the same objectives evaluated on
the CPU through the reference's OpenMP kernels, on identical seeded inputs (both objectives draw their noise
from their own CPU generators with the same seed).  Skipped where the reference is not installed."""
import math

import numpy as np
import pytest
import torch

from tests.parity import assert_grad_parity

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def atl():
    from oracle.refload import load_reference
    try:
        mod = load_reference()
    except ImportError as e:
        pytest.skip(f"reference not installed here: {e}")
    import atl.ops._ext as ref_ext
    import atl.ops.functional as ref_fn
    from x_b200 import functional as xf
    from x_b200 import get_ext
    cpu_ext, cuda_ext = ref_ext._EXT, get_ext()
    ref_plan = ref_fn.build_pair_plan

    def build_pair_plan(x, *args, **kw):
        """CUDA tensors: the device plan builder (bit-identical cells to the reference's CPU plan); CPU tensors:
        the reference's own.  The reference's torch plan on CUDA tensors would divide by the cell size as a
        multiplication by its reciprocal (torch's CUDA kernel for a division by a scalar), which moves an
        entry to a neighbouring cell now and then; its CPU plan divides."""
        return (xf.build_pair_plan if x.is_cuda else ref_plan)(x, *args, **kw)

    class Dispatch:
        """The object atl.ops._ext.get_ext() returns: CUDA tensors -> libatlb200, CPU tensors -> the reference's
        OpenMP module (the routing INTEGRATION.md section 1 describes)."""
        with_cuda = True

        def __getattr__(self, name):
            def call(*args):
                dev = next(a for a in args if torch.is_tensor(a))
                return getattr(cuda_ext if dev.is_cuda else cpu_ext, name)(*args)
            return call

    ref_ext._EXT, ref_ext._TRIED = Dispatch(), True
    ref_fn.build_pair_plan = build_pair_plan
    yield mod
    ref_ext._EXT = cpu_ext
    ref_fn.build_pair_plan = ref_plan


def _window(seed, n, H, W, B=1):
    g = torch.Generator().manual_seed(seed)
    xy = torch.stack([torch.randint(0, W, (n,), generator=g), torch.randint(0, H, (n,), generator=g)], 1).float()
    b = torch.sort(torch.randint(0, B, (n,), generator=g)).values
    t = torch.rand(n, generator=g)
    order = torch.argsort(b.double() * 4 + t.double())
    return xy[order], t[order], b[order]


def _run(obj, ev, m, param):
    ls, _ = obj.log_scores(ev, m)
    loss = -ls.mean()
    loss.backward()
    return ls.detach().cpu().numpy(), float(loss.detach()), param.grad.detach().cpu().numpy()


@pytest.mark.parametrize("kind", ["dense", "affine"])
def test_reference_anchored_exact_on_libatlb200(atl, kind):
    from atl.core.events import EventPacket
    from atl.motion import Affine, DenseLinearFlow
    from atl.objectives import AnchoredExact
    H, W, n = 64, 96, 20000
    xy, t, b = _window(3, n, H, W)
    g = torch.Generator().manual_seed(4)
    out = {}
    for dev in ("cpu", "cuda"):
        ev = EventPacket(xy.to(dev), t.to(dev), torch.ones(n, device=dev), b.to(dev), 1, H, W)
        if kind == "dense":
            init = torch.nn.functional.avg_pool2d(torch.randn(1, 2, H, W, generator=torch.Generator().manual_seed(5)),
                                                  9, 1, 4) * 40
            m = DenseLinearFlow(1, H, W, grid=(H, W), mode="linear", init=init).to(dev)
            param = m.grid
        else:
            init = torch.tensor([[6.0, -4.0, 0.03, -0.02, 0.01, 0.04]])
            m = Affine(1, H, W, mode="linear", init=init).to(dev)
            param = m.theta
        obj = AnchoredExact(h=1.0, tau=1.0, n_anchors=None, n_slices=16, seed=9, visibility=True)
        out[dev] = _run(obj, ev, m, param)
    (ls_c, loss_c, g_c), (ls_g, loss_g, g_g) = out["cpu"], out["cuda"]
    if kind == "affine":
        np.testing.assert_allclose(ls_g, ls_c, rtol=1e-5, atol=1e-5)
    else:
        # the reference's DenseLinearFlow samples its grid at x / (W - 1) (Wg - 1): torch's CUDA kernel for the
        # division by a scalar multiplies by the reciprocal, so a velocity can differ from the CPU one in its
        # last bit, and a pair at the cut can then be accepted on one device only (a few anchors in 1e4)
        off = ~np.isclose(ls_g, ls_c, rtol=1e-5, atol=1e-5)
        assert off.mean() <= 1e-3, off.sum()
        np.testing.assert_allclose(ls_g, ls_c, rtol=1e-3, atol=1e-2)
    assert math.isclose(loss_g, loss_c, rel_tol=1e-5)
    # dense: the same few anchors, and torch's own CUDA backward of the grid sample, move the flow gradient
    e = assert_grad_parity(g_g, g_c, rtol=1e-5 if kind == "affine" else 1e-3,
                           what=f"reference AnchoredExact ({kind}) on libatlb200 vs its CPU path")
    assert e["max_over_max"] <= (1e-5 if kind == "affine" else 1e-3), e


def test_reference_anchored_sliced_on_libatlb200(atl):
    from atl.core.events import EventPacket
    from atl.motion import PixelTrajectories
    from atl.objectives import AnchoredSliced
    H, W, n, B, K = 48, 64, 6000, 2, 3
    xy, t, b = _window(11, n, H, W, B)
    coeff0 = torch.nn.functional.avg_pool2d(torch.randn(B, 2 * K, H, W, generator=torch.Generator().manual_seed(12)),
                                            9, 1, 4) * 10
    out = {}
    for dev in ("cpu", "cuda"):
        ev = EventPacket(xy.to(dev), t.to(dev), torch.ones(n, device=dev), b.to(dev), B, H, W)
        c = coeff0.clone().to(dev).requires_grad_(True)
        m = PixelTrajectories(c, K, basis_kind="bezier", tile=4)
        obj = AnchoredSliced(n_slices=4, sigma=1.5, seed=13)
        out[dev] = _run(obj, ev, m, c)
    (ls_c, loss_c, g_c), (ls_g, loss_g, g_g) = out["cpu"], out["cuda"]
    np.testing.assert_allclose(ls_g, ls_c, rtol=1e-5, atol=2e-5)
    assert math.isclose(loss_g, loss_c, rel_tol=1e-5)
    # the motion here is the reference's torch code on both devices (CUDA vs CPU kernels of torch itself)
    e = assert_grad_parity(g_g, g_c, rtol=1e-4, what="reference AnchoredSliced on libatlb200 vs its CPU path")
    assert e["max_over_max"] <= 1e-4, e
