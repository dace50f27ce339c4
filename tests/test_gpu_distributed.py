"""The source-sharded anchored score (x_b200/distributed.py) on one device: the ranks of a multi-GPU run
are emulated one after another, their partial sums and gradients added, and the result compared with the
single-GPU fused pipeline.  Configuration-5 style input (textured window, dense flow), reduced size."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def window():
    from x_b200 import synth
    from x_b200.motion import DenseLinearFlow
    from x_b200.objectives import AnchoredExact
    H, W = 96, 128
    ev = synth.textured_window(40000, H, W, duration=0.2, seed=500, device="cuda")
    flow = synth.lowpass_flow(1, H, W, sigma=16.0, vmax=20.0, seed=501, device="cuda")
    m = DenseLinearFlow(1, H, W, grid=(H, W), init=flow).cuda()
    obj = AnchoredExact(h=1.0, tau=1.0, n_anchors=None, n_slices=16, seed=502)
    return ev, m, obj, obj.draw(ev)


@pytest.mark.parametrize("world", [2, 3])
def test_partial_sums_and_gradients_add_up(window, world):
    from x_b200.distributed import ExactPartial, shard_range
    from x_b200.objectives import _fused_kind
    ev, m, obj, (anchors, u, z) = window
    m.grid.grad = None
    ls_full, _ = obj.log_scores(ev, m, noise=(anchors, u, z))
    loss = -ls_full.mean()
    loss.backward()
    g_full = m.grid.grad.clone()
    spec = (_fused_kind(m), 1, ev.height, ev.width, obj.h, obj.tau, obj.cut, obj.eps_frac, obj.n_slices,
            obj.visibility, 16)
    parts = [ExactPartial(spec, m.theta, ev.xy, ev.t, ev.b, anchors, u, z, *shard_range(ev.n, r, world))
             for r in range(world)]
    S = sum(p.S for p in parts)
    ls = parts[0].log_scores(S)
    np.testing.assert_allclose(ls.cpu().numpy(), ls_full.detach().cpu().numpy(), rtol=1e-5, atol=1e-5)
    grad_ls = torch.full_like(ls, -1.0 / ls.numel())
    g = sum(p.backward(grad_ls, S, tuple(m.theta.shape)) for p in parts)
    scale = float(g_full.abs().max())
    assert float((g - g_full).abs().max()) / scale < 1e-4


def test_sharded_objective_single_rank_equals_fused(window):
    from x_b200.distributed import ShardedAnchoredExact
    ev, m, obj, noise = window
    sh = ShardedAnchoredExact(h=1.0, tau=1.0, n_anchors=None, n_slices=16, seed=502, rank=0, world=1)
    l1, _ = obj.log_scores(ev, m, noise=noise)
    l2, _ = sh.log_scores(ev, m, noise=noise)
    np.testing.assert_allclose(l2.detach().cpu().numpy(), l1.detach().cpu().numpy(), rtol=1e-5, atol=1e-5)
