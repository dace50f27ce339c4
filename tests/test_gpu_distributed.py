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


@pytest.mark.parametrize("world", [2, 3])
def test_sliced_shards_sum_to_single_gpu(world):
    """ShardedAnchoredSliced's decomposition, ranks emulated in one process: each share of the events
    splats into a partial density stack, the stacks and source / check counts are summed, and each share's
    anchors are scored against the sum (the stages ShardedAnchoredSliced runs between its all-reduces).
    Scores equal the single-GPU ones anchor by anchor; the coefficient gradient within 1e-5 norm-wise."""
    from tests.parity import assert_grad_parity
    from x_b200.distributed import shard_range
    from x_b200.events import EventPacket
    from x_b200.motion import PixelTrajectories
    from x_b200.objectives import AnchoredSliced, slice_counts
    g = torch.Generator().manual_seed(31)
    B, H, W, K, n = 2, 48, 64, 3, 12000
    xy = torch.stack([torch.randint(0, W, (n,), generator=g), torch.randint(0, H, (n,), generator=g)], 1).float()
    b = torch.sort(torch.randint(0, B, (n,), generator=g)).values
    t = torch.rand(n, generator=g)
    order = torch.argsort(b.double() * 4 + t.double())
    ev = EventPacket(xy[order].cuda(), t[order].cuda(), torch.ones(n).cuda(), b[order].cuda(), B, H, W)
    coeff0 = (torch.nn.functional.avg_pool2d(torch.randn(B, 2 * K, H, W, generator=g), 9, 1, 4) * 10).cuda()
    obj = AnchoredSliced(n_slices=5, sigma=1.5, seed=32)
    noise = obj.draw(ev)

    c1 = coeff0.clone().requires_grad_(True)
    m1 = PixelTrajectories(c1, K, basis_kind="bezier", tile=4)
    ls1, idx1 = obj.log_scores(ev, m1, noise=noise)
    (-ls1.mean()).backward()

    c2 = coeff0.clone().requires_grad_(True)
    m2 = PixelTrajectories(c2, K, basis_kind="bezier", tile=4)
    sts = [obj._setup(ev, noise, None, None, *shard_range(n, r, world)) for r in range(world)]
    parts = [obj._density(st, m2) for st in sts]
    img = sum(p[0] for p in parts)
    per_kb = sum(p[1] for p in parts)
    counts = sum(slice_counts(ev, t=st["t"], b=st["b"]) for st in sts)
    assert torch.equal(counts, slice_counts(ev))
    ls_parts, idx_parts = [], []
    for r, st in enumerate(sts):
        ai, ka = obj._pick(st)
        ls_parts.append(obj._scores(st, m2, img, per_kb, counts, ai, ka))
        idx_parts.append(ai + shard_range(n, r, world)[0])
    ls2, idx2 = torch.cat(ls_parts), torch.cat(idx_parts)
    (-ls2.sum() / ls2.numel()).backward()

    assert torch.equal(torch.sort(idx2).values, torch.sort(idx1).values)
    a = torch.empty(n, device="cuda").index_copy_(0, idx1, ls1.detach())
    c = torch.empty(n, device="cuda").index_copy_(0, idx2, ls2.detach())
    # the density stack is a sum of partial stacks (fp32 adds in another order): scores within 1e-5
    torch.testing.assert_close(c[idx1], a[idx1], rtol=1e-5, atol=2e-5)
    e = assert_grad_parity(c2.grad.cpu().numpy(), c1.grad.cpu().numpy(), what="sharded sliced coefficient gradient")
    assert e["max_over_max"] <= 1e-5, e
