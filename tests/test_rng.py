"""Opt-in device draws of the objectives' noise (x_b200.rng, atlb_rng_*): Philox4x32-10 (Salmon et al.,
SC'11).  CPU: the oracle's restatement against the generator's published known-answer vectors and the
moments of its uniforms / normals.  GPU: the library's draws against the oracle (uniforms bit-exact,
normals within float rounding), and the fused AnchoredExact drawing inline equal to the same objective
given the materialised draws."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

# (counter, key) -> output of Philox4x32-10, as published with the generator
KAT = [
    ([0x00000000, 0x00000000, 0x00000000, 0x00000000], [0x00000000, 0x00000000],
     [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]),
    ([0xffffffff, 0xffffffff, 0xffffffff, 0xffffffff], [0xffffffff, 0xffffffff],
     [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]),
    ([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], [0xa4093822, 0x299f31d0],
     [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]),
]


@pytest.mark.parametrize("ctr,key,out", KAT)
def test_philox_known_answers(ctr, key, out):
    assert O.philox4x32_10(ctr, key).tolist() == out


def test_draw_moments():
    u = O.rng_draw2(False, 12345, 7, 200000)
    z = O.rng_draw2(True, 12345, 7, 200000)
    assert u.min() >= 0.0 and u.max() < 1.0
    assert abs(u.mean() - 0.5) < 3e-3 and abs(u.var() - 1 / 12) < 2e-3
    assert abs(z.mean()) < 5e-3 and abs(z.std() - 1.0) < 5e-3
    assert abs(np.corrcoef(z[:, 0], z[:, 1])[0, 1]) < 1e-2
    # another call or seed gives other numbers
    assert not np.array_equal(u, O.rng_draw2(False, 12345, 8, 200000))
    assert not np.array_equal(u, O.rng_draw2(False, 12346, 7, 200000))


@pytest.mark.gpu
@pytest.mark.parametrize("seed,call,n", [(1, 0, 1000), (2**40 + 3, 2**33 + 5, 300001), (0, 0, 1)])
def test_device_draws_match_oracle(seed, call, n):
    from x_b200 import rng as R
    u = R.uniform2(seed, call, n, "cuda").cpu().numpy()
    z = R.normal2(seed, call, n, "cuda").cpu().numpy()
    np.testing.assert_array_equal(u.astype(np.float64), O.rng_draw2(False, seed, call, n))
    np.testing.assert_allclose(z, O.rng_draw2(True, seed, call, n), rtol=1e-5, atol=2e-6)


@pytest.mark.gpu
def test_fused_inline_draws_equal_materialised_draws():
    """AnchoredExact(device_rng=True) draws u and z inside the fused pipeline's prepare kernels; the same
    seed and call materialised by x_b200.rng and passed as noise give the same scores and gradient."""
    from x_b200 import motion as Mo
    from x_b200 import rng as R
    from x_b200 import synth
    from x_b200.objectives import AnchoredExact
    from tests.parity import assert_grad_parity
    H, W = 96, 128
    ev = synth.textured_window(30000, H, W, seed=11, device="cuda")
    flow = synth.lowpass_flow(1, H, W, sigma=8.0, vmax=10.0, seed=12, device="cuda")
    m1 = Mo.DenseLinearFlow(1, H, W, grid=(H, W), init=flow).cuda()
    m2 = Mo.DenseLinearFlow(1, H, W, grid=(H, W), init=flow).cuda()
    obj = AnchoredExact(h=1.0, n_anchors=None, seed=99, device_rng=True)
    ls1, anc = obj.log_scores(ev, m1)  # call 0, drawn inline
    (-ls1.mean()).backward()
    u = R.uniform2(99, 0, ev.n, "cuda")
    z = R.normal2(99, 0, anc.numel(), "cuda")
    ls2, _ = AnchoredExact(h=1.0, n_anchors=None, seed=99).log_scores(ev, m2, noise=(anc, u, z))
    (-ls2.mean()).backward()
    np.testing.assert_allclose(ls1.detach().cpu().numpy(), ls2.detach().cpu().numpy(), rtol=1e-6, atol=1e-6)
    assert_grad_parity(m1.grid.grad.cpu().numpy(), m2.grid.grad.cpu().numpy(), what="inline vs materialised draws")
    # the next call draws new noise; the stage-by-stage path with the same draws agrees with the fused one
    ls3, _ = obj.log_scores(ev, m1)
    assert not torch.allclose(ls1, ls3)
    obj4 = AnchoredExact(h=1.0, n_anchors=None, seed=99, device_rng=True, fused=False)
    obj4.device_draws.calls = 1
    ls4, _ = obj4.log_scores(ev, m1)
    np.testing.assert_allclose(ls3.detach().cpu().numpy(), ls4.detach().cpu().numpy(), rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
def test_sliced_device_draws():
    from x_b200 import motion as Mo
    from x_b200 import synth
    from x_b200.objectives import AnchoredSliced
    H, W = 64, 80
    ev = synth.textured_window(20000, H, W, seed=21, device="cuda")
    m = Mo.Translation(1, H, W, init=torch.tensor([[4.0, -3.0]])).cuda()
    a = AnchoredSliced(n_slices=4, sigma=1.0, seed=5, device_rng=True)
    b = AnchoredSliced(n_slices=4, sigma=1.0, seed=5, device_rng=True)
    la, _ = a.log_scores(ev, m)
    lb, _ = b.log_scores(ev, m)
    np.testing.assert_allclose(la.detach().cpu().numpy(), lb.detach().cpu().numpy(), rtol=1e-5, atol=1e-5)  # same call
    assert torch.isfinite(la).all()
    lc, _ = a.log_scores(ev, m)  # the next call
    assert not torch.allclose(la, lc)
