"""atlb_ats_pair_fwd_noalloc: the pair forward for callers that cannot allocate device memory, whose
anchor buckets live in a fixed device array inside the library.  It is checked against
atlb_ats_pair_fwd (caller workspace) through the C ABI on two calls in a row over different plans, so
that what the first call leaves in the shared array cannot leak into the second.  The file is named so
that pytest collects it last; it builds its own inputs and passes alone in a fresh process too."""
import ctypes

import numpy as np
import pytest
import torch

RTOL = 1e-5  # the tolerance of the other pair-sum parity tests


def _lib():
    from x_b200 import _lib as L
    return L


def _plan(seed, n, B, H, W, tau, S, vs):
    """A device plan over seeded synthetic events, (b, t)-sorted like an EventPacket."""
    from x_b200 import functional as F
    rng = np.random.default_rng(seed)
    xy = np.stack([rng.integers(0, W, n), rng.integers(0, H, n)], 1).astype(np.float32)
    xy += rng.uniform(-0.5, 0.5, xy.shape).astype(np.float32)
    b = np.sort(rng.integers(0, B, n)).astype(np.int64)
    t = np.concatenate([np.sort(rng.uniform(0, 1, (b == k).sum())) for k in range(B)]).astype(np.float32)
    v = (rng.normal(size=(n, 2)) * vs / 3).astype(np.float32)
    anchors = np.sort(rng.choice(n, n // 3, replace=False)).astype(np.int64)
    axy = (xy[anchors] + rng.normal(size=(anchors.size, 2))).astype(np.float32)
    dev = lambda a: torch.as_tensor(a).cuda().contiguous()  # noqa: E731
    return F.build_pair_plan(dev(xy), dev(t), dev(v), dev(b), B, H, W, dev(anchors), 1.0, tau, 3.0, S,
                             anchor_xy=dev(axy))


def _args(p):
    L = _lib()
    return [L.ptr(a) for a in (p.src_y, p.src_v, p.src_t, p.src_id, p.cell_start, p.anc_x, p.anc_t, p.anc_cell,
                               p.anc_id, p.slice_c)]


def _sizes(p):
    return p.src_y.shape[0], p.anc_x.shape[0], p.cell_start.shape[0] - 1


def _with_workspace(p, tau):
    """The existing entry point, with a caller-allocated workspace."""
    L = _lib()
    Ns, M, ncell = _sizes(p)
    out = torch.empty(M, dtype=torch.float32, device="cuda")
    nb = L.lib().atlb_pair_workspace_bytes(M, ncell)
    ws = L.workspace(nb, "cuda")
    L.check(L.lib().atlb_ats_pair_fwd(*_args(p), Ns, M, ncell, p.S, p.GH, p.GW, 1.0, float(tau), 3.0, L.ptr(out),
                                      L.ptr(ws), nb, L.stream()), "ats_pair_fwd")
    return out


def _no_alloc(p, tau, out):
    L = _lib()
    Ns, M, ncell = _sizes(p)
    L.check(L.lib().atlb_ats_pair_fwd_noalloc(*_args(p), Ns, M, ncell, p.S, p.GH, p.GW, 1.0, float(tau), 3.0,
                                              L.ptr(out), L.stream()), "ats_pair_fwd_noalloc")
    return out


@pytest.mark.gpu
def test_no_alloc_matches_workspace_entry_point_on_two_calls():
    L = _lib()
    # a larger plan first, then a smaller one on another grid: the second call reuses the array
    cases = [(11, 60000, 2, 96, 128, 1.0, 16, 20.0), (12, 15000, 1, 40, 56, 0.2, 8, 5.0)]
    plans = [(_plan(*c), c[5]) for c in cases]
    for p, _ in plans:
        Ns, M, ncell = _sizes(p)
        assert L.lib().atlb_pair_workspace_bytes(M, ncell) <= (16 << 20)
    refs = [_with_workspace(p, tau) for p, tau in plans]
    # NaN-filled outputs: every anchor must be written by the call
    outs = [torch.full_like(r, float("nan")) for r in refs]
    for (p, tau), out in zip(plans, outs):
        _no_alloc(p, tau, out)
    torch.cuda.synchronize()
    for r, o in zip(refs, outs):
        assert torch.isfinite(r).all()
        assert (r > 0).any()
        np.testing.assert_allclose(o.cpu().numpy(), r.cpu().numpy(), rtol=RTOL, atol=1e-6)


@pytest.mark.gpu
def test_no_alloc_rejects_sizes_beyond_its_array():
    L = _lib()
    p = _plan(13, 5000, 1, 40, 56, 0.2, 8, 5.0)
    Ns, M, ncell = _sizes(p)
    big_m = (16 << 20) // 28 + 1  # 28 bytes of anchor buckets per anchor
    ax = torch.zeros(big_m, 2, dtype=torch.float32, device="cuda")
    at = torch.zeros(big_m, dtype=torch.float32, device="cuda")
    ac = torch.zeros(big_m, 3, dtype=torch.int64, device="cuda")
    aid = torch.zeros(big_m, dtype=torch.int64, device="cuda")
    out = torch.empty(big_m, dtype=torch.float32, device="cuda")
    a = _args(p)
    a[5], a[6], a[7], a[8] = L.ptr(ax), L.ptr(at), L.ptr(ac), L.ptr(aid)
    st = L.lib().atlb_ats_pair_fwd_noalloc(*a, Ns, big_m, ncell, p.S, p.GH, p.GW, 1.0, 0.2, 3.0, L.ptr(out),
                                           L.stream())
    assert st == L.ATLB_ERR_WORKSPACE
    assert b"scratch bytes" in L.lib().atlb_last_error()
    # the array is still usable afterwards
    r = _with_workspace(p, 0.2)
    o = _no_alloc(p, 0.2, torch.full_like(r, float("nan")))
    np.testing.assert_allclose(o.cpu().numpy(), r.cpu().numpy(), rtol=RTOL, atol=1e-6)


def test_no_alloc_rejects_oversize_without_a_device():
    """The size check comes before any device work, so it answers on a host without a GPU."""
    L = _lib()
    lib = L.load_library()
    fake = ctypes.c_void_p(256)  # never dereferenced: the call fails before any device access
    big_m = (16 << 20) // 28 + 1
    st = lib.atlb_ats_pair_fwd_noalloc(*([fake] * 10), 0, big_m, 1, 1, 1, 1, 1.0, 0.2, 3.0, fake, None)
    assert st == L.ATLB_ERR_WORKSPACE
    assert b"scratch bytes" in lib.atlb_last_error()
    st = lib.atlb_ats_pair_fwd_noalloc(*([fake] * 10), -1, 1, 1, 1, 1, 1, 1.0, 0.2, 3.0, fake, None)
    assert st == L.ATLB_ERR_ARG
