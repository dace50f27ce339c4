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


LIMIT = 16 << 20  # ATLB_PAIR_NOALLOC_SCRATCH_BYTES


def _largest_fitting_m(ncell):
    """The largest anchor count whose workspace, less its 256 bytes of alignment slack, fits the fixed array
    (from the library's own sizing query, so that the boundary tested is the one the entry point checks)."""
    lib = _lib().load_library()
    lo, hi = 0, LIMIT
    while lo < hi:  # largest M with bytes(M) - 256 <= LIMIT
        mid = (lo + hi + 1) // 2
        if lib.atlb_pair_workspace_bytes(mid, ncell) - 256 <= LIMIT:
            lo = mid
        else:
            hi = mid - 1
    return lo


@pytest.mark.gpu
def test_no_alloc_at_its_size_limit():
    """The largest anchor count that fits the array runs and matches the workspace entry point; one anchor
    more is rejected before any device work, and the array stays usable afterwards."""
    L = _lib()
    # 1.5M events, a third of them anchors: more anchors than the array holds for this grid
    p = _plan(13, 1_500_000, 1, 480, 640, 1.0, 16, 20.0)
    Ns, M_all, ncell = _sizes(p)
    m_max = _largest_fitting_m(ncell)
    assert 0 < m_max < M_all
    a = _args(p)
    cut = {k: getattr(p, k)[: m_max + 1].contiguous() for k in ("anc_x", "anc_t", "anc_cell", "anc_id")}
    a[5], a[6], a[7], a[8] = (L.ptr(cut[k]) for k in ("anc_x", "anc_t", "anc_cell", "anc_id"))
    out = torch.full((m_max + 1,), float("nan"), dtype=torch.float32, device="cuda")
    st = L.lib().atlb_ats_pair_fwd_noalloc(*a, Ns, m_max + 1, ncell, p.S, p.GH, p.GW, 1.0, 1.0, 3.0, L.ptr(out),
                                           L.stream())
    assert st == L.ATLB_ERR_WORKSPACE
    assert b"scratch bytes" in L.lib().atlb_last_error()
    L.check(L.lib().atlb_ats_pair_fwd_noalloc(*a, Ns, m_max, ncell, p.S, p.GH, p.GW, 1.0, 1.0, 3.0, L.ptr(out),
                                              L.stream()), "ats_pair_fwd_noalloc at the limit")
    ref = torch.empty(m_max, dtype=torch.float32, device="cuda")
    nb = L.lib().atlb_pair_workspace_bytes(m_max, ncell)
    ws = L.workspace(nb, "cuda")
    L.check(L.lib().atlb_ats_pair_fwd(*a, Ns, m_max, ncell, p.S, p.GH, p.GW, 1.0, 1.0, 3.0, L.ptr(ref), L.ptr(ws), nb,
                                      L.stream()), "ats_pair_fwd")
    torch.cuda.synchronize()
    assert torch.isfinite(out[:m_max]).all()
    np.testing.assert_allclose(out[:m_max].cpu().numpy(), ref.cpu().numpy(), rtol=RTOL, atol=1e-6)
    assert torch.isnan(out[m_max])  # the rejected call wrote nothing
    # a small call after the rejected one still matches
    q = _plan(14, 5000, 1, 40, 56, 0.2, 8, 5.0)
    r = _with_workspace(q, 0.2)
    o = _no_alloc(q, 0.2, torch.full_like(r, float("nan")))
    np.testing.assert_allclose(o.cpu().numpy(), r.cpu().numpy(), rtol=RTOL, atol=1e-6)


def test_no_alloc_rejects_oversize_without_a_device():
    """The size check comes before any device work, so it answers on a host without a GPU: one anchor beyond
    the largest count that fits is rejected, and so are invalid sizes."""
    L = _lib()
    lib = L.load_library()
    fake = ctypes.c_void_p(256)  # never dereferenced: the call fails before any device access
    ncell = 1
    big_m = _largest_fitting_m(ncell) + 1
    assert lib.atlb_pair_workspace_bytes(big_m, ncell) - 256 > LIMIT
    st = lib.atlb_ats_pair_fwd_noalloc(*([fake] * 10), 0, big_m, ncell, 1, 1, 1, 1.0, 0.2, 3.0, fake, None)
    assert st == L.ATLB_ERR_WORKSPACE
    assert b"scratch bytes" in lib.atlb_last_error()
    st = lib.atlb_ats_pair_fwd_noalloc(*([fake] * 10), -1, 1, 1, 1, 1, 1, 1.0, 0.2, 3.0, fake, None)
    assert st == L.ATLB_ERR_ARG
