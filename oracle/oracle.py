"""TEST INFRASTRUCTURE ONLY -- numpy front end of the plain-C oracle (oracle/atl_oracle.c).

Used by tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline leg as the checker of the
CUDA library; the product path (package ``x_b200``) never imports this module.

Each function names the reference (KAVYANSHTYAGI/x, package ``atl``) code it restates.  The C
oracle is pinned bit-for-bit against the reference's own outputs in tests/golden/ (see
tests/test_oracle_golden.py).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i64 = ctypes.c_int64
_dbl = ctypes.c_double
_LIB = None


def build() -> Path:
    """Compile liboracle.so (plain C, gcc) if it is missing or older than its source."""
    src = HERE / "atl_oracle.c"
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-C", str(HERE), "all"], check=True, stdout=subprocess.DEVNULL)
    return LIB_PATH


def lib():
    global _LIB
    if _LIB is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.oracle_vmax.restype = ctypes.c_float
        L.oracle_vmax.argtypes = [_f32p, _i64]
        L.oracle_plan_geometry.restype = None
        L.oracle_plan_geometry.argtypes = [ctypes.c_float, _f32p, _i64, _i64, _i64, _dbl, _dbl, _i64, _f64p]
        L.oracle_plan_count.restype = _i64
        L.oracle_plan_count.argtypes = [_f32p, _f32p, _f32p, _i64p, _i64, _i64, _dbl, _f64p]
        L.oracle_plan_build.restype = None
        L.oracle_plan_build.argtypes = [_f32p, _f32p, _f32p, _i64p, _i64, _i64, _i64, _dbl, _f64p, _i64p,
                                        ctypes.c_void_p, _i64, _f32p, _f32p, _f32p, _i64p, _i64p, _f32p, _f32p,
                                        _i64p, _i64p, _f32p]
        pair = [_f32p, _f32p, _f32p, _i64p, _i64p, _f32p, _f32p, _i64p, _i64p, _f32p]
        L.oracle_pair_fwd.restype = None
        L.oracle_pair_fwd.argtypes = pair + [_i64, _i64, _i64, _i64, _dbl, _dbl, _dbl, _f32p,
                                             ctypes.POINTER(ctypes.c_int64)]
        L.oracle_pair_bwd.restype = None
        L.oracle_pair_bwd.argtypes = [_f32p] + pair + [_i64, _i64, _i64, _i64, _dbl, _dbl, _dbl, _i64, _f32p]
        L.oracle_pair_bwd_f64.restype = None
        L.oracle_pair_bwd_f64.argtypes = [_f32p] + pair + [_i64, _i64, _i64, _i64, _dbl, _dbl, _dbl, _i64, _f64p, _f64p,
                                                          _i64p]
        _u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
        L.oracle_philox4x32_10.restype = None
        L.oracle_philox4x32_10.argtypes = [_u32p, _u32p, _u32p]
        L.oracle_rng_draw2.restype = None
        L.oracle_rng_draw2.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, _i64, _f64p]
        L.oracle_splat_bilinear_fwd.argtypes = [_f32p, _f32p, _i64p, _i64, _i64, _i64, _i64, _f32p]
        L.oracle_splat_bilinear_bwd.argtypes = [_f32p, _f32p, _f32p, _i64p, _i64, _i64, _i64, _f32p, _f32p]
        L.oracle_splat_gauss_fwd.argtypes = [_f32p, _f32p, _i64p, _i64, _i64, _i64, _i64, _dbl, _i64, _f32p]
        L.oracle_splat_gauss_bwd.argtypes = [_f32p, _f32p, _f32p, _i64p, _i64, _i64, _i64, _dbl, _i64, _f32p,
                                             _f32p]
        L.oracle_gather_fwd.argtypes = [_f32p, _f32p, _i64p, _i64, _i64, _i64, _f32p]
        L.oracle_gather_bwd.argtypes = [_f32p, _f32p, _f32p, _i64p, _i64, _i64, _i64, _i64, _f32p, _f32p]
        L.oracle_voxel_grid.argtypes = [_f32p, _f32p, _f32p, _i64p, _i64, _i64, _i64, _i64, _i64, _f32p]
        L.oracle_window_counts.argtypes = [_f32p, _i64p, _i64, _i64p, _i64, _dbl, _f32p]
        L.oracle_velocity.argtypes = [ctypes.c_int, _f32p, _i64, _i64, _i64, _i64, _f32p, _i64p, _i64, _f32p]
        L.oracle_visible_fraction.argtypes = [ctypes.c_int, _f32p, _i64, _i64, _f32p, _f32p, _i64p, _i64, _f32p,
                                              _i64p, _i64, _i64, _i64, _i64, _dbl, _i64, _f32p]
        _LIB = L
    return _LIB


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _l(a):
    return np.ascontiguousarray(a, dtype=np.int64)


MOTION_KIND = {"translation": 0, "affine": 1, "dense": 2}


# ------------------------------------------------------------------------------------------------- plan
def plan_geometry(v, anchor_xy, H, W, h, cut, S):
    """(cell, ox, oy, GW, GH, vmax): atl/ops/functional.py:136-149."""
    L = lib()
    v = _f(v).reshape(-1, 2)
    xa = _f(anchor_xy).reshape(-1, 2)
    vmax = float(L.oracle_vmax(v, v.shape[0])) if v.shape[0] else 0.0
    out = np.zeros(5, np.float64)
    L.oracle_plan_geometry(vmax, xa, xa.shape[0], H, W, float(h), float(cut), int(S), out)
    return out[0], out[1], out[2], int(out[3]), int(out[4]), vmax


def build_pair_plan(x, t, v, b, B, H, W, anchors, h, tau, cut=3.0, n_slices=16, anchor_xy=None) -> dict:
    """Restatement of atl/ops/functional.py:132-178 (stable within-cell order)."""
    L = lib()
    x, t, v, b, anchors = _f(x).reshape(-1, 2), _f(t), _f(v).reshape(-1, 2), _l(b), _l(anchors)
    S = int(n_slices)
    xa = x[anchors] if anchor_xy is None else _f(anchor_xy).reshape(-1, 2)
    cell, ox, oy, GW, GH, vmax = plan_geometry(v, xa, H, W, h, cut, S)
    geom = np.array([cell, ox, oy, GW, GH], np.float64)
    N, M = t.shape[0], anchors.shape[0]
    ns = int(L.oracle_plan_count(x, t, v, b, N, S, float(tau), geom))
    ncell = B * S * GH * GW
    p = dict(src_y=np.zeros((ns, 2), np.float32), src_v=np.zeros((ns, 2), np.float32),
             src_t=np.zeros(ns, np.float32), src_id=np.zeros(ns, np.int64),
             cell_start=np.zeros(ncell + 1, np.int64), anc_x=np.zeros((M, 2), np.float32),
             anc_t=np.zeros(M, np.float32), anc_cell=np.zeros((M, 3), np.int64), anc_id=np.zeros(M, np.int64),
             slice_c=np.zeros(S, np.float32))
    axy = None if anchor_xy is None else xa.ctypes.data
    L.oracle_plan_build(x, t, v, b, N, B, S, float(tau), geom, anchors, axy, M, p["src_y"], p["src_v"],
                        p["src_t"], p["src_id"], p["cell_start"], p["anc_x"], p["anc_t"], p["anc_cell"],
                        p["anc_id"], p["slice_c"])
    p.update(S=S, GH=GH, GW=GW, cell=cell, ox=ox, oy=oy, vmax=vmax)
    return p


def _pair_arrays(p):
    return (p["src_y"], p["src_v"], p["src_t"], p["src_id"], p["cell_start"], p["anc_x"], p["anc_t"],
            p["anc_cell"], p["anc_id"], p["slice_c"])


def pair_fwd(p, h, tau, cut=3.0):
    """S_i (M,) float32 and the number of contributing pairs: csrc/atl_cpu.cpp:203-222."""
    L = lib()
    M = p["anc_t"].shape[0]
    out = np.zeros(M, np.float32)
    hits = ctypes.c_int64(0)
    L.oracle_pair_fwd(*_pair_arrays(p), M, p["S"], p["GH"], p["GW"], float(h), float(tau), float(cut), out,
                      ctypes.byref(hits))
    return out, int(hits.value)


def pair_bwd(p, g, h, tau, cut, N):
    """d(sum g_i S_i)/dv (N, 2): csrc/atl_cpu.cpp:224-253."""
    L = lib()
    M = p["anc_t"].shape[0]
    gv = np.zeros((N, 2), np.float32)
    L.oracle_pair_bwd(_f(g), *_pair_arrays(p), M, p["S"], p["GH"], p["GW"], float(h), float(tau), float(cut), N,
                      gv)
    return gv


def pair_bwd_f64(p, g, h, tau, cut, N):
    """The pair gradient with double accumulation (the accurate value), plus per component the sum of the
    contributions' magnitudes and per event their count: (gv (N,2) f64, gabs (N,2) f64, cnt (N,) i64)."""
    L = lib()
    M = p["anc_t"].shape[0]
    gv, gabs, cnt = np.zeros((N, 2)), np.zeros((N, 2)), np.zeros(N, np.int64)
    L.oracle_pair_bwd_f64(_f(g), *_pair_arrays(p), M, p["S"], p["GH"], p["GW"], float(h), float(tau), float(cut), N,
                          gv, gabs, cnt)
    return gv, gabs, cnt


def ats_pair_sums(x, t, v, b, B, H, W, anchors, h, tau, cut=3.0, n_slices=16, anchor_xy=None):
    """atl/ops/functional.py:199-207 forward value through the plan."""
    p = build_pair_plan(x, t, v, b, B, H, W, anchors, h, tau, cut, n_slices, anchor_xy)
    return pair_fwd(p, h, tau, cut)[0]


# ------------------------------------------------------------------------------------------------- splat etc.
def splat_bilinear_fwd(pos, w, b, B, H, W):
    img = np.zeros((B, H, W), np.float32)
    pos, w, b = _f(pos), _f(w), _l(b)
    lib().oracle_splat_bilinear_fwd(pos, w, b, w.shape[0], B, H, W, img)
    return img


def splat_bilinear_bwd(g, pos, w, b):
    g, pos, w, b = _f(g), _f(pos), _f(w), _l(b)
    gp, gw = np.zeros_like(pos), np.zeros_like(w)
    lib().oracle_splat_bilinear_bwd(g, pos, w, b, w.shape[0], g.shape[1], g.shape[2], gp, gw)
    return gp, gw


def splat_gauss_fwd(pos, w, b, B, H, W, sigma, R):
    img = np.zeros((B, H, W), np.float32)
    pos, w, b = _f(pos), _f(w), _l(b)
    lib().oracle_splat_gauss_fwd(pos, w, b, w.shape[0], B, H, W, float(sigma), int(R), img)
    return img


def splat_gauss_bwd(g, pos, w, b, sigma, R):
    g, pos, w, b = _f(g), _f(pos), _f(w), _l(b)
    gp, gw = np.zeros_like(pos), np.zeros_like(w)
    lib().oracle_splat_gauss_bwd(g, pos, w, b, w.shape[0], g.shape[1], g.shape[2], float(sigma), int(R), gp, gw)
    return gp, gw


def gather_fwd(img, pos, b):
    img, pos, b = _f(img), _f(pos), _l(b)
    out = np.zeros(pos.shape[0], np.float32)
    lib().oracle_gather_fwd(img, pos, b, pos.shape[0], img.shape[1], img.shape[2], out)
    return out


def gather_bwd(g, img, pos, b):
    g, img, pos, b = _f(g), _f(img), _f(pos), _l(b)
    gi, gp = np.zeros_like(img), np.zeros_like(pos)
    lib().oracle_gather_bwd(g, img, pos, b, pos.shape[0], img.shape[0], img.shape[1], img.shape[2], gi, gp)
    return gi, gp


def voxel_grid(pos, t, p, b, B, C, H, W):
    out = np.zeros((B, C, H, W), np.float32)
    pos, t, p, b = _f(pos), _f(t), _f(p), _l(b)
    lib().oracle_voxel_grid(pos, t, p, b, t.shape[0], B, C, H, W, out)
    return out


def window_counts(t, b, idx, tau):
    t, b, idx = _f(t), _l(b), _l(idx)
    out = np.zeros(idx.shape[0], np.float32)
    lib().oracle_window_counts(t, b, t.shape[0], idx, idx.shape[0], float(tau), out)
    return out


# ------------------------------------------------------------------------------------------------- motion
def velocity(kind, theta, xy, b, H, W):
    """Per-event velocity of Translation / Affine / DenseLinearFlow (linear mode)."""
    theta = _f(theta)
    xy, b = _f(xy).reshape(-1, 2), _l(b)
    Hg, Wg = (theta.shape[-2], theta.shape[-1]) if kind == "dense" else (1, 1)
    v = np.zeros_like(xy)
    lib().oracle_velocity(MOTION_KIND[kind], theta.reshape(-1), Hg, Wg, H, W, xy, b, xy.shape[0], v)
    return v


def velocity_backward(kind, theta, xy, b, H, W, gv):
    """d(sum gv . v)/d theta for the three motion kinds (float64 accumulation)."""
    theta = np.asarray(theta)
    xy, gv, b = np.asarray(xy, np.float64).reshape(-1, 2), np.asarray(gv, np.float64).reshape(-1, 2), _l(b)
    g = np.zeros(theta.shape, np.float64)
    if kind == "translation":
        np.add.at(g, b, gv)
    elif kind == "affine":
        c = np.array([np.float32((W - 1) / 2.0), np.float32((H - 1) / 2.0)], np.float64)
        d = (xy.astype(np.float32) - c.astype(np.float32)).astype(np.float64)
        np.add.at(g[:, 0], b, gv[:, 0]); np.add.at(g[:, 1], b, gv[:, 1])
        np.add.at(g[:, 2], b, gv[:, 0] * d[:, 0]); np.add.at(g[:, 3], b, gv[:, 0] * d[:, 1])
        np.add.at(g[:, 4], b, gv[:, 1] * d[:, 0]); np.add.at(g[:, 5], b, gv[:, 1] * d[:, 1])
    else:
        Bn, C, Hg, Wg = theta.shape
        x32 = xy.astype(np.float32)
        gx = (x32[:, 0] / np.float32(max(W - 1, 1))).astype(np.float32) * np.float32(Wg - 1)
        gy = (x32[:, 1] / np.float32(max(H - 1, 1))).astype(np.float32) * np.float32(Hg - 1)
        gx = np.clip(gx.astype(np.float32), 0, Wg - 1); gy = np.clip(gy.astype(np.float32), 0, Hg - 1)
        x0 = np.minimum(np.floor(gx), max(Wg - 2, 0)); y0 = np.minimum(np.floor(gy), max(Hg - 2, 0))
        ax, ay = (gx - x0).astype(np.float64), (gy - y0).astype(np.float64)
        x0, y0 = x0.astype(np.int64), y0.astype(np.int64)
        x1, y1 = np.minimum(x0 + 1, Wg - 1), np.minimum(y0 + 1, Hg - 1)
        for yy, xx, w in ((y0, x0, (1 - ax) * (1 - ay)), (y0, x1, ax * (1 - ay)), (y1, x0, (1 - ax) * ay),
                          (y1, x1, ax * ay)):
            for c in range(C):
                np.add.at(g[:, c], (b, yy, xx), w * gv[:, c])
    return g


def visible_fraction(kind, theta, xa, ta, ba, t, b, B, H, W, tau, n_check=16):
    """atl/objectives/ats.py:31-50 for motions linear at the event."""
    theta = _f(theta)
    xa, ta, ba, t, b = _f(xa).reshape(-1, 2), _f(ta), _l(ba), _f(t), _l(b)
    Hg, Wg = (theta.shape[-2], theta.shape[-1]) if kind == "dense" else (1, 1)
    out = np.zeros(ta.shape[0], np.float32)
    lib().oracle_visible_fraction(MOTION_KIND[kind], theta.reshape(-1), Hg, Wg, xa, ta, ba, ta.shape[0], t, b,
                                  t.shape[0], B, H, W, float(tau), int(n_check), out)
    return out


# ------------------------------------------------------------------------------------------------- objective
def anchored_exact(kind, theta, xs, t, b, B, H, W, anchors, xa, h=1.0, tau=1.0, eps_frac=1e-2, n_slices=16,
                   cut=3.0, visibility=True, with_grad=True, exact_grad=False):
    """AnchoredExact.log_scores + loss + gradient (atl/objectives/ats.py:75-105) on pre-drawn inputs:
    ``xs`` are the dequantised positions, ``xa`` the (smoothed) anchor positions.

    Returns dict(ls (M,), loss, S (M,), Wn (M,), vis (M,), grad_v (N,2), grad_theta, hits); with
    ``exact_grad`` also the double-accumulated gradients (grad_v64, grad_theta64) and the fp32 error-bound
    ingredients (grad_v_abs, grad_v_cnt, grad_theta_abs, grad_theta_terms)."""
    xs, t, b, anchors, xa = _f(xs).reshape(-1, 2), _f(t), _l(b), _l(anchors), _f(xa).reshape(-1, 2)
    N, M = t.shape[0], anchors.shape[0]
    v = velocity(kind, theta, xs, b, H, W)
    p = build_pair_plan(xs, t, v, b, B, H, W, anchors, h, tau, cut, n_slices, anchor_xy=xa)
    S, hits = pair_fwd(p, h, tau, cut)
    Wn = np.maximum(window_counts(t, b, anchors, tau), np.float32(1))
    vis = visible_fraction(kind, theta, xa, t[anchors], b[anchors], t, b, B, H, W, tau) if visibility else None
    if vis is not None:
        Wn = (Wn * vis).astype(np.float32)
    eps = eps_frac / (H * W)
    denom = (((Wn * np.float32(2)).astype(np.float32) * np.float32(math.pi)).astype(np.float32)
             * np.float32(h ** 2)).astype(np.float32)
    q = (S / denom).astype(np.float32)
    ls = np.log((np.float32(eps) + q).astype(np.float32)).astype(np.float32)
    loss = -float(np.mean(ls.astype(np.float64)))
    out = dict(ls=ls, loss=loss, S=S, Wn=Wn, vis=vis, v=v, plan=p, hits=hits)
    if with_grad and M > 0:
        gS = (-(1.0 / M) / (np.float64(eps) + q.astype(np.float64)) / denom.astype(np.float64)).astype(np.float32)
        gv = pair_bwd(p, gS, h, tau, cut, N)
        out["grad_v"] = gv
        out["grad_theta"] = velocity_backward(kind, theta, xs, b, H, W, gv)
        if exact_grad:
            gv64, gabs, cnt = pair_bwd_f64(p, gS, h, tau, cut, N)
            out["grad_v64"], out["grad_v_abs"], out["grad_v_cnt"] = gv64, gabs, cnt
            out["grad_theta64"] = velocity_backward(kind, theta, xs, b, H, W, gv64)
            out["grad_theta_abs"], out["grad_theta_terms"] = velocity_backward_bound(kind, theta, xs, b, H, W, gabs,
                                                                                      cnt)
    return out


def velocity_backward_bound(kind, theta, xy, b, H, W, gabs, cnt):
    """Ingredients of the fp32 error bound of d(sum gv . v)/d theta when every gv_j is itself an fp32 sum of
    cnt_j terms with magnitude sum gabs_j: returns (A, n) per theta element, A = sum_j |w_j| gabs_j (w_j the
    element's weight of event j) and n = max_j cnt_j + (events reaching the element), the term count of the
    two-level sum."""
    theta = np.asarray(theta)
    xy, gabs, b = np.asarray(xy, np.float64).reshape(-1, 2), np.asarray(gabs, np.float64).reshape(-1, 2), _l(b)
    A = np.zeros(theta.shape, np.float64)
    m = np.zeros(theta.shape, np.float64)
    one = np.ones(b.shape[0])
    if kind == "translation":
        np.add.at(A, b, gabs)
        np.add.at(m[:, 0], b, one); m[:, 1] = m[:, 0]
    elif kind == "affine":
        c = np.array([np.float32((W - 1) / 2.0), np.float32((H - 1) / 2.0)], np.float64)
        d = np.abs((xy.astype(np.float32) - c.astype(np.float32)).astype(np.float64))
        np.add.at(A[:, 0], b, gabs[:, 0]); np.add.at(A[:, 1], b, gabs[:, 1])
        np.add.at(A[:, 2], b, gabs[:, 0] * d[:, 0]); np.add.at(A[:, 3], b, gabs[:, 0] * d[:, 1])
        np.add.at(A[:, 4], b, gabs[:, 1] * d[:, 0]); np.add.at(A[:, 5], b, gabs[:, 1] * d[:, 1])
        for k in range(6):
            np.add.at(m[:, k], b, one)
    else:
        Bn, C, Hg, Wg = theta.shape
        x32 = xy.astype(np.float32)
        gx = (x32[:, 0] / np.float32(max(W - 1, 1))).astype(np.float32) * np.float32(Wg - 1)
        gy = (x32[:, 1] / np.float32(max(H - 1, 1))).astype(np.float32) * np.float32(Hg - 1)
        gx = np.clip(gx.astype(np.float32), 0, Wg - 1); gy = np.clip(gy.astype(np.float32), 0, Hg - 1)
        x0 = np.minimum(np.floor(gx), max(Wg - 2, 0)); y0 = np.minimum(np.floor(gy), max(Hg - 2, 0))
        ax, ay = (gx - x0).astype(np.float64), (gy - y0).astype(np.float64)
        x0, y0 = x0.astype(np.int64), y0.astype(np.int64)
        x1, y1 = np.minimum(x0 + 1, Wg - 1), np.minimum(y0 + 1, Hg - 1)
        for yy, xx, w in ((y0, x0, (1 - ax) * (1 - ay)), (y0, x1, ax * (1 - ay)), (y1, x0, (1 - ax) * ay),
                          (y1, x1, ax * ay)):
            for c in range(C):
                np.add.at(A[:, c], (b, yy, xx), w * gabs[:, c])
                np.add.at(m[:, c], (b, yy, xx), one)
    return A, m + float(np.max(cnt, initial=0))


def threads() -> int:
    """Threads the OpenMP parts of the oracle use (pair forward only)."""
    return int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))


# ------------------------------------------------------------------------------------------------- device draws
def philox4x32_10(ctr, key):
    """Philox4x32-10 (Salmon et al., SC'11) of a 4-word counter and a 2-word key."""
    out = np.zeros(4, np.uint32)
    lib().oracle_philox4x32_10(np.asarray(ctr, np.uint32), np.asarray(key, np.uint32), out)
    return out


def rng_draw2(normal, seed, call, n):
    """The library's device draws (atlb_rng_uniform2 / _normal2) in double: (n, 2)."""
    out = np.zeros((n, 2), np.float64)
    lib().oracle_rng_draw2(1 if normal else 0, int(seed), int(call), int(n), out)
    return out

