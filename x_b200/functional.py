"""Differentiable ops of the anchored-score path on B200 -- the mirror of atl/ops/functional.py.

Same functions, signatures and autograd classes as the reference (``splat``, ``gather``,
``ats_pair_sums``, ``build_pair_plan``/``PairPlan``, ``window_counts``, ``voxel_grid``, ``blur``);
the extension they call is libatlb200 (x_b200/_ext.py).  There is no CPU path and no fallback to
torch reference ops: CPU tensors raise.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib as L
from ._ext import get_ext


def _f32(t):
    return t.contiguous().float()


def _need_cuda(t, what):
    if not t.is_cuda:
        raise RuntimeError(f"x_b200.{what}: expected CUDA tensors (there is no CPU path)")


# ------------------------------------------------------------------------------------------- splat
class _SplatBilinear(torch.autograd.Function):
    """atl/ops/functional.py:24-35."""
    @staticmethod
    def forward(ctx, pos, w, b, B, H, W):
        pos, w, b = _f32(pos), _f32(w), b.contiguous().long()
        ctx.save_for_backward(pos, w, b)
        return get_ext().splat_bilinear_fwd(pos, w, b, B, H, W)

    @staticmethod
    def backward(ctx, g):
        pos, w, b = ctx.saved_tensors
        gp, gw = get_ext().splat_bilinear_bwd(g.contiguous().float(), pos, w, b)
        return gp, gw, None, None, None, None


class _SplatGauss(torch.autograd.Function):
    """atl/ops/functional.py:38-50."""
    @staticmethod
    def forward(ctx, pos, w, b, B, H, W, sigma, radius):
        pos, w, b = _f32(pos), _f32(w), b.contiguous().long()
        ctx.save_for_backward(pos, w, b)
        ctx.sigma, ctx.radius = sigma, radius
        return get_ext().splat_gauss_fwd(pos, w, b, B, H, W, sigma, radius)

    @staticmethod
    def backward(ctx, g):
        pos, w, b = ctx.saved_tensors
        gp, gw = get_ext().splat_gauss_bwd(g.contiguous().float(), pos, w, b, ctx.sigma, ctx.radius)
        return gp, gw, None, None, None, None, None, None


def splat(pos: torch.Tensor, w: torch.Tensor, b: torch.Tensor, B: int, H: int, W: int,
          kernel: str = "bilinear", sigma: float = 1.0, radius: int | None = None) -> torch.Tensor:
    """Accumulate weighted events into a (B, H, W) image (atl/ops/functional.py:53-65)."""
    _need_cuda(pos, "splat")
    if kernel == "bilinear":
        return _SplatBilinear.apply(pos, w, b, B, H, W)
    if kernel == "gauss":
        radius = int(math.ceil(3 * sigma)) if radius is None else radius
        return _SplatGauss.apply(pos, w, b, B, H, W, float(sigma), int(radius))
    raise ValueError(kernel)


class _SplatSlices(torch.autograd.Function):
    """Gaussian splats of T point sets sharing one batch index into a (T * B, H, W) stack: set j goes to
    images j * B .. j * B + B - 1 (one atlb_splat_gauss_fwd per set).  Differentiable w.r.t. the positions
    only (the weights are masks): the backward reuses each set's forward buckets (atlb_splat_gauss_bwd_pos)."""

    @staticmethod
    def forward(ctx, pos, w, b, B, H, W, sigma, radius):
        pos, w, b = _f32(pos), _f32(w), b.contiguous().long()
        T, N = pos.shape[0], pos.shape[1]
        img = torch.empty(T * B, H, W, dtype=torch.float32, device=pos.device)
        nb = L.lib().atlb_splat_gauss_workspace_bytes(N, B, H, W)
        # one workspace per set, kept for the backward: its buckets are reused there (weights are constants)
        keep = ctx.needs_input_grad[0]
        wss = [L.workspace(nb, pos.device) for _ in range(T if keep else 1)]
        for j in range(T):
            ws = wss[j if keep else 0]
            L.check(L.lib().atlb_splat_gauss_fwd(L.ptr(pos[j]), L.ptr(w[j]), L.ptr(b), N, B, H, W, float(sigma),
                                                  int(radius), L.ptr(img[j * B:(j + 1) * B]), L.ptr(ws), nb,
                                                  L.stream()), "splat_slices")
        ctx.save_for_backward(w)
        ctx.wss = wss if keep else None
        ctx.meta = (T, N, B, H, W, float(sigma), int(radius), nb)
        return img

    @staticmethod
    def backward(ctx, g):
        (w,) = ctx.saved_tensors
        T, N, B, H, W, sigma, radius, nb = ctx.meta
        g = g.contiguous().float()
        gp = torch.empty(T, N, 2, dtype=torch.float32, device=g.device)
        for j in range(T):
            L.check(L.lib().atlb_splat_gauss_bwd_pos(L.ptr(g[j * B:(j + 1) * B]), L.ptr(w[j]), N, B, H, W, sigma,
                                                      radius, L.ptr(gp[j]), L.ptr(ctx.wss[j]), nb, L.stream()),
                    "splat_slices_bwd")
        ctx.wss = None
        return gp, None, None, None, None, None, None, None


def splat_slices(pos: torch.Tensor, w: torch.Tensor, b: torch.Tensor, B: int, H: int, W: int, sigma: float,
                 radius: int | None = None) -> torch.Tensor:
    """Gaussian splat of T point sets (pos (T, N, 2), weights w (T, N), batch index b (N) shared) into a
    (T * B, H, W) image stack: ``splat(pos[j], w[j], b, B, H, W, "gauss", sigma)`` for each j, stacked.
    Gradient w.r.t. ``pos`` only."""
    _need_cuda(pos, "splat_slices")
    radius = int(math.ceil(3 * sigma)) if radius is None else radius
    return _SplatSlices.apply(pos, w, b, B, H, W, float(sigma), int(radius))


# ------------------------------------------------------------------------------------------- gather
class _Gather(torch.autograd.Function):
    """atl/ops/functional.py:69-80."""
    @staticmethod
    def forward(ctx, img, pos, b):
        img, pos, b = _f32(img), _f32(pos), b.contiguous().long()
        ctx.save_for_backward(img, pos, b)
        return get_ext().gather_bilinear_fwd(img, pos, b)

    @staticmethod
    def backward(ctx, g):
        img, pos, b = ctx.saved_tensors
        gi, gp = get_ext().gather_bilinear_bwd(g.contiguous().float(), img, pos, b)
        return gi, gp, None


def gather(img: torch.Tensor, pos: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Bilinear sample of a (B, H, W) image at event positions, zero outside (functional.py:83-87)."""
    _need_cuda(pos, "gather")
    return _Gather.apply(img, pos, b)


# ------------------------------------------------------------------------------------------- blur
def gaussian_kernel1d(sigma: float, device, dtype=torch.float32) -> torch.Tensor:
    """The normalised 1-D Gaussian kernel of radius max(ceil(3 sigma), 1) that :func:`blur` applies
    (atl/ops/functional.py:89-96): fp32 exp(-i^2 / (2 sigma^2)) for i = -r..r, divided by their sum."""
    r = max(int(math.ceil(3 * sigma)), 1)
    i = np.arange(-r, r + 1, dtype=np.float32)
    k = np.exp(-(i * i) / np.float32(2 * sigma * sigma), dtype=np.float32)
    return torch.as_tensor(k / k.sum(dtype=np.float32), device=device).to(dtype)


class _Blur(torch.autograd.Function):
    """Separable Gaussian blur on the device (atlb_blur).  The zero-padded convolution with a symmetric kernel
    is self-adjoint, so the backward is the same blur of the incoming gradient."""

    @staticmethod
    def forward(ctx, img, sigma):
        ctx.sigma = sigma
        return get_ext().blur(_f32(img), sigma)

    @staticmethod
    def backward(ctx, g):
        return get_ext().blur(_f32(g), ctx.sigma), None


def blur(img: torch.Tensor, sigma: float) -> torch.Tensor:
    """Separable Gaussian blur of a (B, H, W) or (B, C, H, W) image, zero padding, normalised kernel of radius
    max(ceil(3 sigma), 1) (atl/ops/functional.py:99-110; baseline IWEs, not the anchored path)."""
    if sigma <= 0:
        return img
    _need_cuda(img, "blur")
    return _Blur.apply(img, float(sigma)).to(img.dtype)


# ------------------------------------------------------------------------------------------- anchored pairs
@dataclass
class PairPlan:
    """Spatial hash of (source, slice) entries sorted by (batch, slice, cell) (functional.py:114-129),
    built on the device by :func:`build_pair_plan`."""
    src_y: torch.Tensor
    src_v: torch.Tensor
    src_t: torch.Tensor
    src_id: torch.Tensor
    cell_start: torch.Tensor
    anc_x: torch.Tensor
    anc_t: torch.Tensor
    anc_cell: torch.Tensor
    anc_id: torch.Tensor
    slice_c: torch.Tensor
    S: int
    GH: int
    GW: int


def plan_geometry(x, v, anchors, anchor_xy, H, W, h, cut, n_slices) -> L.PlanGeom:
    """vmax, cell size, grid origin and extent (functional.py:136-149); reads 6 numbers back.
    ``anchor_xy`` None means the anchors sit at x[anchors]."""
    lib = L.lib()
    geom = L.PlanGeom()
    scratch = torch.empty(64, dtype=torch.uint8, device=v.device)
    L.check(lib.atlb_plan_geometry(L.ptr(x), L.ptr(v), v.shape[0], L.ptr(anchors), L.ptr(anchor_xy),
                                   anchors.shape[0], H, W, float(h), float(cut), int(n_slices), L.ptr(scratch),
                                   ctypes.byref(geom), L.stream()), "plan_geometry")
    return geom


def build_pair_plan(x, t, v, b, B, H, W, anchors, h, tau, cut=3.0, n_slices=16, anchor_xy=None) -> PairPlan:
    """Device counting-sort replacement of functional.py:132-178; bit-identical keys, CSR offsets and
    anchor cells.  Two small device-to-host reads (grid geometry, entry count), like the reference's
    ``float(...)`` reads."""
    _need_cuda(x, "build_pair_plan")
    lib = L.lib()
    dev = x.device
    S = int(n_slices)
    with torch.no_grad():
        xf = x.detach().float().contiguous()
        tf = t.detach().float().contiguous()
        vd = v.detach().float().contiguous()
        bl = b.contiguous().long()
        anc = anchors.contiguous().long()
        axy = None if anchor_xy is None else anchor_xy.detach().float().contiguous()
        if axy is not None and axy.shape[0] != anc.shape[0]:
            raise ValueError("anchor_xy must have one row per anchor")
        geom = plan_geometry(xf, vd, anc, axy, H, W, h, cut, S)
        GH, GW = int(geom.GH), int(geom.GW)
        ncell = B * S * GH * GW
        cell_start = torch.empty(ncell + 1, dtype=torch.int64, device=dev)
        nb = lib.atlb_plan_workspace_bytes(ncell)
        ws = L.workspace(nb, dev)
        ns = ctypes.c_int64(0)
        N, M = tf.shape[0], anc.shape[0]
        L.check(lib.atlb_plan_count(L.ptr(xf), L.ptr(tf), L.ptr(vd), L.ptr(bl), N, B, float(tau), ctypes.byref(geom),
                                    L.ptr(cell_start), L.ptr(ws), nb, ctypes.byref(ns), L.stream()), "plan_count")
        Ns = int(ns.value)
        src_y = torch.empty(Ns, 2, dtype=torch.float32, device=dev)
        src_v = torch.empty(Ns, 2, dtype=torch.float32, device=dev)
        src_t = torch.empty(Ns, dtype=torch.float32, device=dev)
        src_id = torch.empty(Ns, dtype=torch.int64, device=dev)
        anc_x = torch.empty(M, 2, dtype=torch.float32, device=dev)
        anc_t = torch.empty(M, dtype=torch.float32, device=dev)
        anc_cell = torch.empty(M, 3, dtype=torch.int64, device=dev)
        anc_id = torch.empty(M, dtype=torch.int64, device=dev)
        slice_c = torch.empty(S, dtype=torch.float32, device=dev)
        L.check(lib.atlb_plan_fill(L.ptr(xf), L.ptr(tf), L.ptr(vd), L.ptr(bl), N, B, float(tau), ctypes.byref(geom),
                                   L.ptr(anc), L.ptr(axy), M, L.ptr(cell_start), L.ptr(ws), nb, L.ptr(src_y),
                                   L.ptr(src_v), L.ptr(src_t), L.ptr(src_id), L.ptr(anc_x), L.ptr(anc_t),
                                   L.ptr(anc_cell), L.ptr(anc_id), L.ptr(slice_c), L.stream()), "plan_fill")
    return PairPlan(src_y, src_v, src_t, src_id, cell_start, anc_x, anc_t, anc_cell, anc_id, slice_c, S, GH, GW)


class _ATSPair(torch.autograd.Function):
    """atl/ops/functional.py:181-196."""
    @staticmethod
    def forward(ctx, v, plan: PairPlan, h, tau, cut):
        e = get_ext()
        ctx.plan, ctx.args, ctx.n = plan, (float(h), float(tau), float(cut)), v.shape[0]
        p = plan
        return e.ats_pair_fwd(p.src_y, p.src_v, p.src_t, p.src_id, p.cell_start, p.anc_x, p.anc_t, p.anc_cell,
                              p.anc_id, p.slice_c, p.S, p.GH, p.GW, *ctx.args)

    @staticmethod
    def backward(ctx, g):
        p = ctx.plan
        gv = get_ext().ats_pair_bwd(g.contiguous().float(), p.src_y, p.src_v, p.src_t, p.src_id, p.cell_start,
                                    p.anc_x, p.anc_t, p.anc_cell, p.anc_id, p.slice_c, p.S, p.GH, p.GW,
                                    *ctx.args, ctx.n)
        return gv, None, None, None, None


def ats_pair_sums(x, t, v, b, B, H, W, anchors, h, tau, cut=3.0, n_slices=16, force_ref=False, anchor_xy=None):
    """S_i = sum_{j != i} 1[|t_i - t_j| <= tau] exp(-|x_i - x_j - v_j (t_i - t_j)|^2 / 2h^2) for anchors i
    (atl/ops/functional.py:199-207).  Gradient flows to ``v`` only.  ``force_ref`` selected the
    reference's brute-force torch path, which this library does not ship."""
    if force_ref:
        raise ValueError("x_b200.ats_pair_sums: force_ref (torch brute force) is not part of the B200 path")
    _need_cuda(x, "ats_pair_sums")
    plan = build_pair_plan(x, t, v, b, B, H, W, anchors, h, tau, cut, n_slices, anchor_xy=anchor_xy)
    return _ATSPair.apply(v.float(), plan, h, tau, cut)


def window_counts(t: torch.Tensor, b: torch.Tensor, idx: torch.Tensor, tau: float) -> torch.Tensor:
    """#{j != i, same batch, |t_j - t_i| <= tau} for i in idx (functional.py:210-217).  Sorted (b, t)
    events are searched directly; otherwise the float64 keys are sorted first, as the reference does."""
    _need_cuda(t, "window_counts")
    lib = L.lib()
    tf, bl, il = t.detach().float().contiguous(), b.contiguous().long(), idx.contiguous().long()
    out = torch.empty(il.shape[0], dtype=torch.float32, device=t.device)
    scratch = torch.empty(16, dtype=torch.uint8, device=t.device)
    st = lib.atlb_window_counts(L.ptr(tf), L.ptr(bl), tf.shape[0], L.ptr(il), il.shape[0], float(tau), L.ptr(out),
                                L.ptr(scratch), L.stream())
    if st == L.ATLB_ERR_UNSORTED:
        ks = torch.sort(bl.double() * 4.0 + tf.double()).values.contiguous()
        st = lib.atlb_window_counts_keys(L.ptr(ks), tf.shape[0], L.ptr(tf), L.ptr(bl), L.ptr(il), il.shape[0],
                                         float(tau), L.ptr(out), L.stream())
    L.check(st, "window_counts")
    return out.to(t.dtype)


# ------------------------------------------------------------------------------------------- voxel grid
def voxel_grid(pos, t, p, b, B, C, H, W, normalize: str | None = "mean_std") -> torch.Tensor:
    """Trilinear polarity voxel grid (B, C, H, W) (functional.py:221-238)."""
    _need_cuda(pos, "voxel_grid")
    with torch.no_grad():
        vox = get_ext().voxel_grid(_f32(pos), _f32(t), _f32(p), b.contiguous().long(), B, C, H, W)
        if normalize == "mean_std":
            for k in range(B):
                v = vox[k]
                nz = v != 0
                if nz.any():
                    m, s = v[nz].mean(), v[nz].std()
                    v[nz] = (v[nz] - m) / s if s > 0 else v[nz] - m
        elif normalize == "max":
            mx = vox.abs().amax(dim=(1, 2, 3), keepdim=True).clamp(min=1e-9)
            vox = vox / mx
    return vox
