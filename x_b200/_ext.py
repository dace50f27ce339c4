"""The extension surface the reference's autograd functions call (``get_ext()`` of atl/ops/_ext.py:16-42),
backed by libatlb200.so instead of the reference's pybind11 module (csrc/atl_cpu.cpp:299-329).

Same method names, argument order and return values as the reference's bindings; tensors must be
contiguous CUDA tensors of the reference's dtypes (float32 data, int64 indices), otherwise a
RuntimeError is raised (the reference raises from TORCH_CHECK, csrc/atl_cpu.cpp:11-14).  Outputs are
allocated here with torch (the reference returned ``torch::zeros`` tensors).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib as L

F32, I64 = torch.float32, torch.int64


def _empty(shape, like, dtype=F32):
    return torch.empty(shape, dtype=dtype, device=like.device)


class _AtlB200Ext:
    """Drop-in for the reference's ``atl_ops_cuda`` module object."""
    with_cuda = True

    # ---------------------------------------------------------------------------- splat / gather / voxel
    def splat_bilinear_fwd(self, pos, w, b, B, H, W):
        L.require_cuda("pos", pos, F32); L.require_cuda("w", w, F32); L.require_cuda("bidx", b, I64)
        img = _empty((B, H, W), pos)
        nb = L.lib().atlb_tile_ops_workspace_bytes(pos.shape[0], B, H, W)
        ws = L.workspace(nb, pos.device)
        L.check(L.lib().atlb_splat_bilinear_fwd(L.ptr(pos), L.ptr(w), L.ptr(b), pos.shape[0], B, H, W, L.ptr(img),
                                                 L.ptr(ws), nb, L.stream()), "splat_bilinear_fwd")
        return img

    def splat_bilinear_bwd(self, g, pos, w, b):
        L.require_cuda("gimg", g, F32); L.require_cuda("pos", pos, F32)
        gp, gw = torch.empty_like(pos), torch.empty_like(w)
        B, H, W = g.shape
        nb = L.lib().atlb_tile_ops_workspace_bytes(pos.shape[0], B, H, W)
        ws = L.workspace(nb, pos.device)
        L.check(L.lib().atlb_splat_bilinear_bwd(L.ptr(g), L.ptr(pos), L.ptr(w), L.ptr(b), pos.shape[0], B, H, W,
                                                 L.ptr(gp), L.ptr(gw), L.ptr(ws), nb, L.stream()),
                "splat_bilinear_bwd")
        return [gp, gw]

    def splat_gauss_fwd(self, pos, w, b, B, H, W, sigma, R):
        L.require_cuda("pos", pos, F32); L.require_cuda("w", w, F32); L.require_cuda("bidx", b, I64)
        img = _empty((B, H, W), pos)
        nb = L.lib().atlb_splat_gauss_workspace_bytes(pos.shape[0], B, H, W)
        ws = L.workspace(nb, pos.device)
        L.check(L.lib().atlb_splat_gauss_fwd(L.ptr(pos), L.ptr(w), L.ptr(b), pos.shape[0], B, H, W, float(sigma),
                                              int(R), L.ptr(img), L.ptr(ws), nb, L.stream()), "splat_gauss_fwd")
        return img

    def splat_gauss_bwd(self, g, pos, w, b, sigma, R):
        L.require_cuda("gimg", g, F32); L.require_cuda("pos", pos, F32)
        gp, gw = torch.empty_like(pos), torch.empty_like(w)
        B, H, W = g.shape
        nb = L.lib().atlb_splat_gauss_workspace_bytes(pos.shape[0], B, H, W)
        ws = L.workspace(nb, pos.device)
        L.check(L.lib().atlb_splat_gauss_bwd(L.ptr(g), L.ptr(pos), L.ptr(w), L.ptr(b), pos.shape[0], B, H, W,
                                              float(sigma), int(R), L.ptr(gp), L.ptr(gw), L.ptr(ws), nb, L.stream()),
                "splat_gauss_bwd")
        return [gp, gw]

    def gather_bilinear_fwd(self, img, pos, b):
        L.require_cuda("img", img, F32); L.require_cuda("pos", pos, F32); L.require_cuda("bidx", b, I64)
        out = _empty((pos.shape[0],), pos)
        B, H, W = img.shape
        nb = L.lib().atlb_tile_ops_workspace_bytes(pos.shape[0], B, H, W)
        ws = L.workspace(nb, pos.device)
        L.check(L.lib().atlb_gather_bilinear_fwd(L.ptr(img), L.ptr(pos), L.ptr(b), pos.shape[0], B, H, W, L.ptr(out),
                                                  L.ptr(ws), nb, L.stream()), "gather_bilinear_fwd")
        return out

    def gather_bilinear_bwd(self, g, img, pos, b):
        L.require_cuda("gval", g, F32); L.require_cuda("img", img, F32)
        gi, gp = torch.empty_like(img), torch.empty_like(pos)
        B, H, W = img.shape
        nb = L.lib().atlb_tile_ops_workspace_bytes(pos.shape[0], B, H, W)
        ws = L.workspace(nb, pos.device)
        L.check(L.lib().atlb_gather_bilinear_bwd(L.ptr(g), L.ptr(img), L.ptr(pos), L.ptr(b), pos.shape[0], B, H, W,
                                                  L.ptr(gi), L.ptr(gp), L.ptr(ws), nb, L.stream()),
                "gather_bilinear_bwd")
        return [gi, gp]

    def voxel_grid(self, pos, t, p, b, B, C, H, W):
        for n, x in (("pos", pos), ("t", t), ("p", p)):
            L.require_cuda(n, x, F32)
        L.require_cuda("bidx", b, I64)
        vox = _empty((B, C, H, W), pos)
        nb = L.lib().atlb_tile_ops_workspace_bytes(pos.shape[0], B, H, W)
        ws = L.workspace(nb, pos.device)
        L.check(L.lib().atlb_voxel_grid(L.ptr(pos), L.ptr(t), L.ptr(p), L.ptr(b), pos.shape[0], B, C, H, W,
                                         L.ptr(vox), L.ptr(ws), nb, L.stream()), "voxel_grid")
        return vox

    def blur(self, img, sigma):
        """Separable Gaussian blur of (P, H, W) planes (atl/ops/functional.py:99-110), zero padding."""
        L.require_cuda("img", img, F32)
        x = img.contiguous()
        out = torch.empty_like(x)
        P = x.numel() // (x.shape[-1] * x.shape[-2]) if x.numel() else 0
        L.check(L.lib().atlb_blur(L.ptr(x), P, x.shape[-2], x.shape[-1], float(sigma), L.ptr(out), L.stream()), "blur")
        return out

    # ---------------------------------------------------------------------------- anchored pairs
    @staticmethod
    def _pair_args(sy, sv, st, sid, cs, ax, at, ac, aid, sc):
        for n, x, dt in (("src_y", sy, F32), ("src_v", sv, F32), ("src_t", st, F32), ("src_id", sid, I64),
                         ("cell_start", cs, I64), ("anc_x", ax, F32), ("anc_t", at, F32), ("anc_cell", ac, I64),
                         ("anc_id", aid, I64), ("slice_c", sc, F32)):
            L.require_cuda(n, x, dt)
        return [L.ptr(x) for x in (sy, sv, st, sid, cs, ax, at, ac, aid, sc)]

    def ats_pair_fwd(self, sy, sv, st, sid, cs, ax, at, ac, aid, sc, S, GH, GW, h, tau, cut):
        args = self._pair_args(sy, sv, st, sid, cs, ax, at, ac, aid, sc)
        M, ncell, Ns = ax.shape[0], cs.shape[0] - 1, sy.shape[0]
        out = _empty((M,), ax)
        nb = L.lib().atlb_pair_workspace_bytes(M, ncell)
        ws = L.workspace(nb, ax.device)
        L.check(L.lib().atlb_ats_pair_fwd(*args, Ns, M, ncell, S, GH, GW, float(h), float(tau), float(cut), L.ptr(out),
                                           L.ptr(ws), nb, L.stream()), "ats_pair_fwd")
        return out

    def ats_pair_bwd(self, g, sy, sv, st, sid, cs, ax, at, ac, aid, sc, S, GH, GW, h, tau, cut, N):
        args = self._pair_args(sy, sv, st, sid, cs, ax, at, ac, aid, sc)
        L.require_cuda("gS", g, F32)
        M, ncell, Ns = ax.shape[0], cs.shape[0] - 1, sy.shape[0]
        gv = _empty((N, 2), ax)
        nb = L.lib().atlb_pair_workspace_bytes(M, ncell)
        ws = L.workspace(nb, ax.device)
        L.check(L.lib().atlb_ats_pair_bwd(L.ptr(g), *args, Ns, M, ncell, S, GH, GW, float(h), float(tau), float(cut),
                                           N, L.ptr(gv), L.ptr(ws), nb, L.stream()), "ats_pair_bwd")
        return gv


_EXT = None


def get_ext():
    """The libatlb200-backed extension (mirror of atl/ops/_ext.py:16-42).  Raises if it cannot run:
    there is no silent fallback to torch reference ops."""
    global _EXT
    if _EXT is None:
        L.lib()
        _EXT = _AtlB200Ext()
    return _EXT


def ext_supports(t: torch.Tensor) -> bool:
    """True for CUDA tensors (mirror of atl/ops/_ext.py:45-50); CPU tensors are not supported."""
    return bool(t.is_cuda)
