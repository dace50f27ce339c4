"""One large event window over several GPUs (one process per GPU, torch.distributed over NCCL).

The anchored score of a single window of N events (configuration 5: 64M events) is split by SOURCES.
Every rank prepares all N events and all M anchors, but builds the pair plan of its own contiguous share
of the events only (the events are (b, t)-sorted, so a share is a time slab).  Then:

    forward   S_r = pair sums of all anchors over rank r's sources      (libatlb200, src range)
              S   = all_reduce(sum) S_r                                  (NCCL, M floats)
              ls  = log(eps + S / den)                                   (every rank, identical)
    backward  gS from the full S; gv of rank r's sources and the motion gradient they produce
              gtheta = all_reduce(sum) gtheta_r                          (NCCL, |theta| floats)

so each pair (i, j) is evaluated once, on the rank that owns source j, and the only exchanges are the
M-float partial sums and the parameter gradient.  The normaliser (window counts, exposure correction)
uses all events and is evaluated on every rank.  Sum over ranks of the partial sums equals the
single-GPU sums (leave-one-out: the anchor's own pair is subtracted only on the rank that owns its
event); only the summation order differs.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib as L
from .events import EventPacket
from .objectives import AnchoredExact, _fused_kind


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous share [begin, end) of n items for ``rank`` of ``world`` (sizes differ by at most one)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    return n * rank // world, n * (rank + 1) // world


def allreduce_sum(t: torch.Tensor, group=None) -> torch.Tensor:
    """In-place sum over the ranks of ``group`` (identity without an initialised process group)."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


class ExactPartial:
    """The fused anchored-score pipeline restricted to the sources [src_begin, src_end): partial pair sums
    for every anchor, the normaliser, and the backward of those sources.  Holds the plan between the two."""

    def __init__(self, spec, theta, xy, t, b, anchors, u, z, src_begin: int, src_end: int):
        kind, B, H, W, h, tau, cut, eps_frac, S, visibility, n_check = spec
        lib = L.lib()
        dev = xy.device
        self.th = theta.detach().float().contiguous()
        Hg, Wg = (self.th.shape[-2], self.th.shape[-1]) if kind == L.MOTION_DENSE else (1, 1)
        self.cfg = L.ExactCfg(kind, self.th.data_ptr(), self.th.shape[0], Hg, Wg, B, H, W, float(h), float(tau),
                              float(cut), float(eps_frac), int(S), int(bool(visibility)), int(n_check),
                              int(src_begin), int(src_end))
        self.eps = float(eps_frac) / (H * W)
        xyc, tc, self.bc = xy.detach().float().contiguous(), t.detach().float().contiguous(), b.contiguous().long()
        self.N = N = tc.shape[0]
        anc = None if anchors is None else anchors.contiguous().long()
        self.M = M = N if anc is None else anc.shape[0]
        uc = None if u is None else u.detach().float().contiguous()
        zc = None if z is None else z.detach().float().contiguous()
        self.ev4 = torch.empty(N, 4, dtype=torch.float32, device=dev)
        anc4 = torch.empty(M, 4, dtype=torch.float32, device=dev)
        anc_b = torch.empty(M, dtype=torch.int64, device=dev)
        scratch = torch.empty(64, dtype=torch.uint8, device=dev)
        self.geom = L.PlanGeom()
        L.check(lib.atlb_exact_prepare(ctypes.byref(self.cfg), L.ptr(xyc), L.ptr(uc), L.ptr(tc), L.ptr(self.bc), N,
                                       L.ptr(anc), L.ptr(zc), M, L.ptr(self.ev4), L.ptr(anc4), L.ptr(anc_b),
                                       L.ptr(scratch), ctypes.byref(self.geom), L.stream()), "exact_prepare")
        self.nb = lib.atlb_exact_workspace_bytes(ctypes.byref(self.cfg), N, M, ctypes.byref(self.geom))
        self.ws = L.workspace(self.nb, dev)
        self.S = torch.empty(M, dtype=torch.float32, device=dev)
        self.den = torch.empty(M, dtype=torch.float32, device=dev)
        ls = torch.empty(M, dtype=torch.float32, device=dev)
        L.check(lib.atlb_exact_forward(ctypes.byref(self.cfg), L.ptr(tc), L.ptr(self.bc), N, M, L.ptr(self.ev4),
                                       L.ptr(anc4), L.ptr(anc_b), ctypes.byref(self.geom), L.ptr(self.ws), self.nb,
                                       L.ptr(self.S), L.ptr(self.den), L.ptr(ls), L.stream()), "exact_forward")

    def log_scores(self, S_full: torch.Tensor) -> torch.Tensor:
        """ls = log(eps + S / den), the fused kernel's expression (fp32 division, add, log)."""
        return torch.log(self.eps + S_full / self.den)

    def backward(self, grad_ls: torch.Tensor, S_full: torch.Tensor, theta_shape) -> torch.Tensor:
        """Motion-parameter gradient produced by this call's sources, given dL/dls and the full sums."""
        self.cfg.theta = self.th.data_ptr()
        gv = torch.empty(self.N, 2, dtype=torch.float32, device=self.ev4.device)
        gth = torch.empty(theta_shape, dtype=torch.float32, device=self.ev4.device)
        L.check(L.lib().atlb_exact_backward(ctypes.byref(self.cfg), L.ptr(grad_ls.contiguous().float()),
                                            L.ptr(self.bc), self.N, self.M, L.ptr(self.ev4), ctypes.byref(self.geom),
                                            L.ptr(self.ws), self.nb, L.ptr(S_full.contiguous()), L.ptr(self.den),
                                            L.ptr(gv), L.ptr(gth), L.stream()), "exact_backward")
        return gth


class _ShardedExact(torch.autograd.Function):
    @staticmethod
    def forward(ctx, theta, xy, t, b, anchors, u, z, spec, src, group):
        part = ExactPartial(spec, theta, xy, t, b, anchors, u, z, *src)
        S = allreduce_sum(part.S, group)
        ctx.part, ctx.S, ctx.group, ctx.meta = part, S, group, (theta.dtype, tuple(theta.shape))
        return part.log_scores(S)

    @staticmethod
    def backward(ctx, grad_ls):
        dtype, shape = ctx.meta
        gth = allreduce_sum(ctx.part.backward(grad_ls, ctx.S, shape), ctx.group)
        return gth.to(dtype), None, None, None, None, None, None, None, None, None


class ShardedAnchoredExact(AnchoredExact):
    """AnchoredExact over one window whose sources are split across the ranks of ``group``.  Every rank
    passes the same events, motion and noise (the reference's seeded draws) and receives the same scores
    and the same, fully reduced, parameter gradient."""

    def __init__(self, *args, group=None, rank: Optional[int] = None, world: Optional[int] = None, **kw):
        super().__init__(*args, **kw)
        import torch.distributed as dist
        live = dist.is_available() and dist.is_initialized()
        self.group = group
        self.rank = rank if rank is not None else (dist.get_rank(group) if live else 0)
        self.world = world if world is not None else (dist.get_world_size(group) if live else 1)

    def log_scores(self, ev: EventPacket, motion, anchors=None, noise=None):
        kind = _fused_kind(motion)
        if kind < 0 or not ev.xy.is_cuda:
            raise ValueError("ShardedAnchoredExact needs a CUDA window and a Translation / Affine / DenseLinearFlow "
                             "motion in linear mode")
        anchors, u, z = self.draw(ev, anchors) if noise is None else noise
        spec = (kind, ev.batch_size, ev.height, ev.width, self.h, self.tau, self.cut, self.eps_frac,
                self.n_slices, self.visibility, 16)
        src = shard_range(ev.n, self.rank, self.world)
        ls = _ShardedExact.apply(motion.theta, ev.xy, ev.t, ev.b, anchors, u if self.dequantize else None,
                                 z if self.smooth_anchors else None, spec, src, self.group)
        return ls, anchors
