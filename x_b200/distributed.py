"""Large event windows over several GPUs (one process per GPU, torch.distributed over NCCL).

AnchoredSliced (``ShardedAnchoredSliced``): the events are split across the ranks.  Each rank moves its
share of the events to every slice centre and splats it into a partial density stack (slices x B x H x W);
the partial stacks and the per-(slice, batch) source counts are summed with an all-reduce; each rank then
gathers and scores the anchors among its own events against the full density.  The backward all-reduces
dL/d(density) the same way, so each rank's splat backward sees every rank's anchors.

AnchoredExact (``ShardedAnchoredExact``):

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
from .objectives import AnchoredExact, AnchoredSliced, _fused_kind, slice_counts


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


class _AllReduceSum(torch.autograd.Function):
    """y = the sum over the ranks of x; the gradient of each rank's x is the sum over the ranks of dL/dy
    (every rank's loss reads the same y)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return allreduce_sum(x.detach().clone(), group)

    @staticmethod
    def backward(ctx, g):
        return allreduce_sum(g.contiguous().clone(), ctx.group), None


def allreduce_sum_autograd(x: torch.Tensor, group=None) -> torch.Tensor:
    """Differentiable all-reduce (sum) over ``group``: see :class:`_AllReduceSum`."""
    return _AllReduceSum.apply(x, group)


class ShardedAnchoredSliced(AnchoredSliced):
    """AnchoredSliced over windows whose events are split across the ranks of ``group`` (the north star's
    multi-GPU design for the splat path: local splat, NCCL all-reduce of the density, local gather and score).

    Every rank passes the same events, motion and noise.  Rank r takes the contiguous share
    ``shard_range(ev.n, r, world)`` of the events as its sources and anchor candidates.  ``log_scores``
    returns the scores of the rank's own anchors (ordered by slice, then event index) and their global
    event indices; :meth:`__call__` returns this rank's part of the loss, -sum(ls_r) / M (M = anchors of
    all ranks), whose sum over the ranks is the loss -mean(ls).  After ``backward``,
    :meth:`reduce_gradients` sums the parameter gradients over the ranks (each rank's gradient holds its
    own sources and anchors).  n_anchors_per_slice (a random subset of each slice over the whole window) is
    not supported here."""

    def __init__(self, *args, group=None, rank: Optional[int] = None, world: Optional[int] = None, **kw):
        super().__init__(*args, **kw)
        if self.nap is not None:
            raise ValueError("ShardedAnchoredSliced: n_anchors_per_slice draws over the whole window; not sharded")
        import torch.distributed as dist
        live = dist.is_available() and dist.is_initialized()
        self.group = group
        self.rank = rank if rank is not None else (dist.get_rank(group) if live else 0)
        self.world = world if world is not None else (dist.get_world_size(group) if live else 1)

    def log_scores(self, ev: EventPacket, motion, anchor_mask=None, source_mask=None, noise=None):
        e0, e1 = shard_range(ev.n, self.rank, self.world)
        st = self._setup(ev, noise, anchor_mask, source_mask, e0, e1)
        img_r, per_kb_r = self._density(st, motion)
        img = allreduce_sum_autograd(img_r, self.group)
        per_kb = allreduce_sum(per_kb_r, self.group)  # integer-valued: exact in fp32 below 2^24 per bin
        counts = allreduce_sum(slice_counts(ev, t=st["t"], b=st["b"]), self.group) if self.visibility else None
        picked = self._pick(st)
        if picked is None:  # no anchors here: an empty result that still reads the density, so that the
            z0 = img.reshape(-1)[:0]  # backward all-reduce runs on this rank as on the others
            return z0, torch.zeros(0, dtype=torch.long, device=ev.device)
        ai, ka = picked
        return self._scores(st, motion, img, per_kb, counts, ai, ka), ai + e0

    def __call__(self, ev, motion, noise=None):
        ls, _ = self.log_scores(ev, motion, noise=noise)
        m = allreduce_sum(torch.tensor([float(ls.numel())], device=ls.device), self.group)
        part = -ls.sum() / m.clamp(min=1)[0]
        total = allreduce_sum(part.detach().clone(), self.group)
        return {"loss": part, "score": -total}

    def reduce_gradients(self, tensors) -> None:
        """Sum the ``.grad`` of each tensor over the ranks (after backward)."""
        for p in tensors:
            if p.grad is not None:
                allreduce_sum(p.grad, self.group)

