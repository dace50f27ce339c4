"""Anchored transport score on B200 -- mirror of atl/objectives/ats.py (AnchoredExact, AnchoredSliced).

    S(theta) = mean_i log( eps + rho_{-i}(x_i) ),
    rho_{-i}(x) = (1 / W_i) sum_{j != i, |t_i - t_j| <= tau} K_h( x - Phi_{t_j -> t_i}(x_j) )

Same constructors, same random draws (the objective's CPU ``torch.Generator``) and same outputs as
the reference.  Stage kernels come from libatlb200 through x_b200.functional; the exposure
correction runs as one fused kernel for the motion models of x_b200.motion.  ``log_scores`` also
accepts pre-drawn noise (``noise=(u, z)``), which is how the benchmark keeps the host RNG out of a
device-resident step.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _lib as L
from . import rng as R
from .events import EventPacket
from .functional import ats_pair_sums, gather, splat, splat_slices, window_counts
from .motion import VectorFieldMotion


def _fused_kind(motion) -> int:
    """libatlb200 motion kind if the motion's transport is the linear warp of a fused field, else -1."""
    if isinstance(motion, VectorFieldMotion) and motion.kind >= 0 and motion.mode == "linear":
        return motion.kind
    return -1


@torch.no_grad()
def count_keys(key: torch.Tensor, nbins: int, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Exact counts of the keys in [0, nbins) (atlb_count_keys), int64: (nbins,) without ``mask``, else
    (R, nbins) counting, for each row r of the (R, N) ``mask``, the keys where mask[r] != 0."""
    if not key.is_cuda:
        raise RuntimeError("x_b200.count_keys: expected CUDA tensors (there is no CPU path)")
    kc = key.contiguous().long()
    mc = None if mask is None else mask.reshape(-1, kc.shape[0]).float().contiguous()
    R = 1 if mc is None else mc.shape[0]
    out = torch.empty(R, nbins, dtype=torch.int64, device=key.device)
    L.check(L.lib().atlb_count_keys(L.ptr(kc), kc.shape[0], nbins, L.ptr(mc), R, L.ptr(out), L.stream()),
            "count_keys")
    return out[0] if mc is None else out


@torch.no_grad()
def slice_counts(ev: EventPacket, n_check: int = 16, t: Optional[torch.Tensor] = None,
                 b: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-batch event counts in ``n_check`` equal time slices (ats.py:40-42), as exact integer counts
    (not an accumulating scatter of ones), float32 (B, n_check); of the events (t, b) when given (a share of
    the window's events), else of all of ``ev``'s."""
    t = ev.t if t is None else t
    b = ev.b if b is None else b
    sl = torch.clamp((t * n_check).long(), 0, n_check - 1)
    key = torch.where((b >= 0) & (b < ev.batch_size), b * n_check + sl, -1)
    return count_keys(key, ev.batch_size * n_check).view(ev.batch_size, n_check).to(torch.float32)


@torch.no_grad()
def visible_fraction(motion, xa, ta, ba, ev: EventPacket, tau: float, n_check: int = 16,
                     counts: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Exposure correction (atl/objectives/ats.py:31-50): fraction of the anchor's source mass recorded
    while its scene point was inside the image, checked at ``n_check`` slice centres.  ``counts``: the
    window's :func:`slice_counts`, when the caller evaluates several anchor sets of one window."""
    kind = _fused_kind(motion)
    if kind >= 0 and xa.is_cuda:
        th = motion.theta.detach().float().contiguous()
        Hg, Wg = (th.shape[-2], th.shape[-1]) if kind == L.MOTION_DENSE else (1, 1)
        xac, tac, bac = xa.detach().float().contiguous(), ta.detach().float().contiguous(), ba.contiguous().long()
        out = torch.empty(tac.shape[0], dtype=torch.float32, device=xa.device)
        scratch = torch.empty(ev.batch_size * n_check * 4 + 16, dtype=torch.uint8, device=xa.device)
        tf, bl = ev.t.float().contiguous(), ev.b.contiguous().long()
        L.check(L.lib().atlb_visible_fraction(kind, L.ptr(th), th.shape[0], Hg, Wg, ev.height, ev.width, L.ptr(xac),
                                              L.ptr(tac), L.ptr(bac), tac.shape[0], L.ptr(tf), L.ptr(bl), tf.shape[0],
                                              float(tau), int(n_check), L.ptr(out), L.ptr(scratch), L.stream()),
                "visible_fraction")
        return out.to(ta.dtype)
    # other motion models: the anchors moved to all check centres in one call of the motion's own transport
    edges = torch.linspace(0, 1, n_check + 1, device=ev.device)
    cen = (0.5 * (edges[:-1] + edges[1:])).contiguous()  # the fp32 centres
    if counts is None:
        counts = slice_counts(ev, n_check)
    if getattr(motion, "_device_transport", None) is not None and motion._device_transport(xa, ta):
        return motion.visible_fraction(xa, ta, ba, counts.contiguous(), cen, float(tau), ev.height, ev.width)
    M = ta.shape[0]
    y = motion.transport(xa.repeat(n_check, 1), ta.repeat(n_check), cen.repeat_interleave(M),
                         ba.repeat(n_check)).view(n_check, M, 2)
    inside = (y[..., 0] >= 0) & (y[..., 0] <= ev.width - 1) & (y[..., 1] >= 0) & (y[..., 1] <= ev.height - 1)
    near = (ta[None, :] - cen[:, None]).abs() <= tau
    w = counts[ba].t() * near.to(ta.dtype)  # (n_check, M) integer-valued weights: every sum below is exact
    vis = (w * inside.to(ta.dtype)).sum(0)
    tot = w.sum(0)
    return (vis / tot.clamp(min=1)).clamp(min=1e-3)


# Workspace bytes for the fused pipeline's next window, per (device, motion kind, B, H, W, slices): the last
# window's need and a little slack.
_WS_HINT: dict = {}


class _FusedExact(torch.autograd.Function):
    """AnchoredExact.log_scores (ats.py:84-96) as one libatlb200 pipeline (atlb_exact_*), differentiable
    w.r.t. the motion parameters."""

    @staticmethod
    def forward(ctx, theta, xy, t, b, anchors, u, z, spec):
        kind, B, H, W, h, tau, cut, eps_frac, S, visibility, n_check, rng_bits, rng_seed, rng_call = spec
        lib = L.lib()
        dev = xy.device
        th = theta.detach().float().contiguous()
        Hg, Wg = (th.shape[-2], th.shape[-1]) if kind == L.MOTION_DENSE else (1, 1)
        cfg = L.ExactCfg(kind, th.data_ptr(), th.shape[0], Hg, Wg, B, H, W, float(h), float(tau), float(cut),
                         float(eps_frac), int(S), int(bool(visibility)), int(n_check))
        # noise drawn on the device inside the prepare kernels (device_rng objectives): bit 0 u, bit 1 z
        cfg.rng, cfg.rng_seed, cfg.rng_call = int(rng_bits), int(rng_seed) & (2**64 - 1), int(rng_call)
        xyc, tc, bc = xy.detach().float().contiguous(), t.detach().float().contiguous(), b.contiguous().long()
        N = tc.shape[0]
        anc = None if anchors is None else anchors.contiguous().long()
        M = N if anc is None else anc.shape[0]
        uc = None if u is None else u.detach().float().contiguous()
        zc = None if z is None else z.detach().float().contiguous()
        ev4 = torch.empty(N, 4, dtype=torch.float32, device=dev)
        anc4 = torch.empty(M, 4, dtype=torch.float32, device=dev)
        anc_b = torch.empty(M, dtype=torch.int64, device=dev)
        scratch = torch.empty(64, dtype=torch.uint8, device=dev)
        Sv = torch.empty(M, dtype=torch.float32, device=dev)
        den = torch.empty(M, dtype=torch.float32, device=dev)
        ls = torch.empty(M, dtype=torch.float32, device=dev)
        geom = L.PlanGeom()
        # The plan's workspace depends on the window's geometry, known only after the prepare kernels.  A workspace
        # sized from the previous window of this kind lets prepare and forward run as one call (no return to Python
        # between the geometry read-back and the forward's kernels); a short one falls back to two calls.
        key = (dev.index, kind, B, H, W, S)
        hint = _WS_HINT.get(key, 0)
        ws = L.workspace(hint, dev) if hint else None
        st = lib.atlb_exact_prepare_forward(ctypes.byref(cfg), L.ptr(xyc), L.ptr(uc), L.ptr(tc), L.ptr(bc), N,
                                            L.ptr(anc), L.ptr(zc), M, L.ptr(ev4), L.ptr(anc4), L.ptr(anc_b),
                                            L.ptr(scratch), ctypes.byref(geom), L.ptr(ws), hint, L.ptr(Sv),
                                            L.ptr(den), L.ptr(ls), L.stream())
        nb = hint
        if st in (L.ATLB_OK, L.ATLB_ERR_WORKSPACE):
            need = lib.atlb_exact_workspace_bytes(ctypes.byref(cfg), N, M, ctypes.byref(geom))
            _WS_HINT[key] = need + need // 32  # this window's size and a little slack for the next one
            if st == L.ATLB_ERR_WORKSPACE:
                nb = _WS_HINT[key]
                ws = L.workspace(nb, dev)
                st = lib.atlb_exact_forward(ctypes.byref(cfg), L.ptr(tc), L.ptr(bc), N, M, L.ptr(ev4), L.ptr(anc4),
                                            L.ptr(anc_b), ctypes.byref(geom), L.ptr(ws), nb, L.ptr(Sv), L.ptr(den),
                                            L.ptr(ls), L.stream())
        L.check(st, "exact_prepare_forward")
        ctx.save_for_backward(th, bc, ev4, ws, Sv, den)
        ctx.meta = (cfg, geom, nb, N, M, theta.dtype, tuple(theta.shape))
        ctx.S, ctx.den = Sv, den
        return ls

    @staticmethod
    def backward(ctx, grad_ls):
        th, bc, ev4, ws, Sv, den = ctx.saved_tensors
        cfg, geom, nb, N, M, dtype, shape = ctx.meta
        cfg.theta = th.data_ptr()
        gv = torch.empty(N, 2, dtype=torch.float32, device=ev4.device)
        gth = torch.empty(shape, dtype=torch.float32, device=ev4.device)
        L.check(L.lib().atlb_exact_backward(ctypes.byref(cfg), L.ptr(grad_ls.contiguous().float()), L.ptr(bc), N, M,
                                            L.ptr(ev4), ctypes.byref(geom), L.ptr(ws), nb, L.ptr(Sv), L.ptr(den),
                                            L.ptr(gv), L.ptr(gth), L.stream()), "exact_backward")
        return gth.to(dtype), None, None, None, None, None, None, None


def _pick_anchors(ev: EventPacket, n_anchors: Optional[int], gen: Optional[torch.Generator]) -> torch.Tensor:
    """ats.py:53-57."""
    if n_anchors is None or n_anchors >= ev.n:
        return torch.arange(ev.n, device=ev.device)
    idx = torch.randperm(ev.n, generator=gen, device="cpu")[:n_anchors].to(ev.device)
    return torch.sort(idx).values


class Objective:
    """Callable ``(events, motion) -> {'loss': ...}`` (atl/objectives/base.py:18-27)."""
    name = "objective"
    reference_frame = True

    def __call__(self, ev: EventPacket, motion) -> dict:
        raise NotImplementedError


class AnchoredExact(Objective):
    """Anchored transport score with the exact pair kernel (ats.py:60-105); motion linear at the event."""
    name = "ats_exact"
    reference_frame = False

    def __init__(self, h: float = 1.0, tau: float = 1.0, eps_frac: float = 1e-2, n_anchors: Optional[int] = 20000,
                 n_slices: int = 16, cut: float = 3.0, seed: Optional[int] = None, smooth_anchors: bool = True,
                 dequantize: bool = True, visibility: bool = True, anchor_margin: float = 0.0, fused: bool = True,
                 device_rng: bool = False):
        self.visibility, self.anchor_margin = visibility, anchor_margin
        self.fused = fused  # one libatlb200 pipeline for the motion fields it implements
        # opt-in: u and z from the device generator (x_b200.rng) instead of the host generator's stream
        self.device_draws = R.DeviceDraws(seed) if device_rng else None
        self.h, self.tau, self.eps_frac, self.n_anchors, self.n_slices, self.cut = h, tau, eps_frac, n_anchors, n_slices, cut
        self.smooth_anchors, self.dequantize = smooth_anchors, dequantize
        self.gen = torch.Generator().manual_seed(seed) if seed is not None else None

    def draw(self, ev: EventPacket, anchors: Optional[torch.Tensor] = None):
        """The objective's random draws (ats.py:79-88), in the reference's order: anchors, dequantisation
        jitter u ~ U[0,1)^2 per event, smoothing noise z ~ N(0, I) per anchor.  Returns (anchors, u, z)
        with u / z on the events' device (None when the option is off)."""
        anchors = self._anchors(ev, anchors)
        if self.device_draws is not None:  # opt-in device draws: the same numbers the fused path draws inline
            call = self.device_draws.next_call()
            u = R.uniform2(self.device_draws.seed, call, ev.n, ev.device) if self.dequantize else None
            z = R.normal2(self.device_draws.seed, call, anchors.numel(), ev.device) if self.smooth_anchors else None
            return anchors, u, z
        u = torch.rand(ev.xy.shape, generator=self.gen).to(ev.xy) if self.dequantize else None
        z = torch.randn((anchors.numel(), 2), generator=self.gen).to(ev.xy) if self.smooth_anchors else None
        return anchors, u, z

    def _anchors(self, ev: EventPacket, anchors: Optional[torch.Tensor]) -> torch.Tensor:
        if anchors is None:
            anchors = _pick_anchors(ev, self.n_anchors, self.gen)
            if self.anchor_margin > 0:
                anchors = anchors[ev.inside(ev.xy[anchors], margin=-self.anchor_margin)]
        return anchors

    def log_scores(self, ev: EventPacket, motion, anchors: Optional[torch.Tensor] = None, noise=None):
        """Per-anchor log predictive densities and the anchor indices (ats.py:75-96).  ``noise`` =
        (anchors, u, z) as returned by :meth:`draw` replaces the generator draws."""
        if not getattr(motion, "linear_at_event", False):
            raise ValueError("AnchoredExact needs a motion that is linear at the event; use AnchoredSliced")
        kind = _fused_kind(motion)
        fused = self.fused and kind >= 0 and ev.xy.is_cuda
        rng_bits, rng_seed, rng_call = 0, 0, 0
        if noise is None and fused and self.device_draws is not None:
            # device draws inside the fused pipeline's prepare kernels: no noise buffers
            anchors, u, z = self._anchors(ev, anchors), None, None
            rng_bits = (1 if self.dequantize else 0) | (2 if self.smooth_anchors else 0)
            rng_seed, rng_call = self.device_draws.seed, self.device_draws.next_call()
        else:
            anchors, u, z = self.draw(ev, anchors) if noise is None else noise
        if fused:
            spec = (kind, ev.batch_size, ev.height, ev.width, self.h, self.tau, self.cut, self.eps_frac,
                    self.n_slices, self.visibility, 16, rng_bits, rng_seed, rng_call)
            try:
                ls = _FusedExact.apply(motion.theta, ev.xy, ev.t, ev.b, anchors, u if self.dequantize else None,
                                       z if self.smooth_anchors else None, spec)
                return ls, anchors
            except RuntimeError as e:
                if "not sorted" not in str(e):
                    raise
                # unsorted events: the stage-by-stage path below sorts the window keys like the reference
                if rng_bits:  # the same draws, materialised
                    u = R.uniform2(rng_seed, rng_call, ev.n, ev.device) if self.dequantize else None
                    z = R.normal2(rng_seed, rng_call, anchors.numel(), ev.device) if self.smooth_anchors else None
        xs = ev.xy
        if self.dequantize:
            xs = xs + (u - 0.5)
        xa = xs[anchors]
        if self.smooth_anchors:
            xa = xa + self.h * z
        v = motion.velocity(xs, ev.t, ev.b)
        S = ats_pair_sums(xs, ev.t, v, ev.b, ev.batch_size, ev.height, ev.width, anchors, self.h, self.tau,
                          self.cut, self.n_slices, anchor_xy=xa)
        Wn = window_counts(ev.t, ev.b, anchors, self.tau).clamp(min=1)
        if self.visibility:
            Wn = Wn * visible_fraction(motion, xa.detach(), ev.t[anchors], ev.b[anchors], ev, self.tau)
        eps = self.eps_frac / (ev.height * ev.width)
        return torch.log(eps + S / (Wn * 2 * math.pi * self.h ** 2)), anchors

    def set_bandwidth(self, h: float):
        self.h = float(h)

    def __call__(self, ev, motion, noise=None):
        ls, _ = self.log_scores(ev, motion, noise=noise)
        s = ls.mean()
        return {"loss": -s, "score": s.detach()}


def _spatial_order(motion, xy: torch.Tensor, b: torch.Tensor) -> Optional[torch.Tensor]:
    """For trajectory motions evaluated on the device: a permutation of the points that sorts them by
    (batch, coefficient tile of their position), so that the lanes of a warp read the same coefficient
    samples; None for other motions (their transports read no per-position coefficients)."""
    if not (hasattr(motion, "transport_targets") and motion._device_transport(xy, xy[:, 0])):
        return None
    if xy.shape[0] < 2:
        return None
    tile, Hq, Wq = float(motion.tile), motion.Hq, motion.Wq
    cx = torch.clamp(torch.floor(xy[:, 0] / tile), 0, Wq - 1).to(torch.int32)
    cy = torch.clamp(torch.floor(xy[:, 1] / tile), 0, Hq - 1).to(torch.int32)
    key = (b.to(torch.int32) * Hq + cy) * Wq + cx
    return torch.sort(key).indices


class _SlicedScore(torch.autograd.Function):
    """AnchoredSliced's per-anchor score from the transported anchor records (atlb_sliced_score / _bwd):
    ls = log(eps + max(val - src loo(a, own), 0) / max(cnt vis, 1)) + log|det J| (ats.py:154-169),
    differentiable w.r.t. the records ``pos`` (N, P, 2) and the gathered density ``val``."""

    @staticmethod
    def forward(ctx, pos, val, cnt, vis, src, slots, sigma, delta, eps, H, W):
        P, ia, io, ip = slots
        posc, valc = pos.detach().float().contiguous(), val.detach().float().contiguous()
        cntc, srcc = cnt.float().contiguous(), src.float().contiguous()
        visc = None if vis is None else vis.float().contiguous()
        n = valc.shape[0]
        ls = torch.empty(n, dtype=torch.float32, device=valc.device)
        L.check(L.lib().atlb_sliced_score(n, P, ia, io, ip, L.ptr(posc), L.ptr(valc), L.ptr(cntc), L.ptr(visc),
                                          L.ptr(srcc), float(sigma), float(delta), float(eps), H, W, L.ptr(ls),
                                          L.stream()), "sliced_score")
        ctx.save_for_backward(posc, valc, cntc, srcc, *(() if visc is None else (visc,)))
        ctx.meta = (slots, float(sigma), float(delta), float(eps), H, W, pos.dtype, val.dtype)
        return ls.to(val.dtype)

    @staticmethod
    def backward(ctx, gls):
        posc, valc, cntc, srcc, *rest = ctx.saved_tensors
        visc = rest[0] if rest else None
        (P, ia, io, ip), sigma, delta, eps, H, W, pdt, vdt = ctx.meta
        n = valc.shape[0]
        gval = torch.empty_like(valc)
        gpos = torch.empty_like(posc)
        L.check(L.lib().atlb_sliced_score_bwd(n, P, ia, io, ip, L.ptr(gls.contiguous().float()), L.ptr(posc),
                                              L.ptr(valc), L.ptr(cntc), L.ptr(visc), L.ptr(srcc), sigma, delta, eps,
                                              H, W, L.ptr(gval), L.ptr(gpos), L.stream()), "sliced_score_bwd")
        return gpos.to(pdt), gval.to(vdt), None, None, None, None, None, None, None, None, None


class AnchoredSliced(Objective):
    """Anchored transport score for any motion model (ats.py:108-183): Gaussian splats at slice centres,
    anchors moved by the small step t_i -> c_s with the exact finite-difference log|det|."""
    name = "ats_sliced"
    reference_frame = False

    def __init__(self, n_slices: int = 10, slices_per_step: Optional[int] = None, sigma: float = 1.0,
                 tau: float = 1.0, eps_frac: float = 1e-2, n_anchors_per_slice: Optional[int] = None,
                 logdet: bool = True, seed: Optional[int] = None, smooth_anchors: bool = True,
                 dequantize: bool = True, visibility: bool = True, device_rng: bool = False):
        self.smooth_anchors, self.dequantize, self.visibility = smooth_anchors, dequantize, visibility
        self.S, self.sps, self.sigma, self.tau, self.eps_frac = n_slices, slices_per_step, sigma, tau, eps_frac
        self.device_draws = R.DeviceDraws(seed) if device_rng else None  # opt-in: see AnchoredExact
        self.nap, self.logdet = n_anchors_per_slice, logdet
        self.gen = torch.Generator().manual_seed(seed) if seed is not None else None

    def draw(self, ev: EventPacket):
        """The objective's random draws in the reference's order (ats.py:127-135): the slice subset (when
        slices_per_step < n_slices), dequantisation jitter u ~ U[0,1)^2 and anchor smoothing noise
        z ~ N(0, I) per event.  Returns (slices, u, z), u / z on the events' device (None when off)."""
        S = self.S
        slices = list(range(S))
        if self.sps is not None and self.sps < S:
            slices = torch.randperm(S, generator=self.gen)[: self.sps].tolist()
        if self.device_draws is not None:
            call = self.device_draws.next_call()
            u = R.uniform2(self.device_draws.seed, call, ev.n, ev.device) if self.dequantize else None
            z = R.normal2(self.device_draws.seed, call, ev.n, ev.device) if self.smooth_anchors else None
            return slices, u, z
        u = torch.rand(ev.xy.shape, generator=self.gen).to(ev.xy) if self.dequantize else None
        z = torch.randn(ev.xy.shape, generator=self.gen).to(ev.xy) if self.smooth_anchors else None
        return slices, u, z

    def log_scores(self, ev: EventPacket, motion, anchor_mask: Optional[torch.Tensor] = None,
                   source_mask: Optional[torch.Tensor] = None, noise=None):
        """Per-anchor log scores and anchor indices (ats.py:122-174).  ``noise`` = :meth:`draw`'s
        (slices, u, z) replaces the generator draws.

        All slices are evaluated at once: every event moved to every evaluated slice centre and splatted,
        weighted by its source mask, into a stack of len(slices) x B density images; every anchor's record
        (its position, the four log-determinant probes and its unsmoothed source copy) moved to its own
        slice centre; one gather and the fused per-anchor score kernel (atlb_sliced_score).  Anchors come
        out in the reference's order: slice by slice in ``slices`` order, ascending event index inside a
        slice (or the slice's random subset when n_anchors_per_slice is set, drawn as the reference draws
        it)."""
        st = self._setup(ev, noise, anchor_mask, source_mask, 0, ev.n)
        picked = self._pick(st)
        if picked is None:
            z0 = ev.t.new_zeros(0)
            return z0, z0.long()
        ai, ka = picked
        img, per_kb = self._density(st, motion)
        counts = slice_counts(ev) if self.visibility else None
        return self._scores(st, motion, img, per_kb, counts, ai, ka), ai

    # -- stages (also used by x_b200.distributed.ShardedAnchoredSliced over a share of the events) --------
    def _setup(self, ev: EventPacket, noise, anchor_mask, source_mask, e0: int, e1: int) -> dict:
        """Draws, jittered positions, slice ranks, centres and source masks of the events [e0, e1)."""
        S, dev = self.S, ev.device
        delta = 1.0 / S
        slices, u, z = self.draw(ev) if noise is None else noise
        part = (e0, e1) != (0, ev.n)
        cut = (lambda x: x[e0:e1]) if part else (lambda x: x)  # noqa: E731
        xy, t, b = cut(ev.xy), cut(ev.t), cut(ev.b)
        xs = xy + (cut(u) - 0.5) if self.dequantize else xy
        xsm = xs + self.sigma * cut(z) if self.smooth_anchors else xs
        Sp = len(slices)
        # slice of each event, floor(t / delta) divided (not multiplied by a reciprocal) as the CPU reference
        sl = torch.clamp(torch.floor(t / torch.tensor(delta, dtype=t.dtype, device=dev)), 0, S - 1).long()
        rank_of = torch.full((S,), Sp, dtype=torch.long)
        rank_of[torch.tensor(slices, dtype=torch.long)] = torch.arange(Sp)
        rank = rank_of.to(dev)[sl]  # position of the event's slice in `slices` (Sp: not evaluated)
        if anchor_mask is not None:
            rank = torch.where(cut(anchor_mask), rank, torch.full_like(rank, Sp))
        centres = torch.tensor([(s + 0.5) * delta for s in slices], dtype=t.dtype).to(dev)
        src = (t[None, :] - centres[:, None]).abs() <= torch.tensor(self.tau + delta / 2, dtype=t.dtype, device=dev)
        if source_mask is not None:
            src = src & cut(source_mask)[None, :]
        # every event an anchor candidate of an evaluated slice: the anchors are all of them, no count needed
        every = anchor_mask is None and Sp == S
        return dict(ev=ev, xy=xy, t=t, b=b, xs=xs, xsm=xsm, Sp=Sp, rank=rank, centres=centres, src=src,
                    eps=self.eps_frac / (ev.height * ev.width), every=every)

    def _pick(self, st: dict):
        """Anchors (indices into the setup's events) and their slice ranks, in the reference's order."""
        Sp, rank, dev = st["Sp"], st["rank"], st["t"].device
        if st.get("every") and self.nap is None:
            # every slice evaluated, no anchor mask, no per-slice subsets: every event is an anchor, in slice order,
            # so the step needs no per-slice counts on the host (and no synchronisation)
            if rank.numel() == 0:
                return None
            rank_sorted, order = torch.sort(rank.to(torch.int32), stable=True)
            return order, rank_sorted.long()
        n_anc = count_keys(rank, Sp).tolist()  # the one read-back of the step
        rank_sorted, order = torch.sort(rank.to(torch.int32), stable=True)  # 32-bit keys: a shorter radix sort
        rank_sorted = rank_sorted.long()
        pieces, ranks, off = [], [], 0
        for k in range(Sp):
            ai = order[off:off + n_anc[k]]
            off += n_anc[k]
            if ai.numel() == 0:
                continue
            if self.nap is not None and ai.numel() > self.nap:
                ai = ai[torch.randperm(ai.numel(), generator=self.gen)[: self.nap].to(dev)]
            pieces.append(ai)
            ranks.append(k)
        if not pieces:
            return None
        if self.nap is None:
            return order[:off], rank_sorted[:off]
        ka = torch.cat([torch.full((p.numel(),), k, dtype=torch.long, device=dev) for p, k in zip(pieces, ranks)])
        return torch.cat(pieces), ka

    def _density(self, st: dict, motion):
        """The setup's events at every evaluated slice centre, splatted with their source masks as weights
        (zero weights add nothing) into images k * B + b; and the sources per (slice, batch)."""
        ev, B = st["ev"], st["ev"].batch_size
        xs, t, b, wsrc = st["xs"], st["t"], st["b"], st["src"].to(st["xs"].dtype)
        per_kb = count_keys(b, B, wsrc).to(xs.dtype)
        order = _spatial_order(motion, xs, b)
        if order is not None:  # the events in coefficient-tile order: neighbouring lanes share their samples
            xs, t, b, wsrc = xs[order], t[order], b[order], wsrc[:, order]
            st["order"] = order  # kept for the anchors (_scores) with the gathered times and batch indices
            st["in_order"] = {"t": t, "b": b}
        Y = self._events_at_centres(motion, xs, t, b, st["centres"])
        return splat_slices(Y, wsrc, b, B, ev.height, ev.width, self.sigma), per_kb

    def _scores(self, st: dict, motion, img, per_kb, counts, ai, ka):
        """Log scores of the anchors ``ai`` (slice ranks ``ka``) against the full density stack ``img`` and
        source counts ``per_kb``; ``counts``: the window's exposure-check slice counts."""
        n = st["t"].shape[0]
        if "order" in st and ai.numel() == n:
            # every event is an anchor: evaluate them in the events' coefficient-tile order (the density's), and
            # return them in the reference's order (ai)
            order = st["order"]
            pos = torch.empty_like(order)
            pos[order] = torch.arange(n, device=order.device)
            ls = self._scores_in_order(st, motion, img, per_kb, counts, order, st["rank"][order], reuse=True)
            return ls.index_select(0, pos[ai])  # (its backward scatters without sorting)
        order = _spatial_order(motion, st["xsm"][ai], st["b"][ai])
        if order is not None:  # evaluated in coefficient-tile order, returned in the reference's order
            inv = torch.empty_like(order)
            inv[order] = torch.arange(order.numel(), device=order.device)
            ls = self._scores_in_order(st, motion, img, per_kb, counts, ai[order], ka[order])
            return ls.index_select(0, inv)  # (its backward scatters without sorting)
        return self._scores_in_order(st, motion, img, per_kb, counts, ai, ka)

    def _scores_in_order(self, st: dict, motion, img, per_kb, counts, ai, ka, reuse: bool = False):
        ev, B, xs, xsm = st["ev"], st["ev"].batch_size, st["xs"], st["xsm"]
        if reuse:  # ai is the density's event order: its times and batch indices are gathered already
            ta, ba = st["in_order"]["t"], st["in_order"]["b"]
        else:
            ta, ba = st["t"][ai], st["b"][ai]
        xa, ca = xsm[ai], st["centres"][ka]
        # anchor records at their slice centres: [x +- d e_x, x +- d e_y,] a [, unsmoothed copy], the probes
        # x + (d, 0), x - (d, 0), x + (0, d), x - (0, d) of Motion.transport_logdet (atl/motion/base.py:43-50,
        # d = 0.5) made with one broadcast add
        d = 0.5
        offs = [[d, 0.0], [-d, 0.0], [0.0, d], [0.0, -d]] if self.logdet else []
        ia = len(offs)
        offs.append([0.0, 0.0])
        io = ia + 1 if self.smooth_anchors else -1
        P = len(offs) + (1 if self.smooth_anchors else 0)
        rec = torch.empty(xa.shape[0], P, 2, dtype=xa.dtype, device=xa.device)
        torch.add(xa[:, None, :], xa.new_tensor(offs)[None], out=rec[:, :ia + 1])
        if self.smooth_anchors:
            rec[:, io] = xs[ai]
        if hasattr(motion, "transport_records") and motion._device_transport(xa, ta):
            pos = motion.transport_records(rec, ta, ca, ba)
        else:
            pos = motion.transport(rec.reshape(-1, 2), ta.repeat_interleave(P), ca.repeat_interleave(P),
                                   ba.repeat_interleave(P)).reshape(-1, P, 2)
        img_a = ka * B + ba
        val = gather(img, pos[:, ia], img_a)
        src_a = st["src"][ka, ai].to(val.dtype)
        cnt = per_kb[ka, ba] - src_a
        vis = None
        if self.visibility:
            vis = visible_fraction(motion, xa.detach(), ta, ba, ev, self.tau, counts=counts)
        return _SlicedScore.apply(pos, val, cnt, vis, src_a, (P, ia, io, 0 if self.logdet else -1), self.sigma,
                                  0.5, st["eps"], ev.height, ev.width)

    @staticmethod
    def _events_at_centres(motion, xs, t, b, centres):
        """(Sp, n, 2): every event at every centre.  Trajectories: one kernel, one origin solve per event;
        linear vector fields: each velocity once, x + v (c - t) (the reference's warp); other models: their
        transport of every (event, centre) pair."""
        n, Sp = t.shape[0], centres.shape[0]
        if hasattr(motion, "transport_targets") and motion._device_transport(xs, t):
            return motion.transport_targets(xs, t, centres, b)
        if _fused_kind(motion) >= 0:
            v = motion.velocity(xs, t, b)
            return xs[None] + v[None] * (centres[:, None] - t[None])[..., None]
        return motion.transport(xs.repeat(Sp, 1), t.repeat(Sp), centres.repeat_interleave(n),
                                b.repeat(Sp)).view(Sp, n, 2)

    def set_bandwidth(self, h: float):
        self.sigma = float(h)

    def __call__(self, ev, motion, noise=None):
        ls, _ = self.log_scores(ev, motion, noise=noise)
        s = ls.mean() if ls.numel() else ev.t.new_zeros(())
        return {"loss": -s, "score": s.detach()}


def build(name: str, **kw) -> Objective:
    """Registry of the anchored objectives (atl/objectives/__init__.py:10-35, 'ats_exact' / 'ats_sliced')."""
    reg = {
        "ats_exact": lambda: AnchoredExact(**{k: v for k, v in kw.items() if k in (
            "h", "tau", "eps_frac", "n_anchors", "n_slices", "seed", "smooth_anchors", "dequantize", "visibility",
            "anchor_margin")}),
        "ats_sliced": lambda: AnchoredSliced(**{k: v for k, v in kw.items() if k in (
            "n_slices", "slices_per_step", "sigma", "tau", "eps_frac", "n_anchors_per_slice", "seed")}),
    }
    if name not in reg:
        raise KeyError(f"unknown objective {name}; available: {sorted(reg)}")
    return reg[name]()
