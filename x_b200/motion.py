"""Motion models of stage 1 -- mirror of atl/motion/{base,parametric,trajectories}.py for the models on the path.

``Translation``, ``Affine`` and ``DenseLinearFlow`` evaluate their velocity field (and its gradient
w.r.t. ``theta`` / the flow grid) in libatlb200 kernels that round exactly like the reference's torch
CPU ops, so the pair plan built from the velocities is bit-identical.  ``transport`` in
``mode="linear"`` is x + v(x) (t' - t); ``mode="exact"`` is the closed-form flow of the affine fields
(atlb_flow_exact) or RK4 of the dense grid (atlb_flow_rk4), both kernels.  ``PixelTrajectories``
(atl/motion/trajectories.py) transports, solves origins and evaluates velocities in the trajectory
kernels (atlb_traj_*).  There is no torch or CPU path: positions are data (no gradient), the
parameters are CUDA tensors.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
from torch import nn

from . import _lib as L


def as_time(t_dst, like: torch.Tensor) -> torch.Tensor:
    """Broadcast a scalar or tensor target time to the shape of ``like`` (atl/motion/base.py:57-61)."""
    if torch.is_tensor(t_dst):
        return t_dst.to(like.dtype).expand_as(like) if t_dst.dim() == 0 else t_dst.to(like.dtype)
    return torch.full_like(like, float(t_dst))


class Motion(nn.Module):
    """Base class (atl/motion/base.py:21-54)."""
    linear_at_event: bool = False

    def transport(self, xy, t, t_dst, b):
        raise NotImplementedError

    def velocity(self, xy, t, b):
        raise NotImplementedError(f"{type(self).__name__} has no per-event velocity")

    def transport_logdet(self, xy, t, t_dst, b, delta: float = 0.5):
        """Transport plus log|det d transport / d xy| by central differences (base.py:43-50)."""
        y = self.transport(xy, t, t_dst, b)
        ex = xy.new_tensor([delta, 0.0]); ey = xy.new_tensor([0.0, delta])
        jx = (self.transport(xy + ex, t, t_dst, b) - self.transport(xy - ex, t, t_dst, b)) / (2 * delta)
        jy = (self.transport(xy + ey, t, t_dst, b) - self.transport(xy - ey, t, t_dst, b)) / (2 * delta)
        det = jx[:, 0] * jy[:, 1] - jx[:, 1] * jy[:, 0]
        return y, torch.log(det.abs().clamp(min=1e-12))


class _VelocityFn(torch.autograd.Function):
    """v = field(xy; theta) on the device; gradient w.r.t. theta only (event positions are data)."""

    @staticmethod
    def forward(ctx, theta, xy, b, kind, H, W):
        if xy.requires_grad:
            raise RuntimeError("x_b200 motion fields give no gradient w.r.t. event positions")
        if not theta.is_cuda:
            raise RuntimeError("x_b200 motion models need CUDA parameters (there is no CPU path)")
        th = theta.detach().float().contiguous()
        xyc = xy.detach().float().contiguous()
        bl = b.contiguous().long()
        B = th.shape[0]
        Hg, Wg = (th.shape[-2], th.shape[-1]) if kind == L.MOTION_DENSE else (1, 1)
        v = torch.empty(xyc.shape[0], 2, dtype=torch.float32, device=xyc.device)
        L.check(L.lib().atlb_velocity(kind, L.ptr(th), B, Hg, Wg, H, W, L.ptr(xyc), L.ptr(bl), xyc.shape[0], L.ptr(v),
                                      L.stream()), "velocity")
        ctx.save_for_backward(xyc, bl)
        ctx.meta = (kind, tuple(th.shape), B, Hg, Wg, H, W, theta.dtype)
        return v

    @staticmethod
    def backward(ctx, gv):
        xyc, bl = ctx.saved_tensors
        kind, shape, B, Hg, Wg, H, W, dtype = ctx.meta
        g = torch.empty(shape, dtype=torch.float32, device=xyc.device)
        L.check(L.lib().atlb_velocity_bwd(kind, L.ptr(gv.contiguous().float()), B, Hg, Wg, H, W, L.ptr(xyc), L.ptr(bl),
                                          xyc.shape[0], L.ptr(g), L.stream()), "velocity_bwd")
        return g.to(dtype), None, None, None, None, None


class _FlowExactFn(torch.autograd.Function):
    """Exact flow of an affine field on the device (atlb_flow_exact / _bwd), differentiable w.r.t. theta and the
    positions."""

    @staticmethod
    def forward(ctx, theta, xy, t, t_dst, b, kind, H, W):
        th = theta.detach().float().contiguous()
        xyc, tc, bl = xy.detach().float().contiguous(), t.detach().float().contiguous(), b.contiguous().long()
        if torch.is_tensor(t_dst) and t_dst.dim() > 0:
            td, tds = t_dst.detach().float().contiguous().expand_as(tc).contiguous(), 0.0
        else:
            td, tds = None, float(t_dst)
        out = torch.empty_like(xyc)
        L.check(L.lib().atlb_flow_exact(kind, L.ptr(th), th.shape[0], H, W, L.ptr(xyc), L.ptr(tc), L.ptr(td), tds,
                                        L.ptr(bl), tc.shape[0], L.ptr(out), L.stream()), "flow_exact")
        ctx.save_for_backward(th, xyc, tc, bl, td if td is not None else tc.new_empty(0))
        ctx.meta = (kind, H, W, tds, td is not None, theta.dtype, xy.dtype)
        return out.to(xy.dtype)

    @staticmethod
    def backward(ctx, gy):
        th, xyc, tc, bl, td = ctx.saved_tensors
        kind, H, W, tds, per_event, tdt, xdt = ctx.meta
        gth = torch.empty_like(th)
        gxy = torch.empty_like(xyc) if ctx.needs_input_grad[1] else None
        L.check(L.lib().atlb_flow_exact_bwd(kind, L.ptr(gy.contiguous().float()), L.ptr(th), th.shape[0], H, W,
                                            L.ptr(xyc), L.ptr(tc), L.ptr(td if per_event else None), tds, L.ptr(bl),
                                            tc.shape[0], L.ptr(gth), L.ptr(gxy), L.stream()), "flow_exact_bwd")
        return gth.to(tdt), (None if gxy is None else gxy.to(xdt)), None, None, None, None, None, None


class _FlowRK4Fn(torch.autograd.Function):
    """RK4 transport of the dense velocity grid on the device (atlb_flow_rk4 / _bwd), differentiable w.r.t. the
    grid (positions are data)."""

    @staticmethod
    def forward(ctx, grid, xy, t, t_dst, b, H, W, steps):
        g = grid.detach().float().contiguous()
        xyc, tc, bl = xy.detach().float().contiguous(), t.detach().float().contiguous(), b.contiguous().long()
        if torch.is_tensor(t_dst) and t_dst.dim() > 0:
            td, tds = t_dst.detach().float().contiguous().expand_as(tc).contiguous(), 0.0
        else:
            td, tds = None, float(t_dst)
        B, _, Hg, Wg = g.shape
        out = torch.empty_like(xyc)
        L.check(L.lib().atlb_flow_rk4(L.ptr(g), B, Hg, Wg, H, W, L.ptr(xyc), L.ptr(tc), L.ptr(td), tds, L.ptr(bl),
                                      tc.shape[0], int(steps), L.ptr(out), L.stream()), "flow_rk4")
        ctx.save_for_backward(g, xyc, tc, bl, td if td is not None else tc.new_empty(0))
        ctx.meta = (H, W, tds, td is not None, int(steps), grid.dtype, xy.dtype)
        return out.to(xy.dtype)

    @staticmethod
    def backward(ctx, gy):
        g, xyc, tc, bl, td = ctx.saved_tensors
        H, W, tds, per_event, steps, gdt, _ = ctx.meta
        B, _, Hg, Wg = g.shape
        gg = torch.empty_like(g)
        L.check(L.lib().atlb_flow_rk4_bwd(L.ptr(gy.contiguous().float()), L.ptr(g), B, Hg, Wg, H, W, L.ptr(xyc),
                                          L.ptr(tc), L.ptr(td if per_event else None), tds, L.ptr(bl), tc.shape[0],
                                          steps, L.ptr(gg), L.stream()), "flow_rk4_bwd")
        return gg.to(gdt), None, None, None, None, None, None, None


class VectorFieldMotion(Motion):
    """Autonomous velocity field v(x; theta) (parametric.py:84-145)."""
    n_params: int = 0
    kind: int = -1

    @property
    def linear_at_event(self) -> bool:
        return self.mode == "linear"

    def __init__(self, batch_size: int, height: int, width: int, mode: str = "linear", rk4_steps: int = 8,
                 init: Optional[torch.Tensor] = None):
        super().__init__()
        self.H, self.W, self.mode, self.rk4_steps = height, width, mode, rk4_steps
        self.c = torch.tensor([(width - 1) / 2.0, (height - 1) / 2.0])
        theta = torch.zeros(batch_size, self.n_params) if init is None else init.clone().float()
        self.theta = nn.Parameter(theta)

    def field(self, xy: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        return _VelocityFn.apply(self.theta, xy, b, self.kind, self.H, self.W)

    def velocity(self, xy, t, b):
        return self.field(xy, b)

    def affine_parts(self, b):
        return None

    def transport(self, xy, t, t_dst, b):
        """Where the scene point of event (xy, t) is at t_dst (atl/motion/parametric.py:53-78).  mode="linear": the
        warp x + v(x) (t_dst - t).  mode="exact": the flow of the field -- in closed form on the device for the
        affine fields (the augmented matrix exponential, atlb_flow_exact), by classic fourth-order Runge-Kutta
        stages of the field otherwise (rk4_steps steps)."""
        if self.mode == "linear":
            dt = as_time(t_dst, t) - t
            return xy + self.field(xy, b) * dt[:, None]
        if self.kind in (L.MOTION_TRANSLATION, L.MOTION_AFFINE):
            return _FlowExactFn.apply(self.theta, xy, t, t_dst, b, self.kind, self.H, self.W)
        return _FlowRK4Fn.apply(self.theta, xy, t, t_dst, b, self.H, self.W, self.rk4_steps)


class Translation(VectorFieldMotion):
    """v = (tx, ty) (parametric.py:148-157)."""
    n_params = 2
    kind = L.MOTION_TRANSLATION

    def affine_parts(self, b):
        z = self.theta.new_zeros(b.numel(), 2, 2)
        return z, self.theta[b]


class Affine(VectorFieldMotion):
    """v = A (x - c) + t, theta = (tx, ty, a11, a12, a21, a22) (parametric.py:207-217)."""
    n_params = 6
    kind = L.MOTION_AFFINE

    def affine_parts(self, b):
        th = self.theta[b]
        return th[:, 2:6].view(-1, 2, 2), th[:, :2]



class DenseLinearFlow(VectorFieldMotion):
    """Dense velocity grid (B, 2, Hg, Wg) bilinearly interpolated over the image (parametric.py:257-293)."""
    kind = L.MOTION_DENSE

    def __init__(self, batch_size, height, width, grid=(1, 1), mode="linear", init=None, rk4_steps=4):
        Motion.__init__(self)
        self.H, self.W, self.mode, self.rk4_steps = height, width, mode, rk4_steps
        self.c = torch.tensor([(width - 1) / 2.0, (height - 1) / 2.0])
        g = torch.zeros(batch_size, 2, *grid) if init is None else init.clone().float()
        self.grid = nn.Parameter(g)

    @property
    def theta(self):
        return self.grid


    def upsample(self, factor: int = 2):
        """Refine the velocity grid by ``factor`` (parametric.py:282-289)."""
        with torch.no_grad():
            Hg, Wg = self.grid.shape[-2:]
            new = torch.nn.functional.interpolate(self.grid, size=(Hg * factor, Wg * factor), mode="bilinear",
                                                  align_corners=True)
        self.grid = nn.Parameter(new)
        return self


class _TrajTransport(torch.autograd.Function):
    """PixelTrajectories transport on the device (atlb_traj_transport), differentiable w.r.t. the tile
    coefficients.  mode 0: xy -> transport to t_dst; 1: xy -> trajectory origin; 2: xy are origins ->
    position at t_dst (also differentiable w.r.t. those origins); 3: xy -> velocity of the degree-1
    trajectories.  Event positions and times are data."""

    @staticmethod
    def forward(ctx, tile_c, xy, t, t_dst, b, model, mode):
        C = tile_c.detach().float().permute(0, 2, 3, 1).contiguous()
        xyc, tc, bc = xy.detach().float().contiguous(), t.detach().float().contiguous(), b.contiguous().long()
        if torch.is_tensor(t_dst) and t_dst.dim() > 0:
            tdc, tds = t_dst.detach().float().contiguous(), 0.0
        else:
            tdc, tds = None, float(t_dst)
        out = torch.empty_like(xyc)
        B, Hq, Wq, C2 = C.shape
        L.check(L.lib().atlb_traj_transport(mode, L.ptr(C), B, Hq, Wq, C2 // 2, model._basis_id, L.ptr(model._bc),
                                            model.offset, float(model.tile), model.n_fp, L.ptr(xyc), L.ptr(tc),
                                            L.ptr(tdc), tds, L.ptr(bc), xyc.shape[0], L.ptr(out), L.stream()),
                "traj_transport")
        ctx.save_for_backward(C, xyc, tc, bc, *(() if tdc is None else (tdc,)))
        ctx.tds, ctx.model, ctx.mode = tds, model, mode
        return out

    @staticmethod
    def backward(ctx, gy):
        C, xyc, tc, bc, *rest = ctx.saved_tensors
        tdc = rest[0] if rest else None
        m, mode = ctx.model, ctx.mode
        gC = torch.zeros_like(C)
        gp = torch.empty_like(xyc) if mode == 2 else None
        B, Hq, Wq, C2 = C.shape
        L.check(L.lib().atlb_traj_transport_bwd(mode, L.ptr(gy.contiguous().float()), L.ptr(C), B, Hq, Wq, C2 // 2,
                                                m._basis_id, L.ptr(m._bc), m.offset, float(m.tile), m.n_fp,
                                                L.ptr(xyc), L.ptr(tc), L.ptr(tdc), ctx.tds, L.ptr(bc), xyc.shape[0],
                                                L.ptr(gC), L.ptr(gp), L.stream()), "traj_transport_bwd")
        return gC.permute(0, 3, 1, 2), gp, None, None, None, None, None


def _traj_args(model):
    """(coefficients channels-last, the leading C-ABI arguments) of a PixelTrajectories model."""
    C = model.tile_c.detach().float().permute(0, 2, 3, 1).contiguous()
    B, Hq, Wq, C2 = C.shape
    return C, (L.ptr(C), B, Hq, Wq, C2 // 2, model._basis_id, L.ptr(model._bc), model.offset, float(model.tile),
               model.n_fp)


class _TrajRecords(torch.autograd.Function):
    """R positions per event (xy (N, R, 2), at the event's time) moved to one target time per event
    (atlb_traj_records), differentiable w.r.t. the tile coefficients; each record as mode 0 moves it."""

    @staticmethod
    def forward(ctx, tile_c, xy, t, t_dst, b, model):
        C, head = _traj_args(model)
        xyc, tc, bc = xy.detach().float().contiguous(), t.detach().float().contiguous(), b.contiguous().long()
        if torch.is_tensor(t_dst) and t_dst.dim() > 0:
            tdc, tds = t_dst.detach().float().contiguous(), 0.0
        else:
            tdc, tds = None, float(t_dst)
        N, R = xyc.shape[0], xyc.shape[1]
        out = torch.empty_like(xyc)
        # the fixed-point iterates are kept for the backward when it will run (n_fp x 8 bytes per record)
        its = torch.empty(model.n_fp, N, R, 2, dtype=torch.float32, device=xyc.device) \
            if ctx.needs_input_grad[0] and model.n_fp > 0 else None
        L.check(L.lib().atlb_traj_records(*head, L.ptr(xyc), R, L.ptr(tc), L.ptr(tdc), tds, L.ptr(bc), N, L.ptr(out),
                                          L.ptr(its), L.stream()), "traj_records")
        ctx.save_for_backward(C, xyc, tc, bc, *(() if tdc is None else (tdc,)))
        ctx.tds, ctx.model, ctx.its = tds, model, its
        return out

    @staticmethod
    def backward(ctx, gy):
        C, xyc, tc, bc, *rest = ctx.saved_tensors
        tdc = rest[0] if rest else None
        _, head = _traj_args(ctx.model)
        gC = torch.zeros_like(C)
        N, R = xyc.shape[0], xyc.shape[1]
        L.check(L.lib().atlb_traj_records_bwd(L.ptr(gy.contiguous().float()), *head, L.ptr(xyc), R, L.ptr(tc),
                                              L.ptr(tdc), ctx.tds, L.ptr(bc), N, L.ptr(ctx.its), L.ptr(gC),
                                              L.stream()), "traj_records_bwd")
        ctx.its = None
        return gC.permute(0, 3, 1, 2), None, None, None, None, None


class _TrajTargets(torch.autograd.Function):
    """Every event moved to each of T target times (atlb_traj_targets): (T, N, 2), differentiable w.r.t. the
    tile coefficients; entry (j, n) as mode 0 moves event n to targets[j]."""

    @staticmethod
    def forward(ctx, tile_c, xy, t, targets, b, model):
        C, head = _traj_args(model)
        xyc, tc, bc = xy.detach().float().contiguous(), t.detach().float().contiguous(), b.contiguous().long()
        tg = targets.detach().float().contiguous()
        N, T = xyc.shape[0], tg.shape[0]
        out = torch.empty(T, N, 2, dtype=torch.float32, device=xyc.device)
        L.check(L.lib().atlb_traj_targets(*head, L.ptr(xyc), L.ptr(tc), L.ptr(bc), N, L.ptr(tg), T, L.ptr(out),
                                          L.stream()), "traj_targets")
        ctx.save_for_backward(C, xyc, tc, bc, tg)
        ctx.model = model
        return out

    @staticmethod
    def backward(ctx, gy):
        C, xyc, tc, bc, tg = ctx.saved_tensors
        _, head = _traj_args(ctx.model)
        gC = torch.zeros_like(C)
        L.check(L.lib().atlb_traj_targets_bwd(L.ptr(gy.contiguous().float()), *head, L.ptr(xyc), L.ptr(tc),
                                              L.ptr(bc), xyc.shape[0], L.ptr(tg), tg.shape[0], L.ptr(gC), L.stream()),
                "traj_targets_bwd")
        return gC.permute(0, 3, 1, 2), None, None, None, None, None


class PixelTrajectories(Motion):
    """One continuous-time trajectory per ``tile`` x ``tile`` patch, coefficients from a (B, 2K, H, W) grid
    (atl/motion/trajectories.py:40-120): q(p, t) = p + sum_k c_k(p) g_k(t), channels [y_1..y_K, x_1..x_K].
    Transport inverts q(p, t) = x by fixed-point iteration, then evaluates q(p, t')."""

    def __init__(self, coeff_grid: torch.Tensor, K: int, basis_kind: str = "polynomial", tile: int = 4,
                 assign: str = "invert", n_fixed_point: int = 6):
        super().__init__()
        self.coeff_grid = coeff_grid
        self.K, self.basis_kind, self.tile, self.assign, self.n_fp = K, basis_kind, tile, assign, n_fixed_point
        B, C, H, W = coeff_grid.shape
        assert C == 2 * K
        self.B, self.H, self.W = B, H, W
        s = tile // 2
        self.tile_c = coeff_grid[:, :, s::tile, s::tile]
        self.Hq, self.Wq = self.tile_c.shape[-2:]
        self.offset = float(s)
        self.linear_at_event = (K == 1 and basis_kind == "polynomial")
        # Bezier binomial factors as the reference evaluates them (fp32 torch on the host), for the kernels
        k = torch.arange(1, K + 1, dtype=torch.float32)
        self._bc = torch.exp(math.lgamma(K + 1) - torch.lgamma(k + 1) - torch.lgamma(K - k + 1)).contiguous()
        self._basis_id = {"polynomial": 0, "bezier": 1}.get(basis_kind, -1)

    def transport(self, xy, t, t_dst, b):
        self._require_device(xy, t)
        return _TrajTransport.apply(self.tile_c, xy, t, t_dst, b, self, 0)

    def origin_on_device(self, xy, t, b):
        """The trajectory origins of events (xy, t) (the fixed point of :meth:`origin`), on the device."""
        return _TrajTransport.apply(self.tile_c, xy, t, 0.0, b, self, 1)

    def from_origin(self, p, t, t_dst, b):
        """Positions at t_dst of the trajectories starting at origins p: with p = :meth:`origin_on_device`,
        exactly :meth:`transport`; differentiable w.r.t. p (a caller moving the same events to several
        times solves each origin once)."""
        return _TrajTransport.apply(self.tile_c, p, t, t_dst, b, self, 2)

    def transport_records(self, xy, t, t_dst, b):
        """xy (N, R, 2): R positions per event at its time t, each moved to t_dst (scalar or per event) as
        :meth:`transport` moves it, in one kernel (the anchor and its log-determinant probes)."""
        return _TrajRecords.apply(self.tile_c, xy, t, t_dst, b, self)

    def transport_targets(self, xy, t, targets, b):
        """(T, N, 2): every event moved to each of the T times ``targets`` as :meth:`transport` moves it; one
        origin solve per event (the sources at every slice centre)."""
        return _TrajTargets.apply(self.tile_c, xy, t, targets, b, self)

    def _device_transport(self, xy, t) -> bool:
        """The kernels cover the invert assignment, K <= 16 and n_fp <= 16, for positions without gradient."""
        return (self.tile_c.is_cuda and xy.is_cuda and self.assign == "invert" and self._basis_id >= 0
                and self.K <= 16 and self.n_fp <= 16 and not xy.requires_grad and not t.requires_grad)

    def _require_device(self, xy, t):
        if not self._device_transport(xy, t):
            raise NotImplementedError(
                "x_b200 PixelTrajectories: the trajectory kernels need CUDA tensors, assign='invert', a polynomial or "
                "Bezier basis, K <= 16, n_fixed_point <= 16 and positions without gradient (there is no torch path)")

    def velocity(self, xy, t, b):
        """v = c_1 sampled at the trajectory origin of (xy, t) (trajectories.py:79-83), for the degree-1
        polynomial trajectories (the only ones linear at the event), in the trajectory kernel's mode 3."""
        if not self.linear_at_event:
            raise NotImplementedError("per-event velocity only for the degree-1 polynomial prior")
        self._require_device(xy, t)
        return _TrajTransport.apply(self.tile_c, xy, t, 0.0, b, self, 3)

    @torch.no_grad()
    def visible_fraction(self, xa, ta, ba, counts, centres, tau, H, W):
        """The exposure correction of the anchors (atl/objectives/ats.py:31-50) in one kernel
        (atlb_traj_visible_fraction): counts (B, n_check) slice counts, centres (n_check) slice centres."""
        C = self.tile_c.detach().float().permute(0, 2, 3, 1).contiguous()
        xac, tac, bac = xa.detach().float().contiguous(), ta.detach().float().contiguous(), ba.contiguous().long()
        out = torch.empty(tac.shape[0], dtype=torch.float32, device=xa.device)
        B, Hq, Wq, C2 = C.shape
        L.check(L.lib().atlb_traj_visible_fraction(L.ptr(C), B, Hq, Wq, C2 // 2, self._basis_id, L.ptr(self._bc),
                                                   self.offset, float(self.tile), self.n_fp, L.ptr(xac), L.ptr(tac),
                                                   L.ptr(bac), tac.shape[0], L.ptr(counts.float()), L.ptr(centres),
                                                   centres.shape[0], float(tau), H, W, L.ptr(out), L.stream()),
                "traj_visible_fraction")
        return out.to(ta.dtype)

    def regulariser_fields(self, B, H, W):
        return self.tile_c


MODELS = {"translation": Translation, "affine": Affine, "dense": DenseLinearFlow}
