"""Plain torch (fp32) statements of two motion transports, used as checkers of the trajectory and RK4
kernels in the GPU tests (test infrastructure; the library itself has no torch path):

* ``trajectory_transport``: the PixelTrajectories model of atl/motion/trajectories.py:40-83 -- per-tile
  trajectory coefficients (the coefficient grid sampled at tile centres), sampled bilinearly with a border
  clamp at (p - offset) / tile; the origin of (x, t) is the fixed point of p = x - d(p, t); the position at
  t' is p + d(p, t');
* ``dense_rk4``: the RK4 transport of a dense velocity grid of atl/motion/parametric.py:72-80.
Both are differentiable w.r.t. their parameters by torch autograd.
"""
from __future__ import annotations

import math

import torch


def _bilinear_clamped(field: torch.Tensor, u: torch.Tensor, v: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """field (B, C, Hn, Wn) sampled at continuous grid coordinates (u along W, v along H), border clamp:
    (n, C).  Corner indices from the clamped coordinate, the last cell reused at the far border."""
    Bn, C, Hn, Wn = field.shape
    u = torch.clamp(u, 0, Wn - 1)
    v = torch.clamp(v, 0, Hn - 1)
    i0 = torch.clamp(torch.floor(u), max=max(Wn - 2, 0))
    j0 = torch.clamp(torch.floor(v), max=max(Hn - 2, 0))
    fu, fv = u - i0, v - j0
    i0, j0 = i0.long(), j0.long()
    i1, j1 = torch.clamp(i0 + 1, max=Wn - 1), torch.clamp(j0 + 1, max=Hn - 1)
    flat = field.permute(0, 2, 3, 1).reshape(Bn * Hn * Wn, C)
    row = b * Hn
    corner = lambda j, i: flat[(row + j) * Wn + i]  # noqa: E731
    return (corner(j0, i0) * ((1 - fu) * (1 - fv))[:, None] + corner(j0, i1) * (fu * (1 - fv))[:, None]
            + corner(j1, i0) * ((1 - fu) * fv)[:, None] + corner(j1, i1) * (fu * fv)[:, None])


def trajectory_basis(t: torch.Tensor, K: int, kind: str) -> torch.Tensor:
    """(n, K): t^k (polynomial) or the Bernstein polynomials C(K, k) t^k (1 - t)^(K - k) (Bezier), k = 1..K."""
    k = torch.arange(1, K + 1, device=t.device, dtype=t.dtype)
    tt = t[:, None]
    if kind == "polynomial":
        return tt ** k
    binom = torch.tensor([math.comb(K, int(j)) for j in range(1, K + 1)], device=t.device, dtype=t.dtype)
    return binom * tt ** k * (1 - tt) ** (K - k)


def trajectory_transport(coeff: torch.Tensor, K: int, kind: str, tile: int, n_fp: int, xy: torch.Tensor,
                         t: torch.Tensor, t_dst: torch.Tensor, b: torch.Tensor, velocity: bool = False):
    """Positions at t_dst of the events (xy, t) under the trajectories of ``coeff`` (B, 2K, H, W), channels
    [y_1..y_K, x_1..x_K]; ``velocity``: instead, (c_x1, c_y1) at the origin."""
    s = tile // 2
    tc = coeff[:, :, s::tile, s::tile]

    def coeffs(p):  # (n, K, 2) as (x, y)
        c = _bilinear_clamped(tc, (p[:, 0] - s) / tile, (p[:, 1] - s) / tile, b)
        return torch.stack([c[:, K:], c[:, :K]], -1)

    def disp(p, tt):
        return (coeffs(p) * trajectory_basis(tt, K, kind)[..., None]).sum(1)

    p = xy
    for _ in range(n_fp):
        p = xy - disp(p, t)
    if velocity:
        return coeffs(p)[:, 0]
    return p + disp(p, t_dst)


def dense_rk4(grid: torch.Tensor, H: int, W: int, xy: torch.Tensor, t: torch.Tensor, t_dst: torch.Tensor,
              b: torch.Tensor, steps: int) -> torch.Tensor:
    """RK4 (classic weights) of dx/ds = v(x) over t_dst - t, v the grid (B, 2, Hg, Wg) sampled at
    x / (W - 1) (Wg - 1), y / (H - 1) (Hg - 1)."""
    Hg, Wg = grid.shape[-2:]

    def v(p):
        return _bilinear_clamped(grid, p[:, 0] / max(W - 1, 1) * (Wg - 1), p[:, 1] / max(H - 1, 1) * (Hg - 1), b)

    h = ((t_dst - t) / steps)[:, None]
    x = xy
    for _ in range(steps):
        k1 = v(x)
        k2 = v(x + 0.5 * h * k1)
        k3 = v(x + 0.5 * h * k2)
        k4 = v(x + h * k3)
        x = x + h * (k1 + 2 * k2 + 2 * k3 + k4) / 6
    return x
