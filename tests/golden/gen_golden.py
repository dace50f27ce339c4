"""Generate the golden fixtures under tests/golden/ by running the REFERENCE implementation.

    python tests/golden/gen_golden.py          # needs the reference tree (build container only)

The reference (KAVYANSHTYAGI/x, package ``atl``) is loaded by ``oracle/refload.py``: its unmodified
Python package plus its OpenMP extension csrc/atl_cpu.cpp compiled by ``oracle/Makefile``.  Every
fixture stores the seeded inputs and the reference's outputs; tests/test_oracle_golden.py pins the
C oracle against them and the GPU tests compare the CUDA library against both.

Inputs are seeded synthetic events (no dataset items).  Sizes are kept small so the fixtures stay a
few hundred KB in total.
"""
from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
from oracle.refload import load_reference  # noqa: E402

atl = load_reference()
from atl.motion import Affine, DenseLinearFlow, PixelTrajectories, Translation  # noqa: E402
from atl.objectives import ats as ATS  # noqa: E402
from atl.ops import functional as F  # noqa: E402
from atl.core.events import EventPacket  # noqa: E402

torch.set_num_threads(8)


def rand_events(n=500, B=2, H=20, W=24, seed=0):
    """Same construction as the reference's tests/test_ops.py:16-23 (positions spill 2 px outside)."""
    g = torch.Generator().manual_seed(seed)
    pos = torch.stack([torch.rand(n, generator=g) * (W + 4) - 2, torch.rand(n, generator=g) * (H + 4) - 2], 1)
    w = torch.rand(n, generator=g) + 0.1
    b = torch.randint(0, B, (n,), generator=g)
    t = torch.rand(n, generator=g)
    order = torch.argsort(b.double() * 4 + t.double())
    return pos[order], w[order], b[order], t[order]


def save(name, **arrs):
    out = {}
    for k, v in arrs.items():
        if torch.is_tensor(v):
            v = v.detach().cpu().numpy()
        out[k] = np.asarray(v)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"{name}: " + ", ".join(f"{k}{tuple(v.shape)}" for k, v in out.items()))


def gen_ops():
    pos, w, b, t = rand_events(500, seed=0)
    B, H, W = 2, 20, 24
    # pin the lround tie-breaking (half away from zero) with exact .5 positions
    pos[:8, 0] = torch.tensor([2.5, 3.5, -0.5, 10.5, 7.5, 0.5, 22.5, 5.5])
    pos[:8, 1] = torch.tensor([4.5, 1.5, 6.5, -0.5, 18.5, 9.5, 3.5, 12.5])
    E = atl.ops.get_ext()
    g = torch.Generator().manual_seed(11)
    gimg = torch.randn(B, H, W, generator=g)
    img = torch.randn(B, H, W, generator=g)
    gval = torch.randn(pos.shape[0], generator=g)
    sigma, R = 1.3, int(math.ceil(3 * 1.3))
    sb = E.splat_bilinear_fwd(pos, w, b, B, H, W)
    sb_gp, sb_gw = E.splat_bilinear_bwd(gimg, pos, w, b)
    sg = E.splat_gauss_fwd(pos, w, b, B, H, W, sigma, R)
    sg_gp, sg_gw = E.splat_gauss_bwd(gimg, pos, w, b, sigma, R)
    ga = E.gather_bilinear_fwd(img, pos, b)
    ga_gi, ga_gp = E.gather_bilinear_bwd(gval, img, pos, b)
    p = torch.where(torch.rand(pos.shape[0], generator=g) > 0.5, 1.0, -1.0)
    vox = E.voxel_grid(pos, t, p, b, B, 5, H, W)
    save("ops", pos=pos, w=w, b=b, t=t, p=p, gimg=gimg, img=img, gval=gval, sigma=sigma, R=R,
         splat_bilinear=sb, splat_bilinear_gpos=sb_gp, splat_bilinear_gw=sb_gw,
         splat_gauss=sg, splat_gauss_gpos=sg_gp, splat_gauss_gw=sg_gw,
         gather=ga, gather_gimg=ga_gi, gather_gpos=ga_gp, voxel=vox)


def gen_plan(name, n, B, H, W, seed, vscale, tau, S, h, anchor_step=3, smooth=False):
    pos, _, b, t = rand_events(n, B=B, H=H, W=W, seed=seed)
    g = torch.Generator().manual_seed(seed + 100)
    v = torch.randn(n, 2, generator=g) * vscale
    anchors = torch.arange(0, n, anchor_step)
    axy = pos[anchors] + h * torch.randn(anchors.numel(), 2, generator=g) if smooth else None
    plan = F.build_pair_plan(pos, t, v, b, B, H, W, anchors, h, tau, 3.0, S, anchor_xy=axy)
    E = atl.ops.get_ext()
    args = (plan.src_y, plan.src_v, plan.src_t, plan.src_id, plan.cell_start, plan.anc_x, plan.anc_t, plan.anc_cell,
            plan.anc_id, plan.slice_c, plan.S, plan.GH, plan.GW, float(h), float(tau), 3.0)
    Sv = E.ats_pair_fwd(*args)
    gS = torch.randn(anchors.numel(), generator=g)
    gv = E.ats_pair_bwd(gS, *args, n)
    brute = atl.ops.reference.ats_pair_sums(pos, t, v, b, anchors, h, tau, 3.0, anchor_xy=axy)
    save(name, pos=pos, b=b, t=t, v=v, anchors=anchors, anchor_xy=(axy if axy is not None else np.zeros((0, 2))),
         B=B, H=H, W=W, h=h, tau=tau, S=S, GH=plan.GH, GW=plan.GW,
         src_y=plan.src_y, src_v=plan.src_v, src_t=plan.src_t, src_id=plan.src_id, cell_start=plan.cell_start,
         anc_x=plan.anc_x, anc_t=plan.anc_t, anc_cell=plan.anc_cell, anc_id=plan.anc_id, slice_c=plan.slice_c,
         pair_S=Sv, gS=gS, pair_gv=gv, brute_S=brute)


def gen_window():
    t = torch.tensor([0.0, 0.1, 0.2, 0.9, 0.0, 0.5])
    b = torch.tensor([0, 0, 0, 0, 1, 1])
    kat = F.window_counts(t, b, torch.arange(6), 0.15)
    _, _, b2, t2 = rand_events(3000, B=3, seed=5)
    idx = torch.arange(0, 3000, 7)
    r = {f"tau{k}": F.window_counts(t2, b2, idx, tau) for k, tau in enumerate((0.05, 0.2, 1.0))}
    # unsorted input with ties (the reference sorts the keys itself)
    g = torch.Generator().manual_seed(9)
    t3 = torch.round(torch.rand(800, generator=g) * 50) / 50
    b3 = torch.randint(0, 2, (800,), generator=g)
    idx3 = torch.randperm(800, generator=g)[:300]
    r3 = F.window_counts(t3, b3, idx3, 0.1)
    save("window", kat_t=t, kat_b=b, kat=kat, t=t2, b=b2, idx=idx, taus=np.array([0.05, 0.2, 1.0]),
         unsorted_t=t3, unsorted_b=b3, unsorted_idx=idx3, unsorted=r3, **r)


def _motion(kind, B, H, W, seed):
    g = torch.Generator().manual_seed(seed)
    if kind == "translation":
        th = (torch.rand(B, 2, generator=g) - 0.5) * 40
        return Translation(B, H, W, mode="linear", init=th), th
    if kind == "affine":
        th = torch.cat([(torch.rand(B, 2, generator=g) - 0.5) * 40, (torch.rand(B, 4, generator=g) - 0.5) * 0.1], 1)
        return Affine(B, H, W, mode="linear", init=th), th
    grid = torch.randn(B, 2, H, W, generator=g)
    grid = torch.nn.functional.avg_pool2d(grid, 7, 1, 3) * 40
    return DenseLinearFlow(B, H, W, grid=(H, W), mode="linear", init=grid), grid


def gen_motion():
    B, H, W = 2, 48, 64
    g = torch.Generator().manual_seed(21)
    n = 4000
    xy = torch.stack([torch.rand(n, generator=g) * (W + 10) - 5, torch.rand(n, generator=g) * (H + 10) - 5], 1)
    # exact grid nodes and borders
    xy[:6] = torch.tensor([[0.0, 0.0], [W - 1.0, H - 1.0], [W - 1.0, 0.0], [31.0, 17.0], [-3.0, 50.0], [70.0, -2.0]])
    b = torch.randint(0, B, (n,), generator=g)
    t = torch.sort(torch.rand(n, generator=g)).values
    order = torch.argsort(b.double() * 4 + t.double())
    xy, b, t = xy[order], b[order], t[order]
    out = {}
    for k, kind in enumerate(("translation", "affine", "dense")):
        m, th = _motion(kind, B, H, W, 30 + k)
        ev = EventPacket(xy, t, torch.ones(n), b, B, H, W)
        v = m.velocity(xy, t, b).detach()
        ia = torch.arange(0, n, 5)
        vis = ATS.visible_fraction(m, xy[ia], t[ia], b[ia], ev, 0.3)
        vis1 = ATS.visible_fraction(m, xy[ia], t[ia], b[ia], ev, 1.0)
        out.update({f"{kind}_theta": th, f"{kind}_v": v, f"{kind}_vis_tau03": vis, f"{kind}_vis_tau1": vis1})
    save("motion", xy=xy, b=b, t=t, B=B, H=H, W=W, vis_idx=torch.arange(0, n, 5), **out)


def synth_window(n, H, W, seed, B=1):
    """Seeded synthetic window: integer pixel coordinates, uniform times (normalised), +-1 polarity."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(0, W, (n,), generator=g).float()
    y = torch.randint(0, H, (n,), generator=g).float()
    t = torch.sort(torch.rand(n, generator=g)).values
    b = torch.sort(torch.randint(0, B, (n,), generator=g)).values
    order = torch.argsort(b.double() * 4 + t.double())
    return torch.stack([x, y], 1)[order], t[order], b[order]


def gen_exact(kind, n, B, H, W, seed, n_anchors, h=1.0, tau=1.0, S=16, visibility=True):
    xy, t, b = synth_window(n, H, W, seed, B)
    ev = EventPacket(xy, t, torch.ones(n), b, B, H, W)
    m, th = _motion(kind, B, H, W, seed + 1)
    obj = ATS.AnchoredExact(h=h, tau=tau, n_anchors=n_anchors, n_slices=S, seed=seed + 2, visibility=visibility)
    # replay the objective's generator to record the noise it draws (ats.py:53-57, 84-88)
    gen = torch.Generator().manual_seed(seed + 2)
    if n_anchors is None or n_anchors >= n:
        anchors = torch.arange(n)
    else:
        anchors = torch.sort(torch.randperm(n, generator=gen)[:n_anchors]).values
    u = torch.rand(xy.shape, generator=gen)
    z = torch.randn((anchors.numel(), 2), generator=gen)
    out = obj(ev, m)
    out["loss"].backward()
    xs = xy + (u - 0.5)
    xa = xs[anchors] + h * z
    v = m.velocity(xs, t, b).detach()
    Sv = F.ats_pair_sums(xs, t, v, b, B, H, W, anchors, h, tau, 3.0, S, anchor_xy=xa)
    Wn = F.window_counts(t, b, anchors, tau).clamp(min=1)
    vis = ATS.visible_fraction(m, xa, t[anchors], b[anchors], ev, tau) if visibility else torch.ones(anchors.numel())
    # per-anchor log scores of a second objective instance with the same seed
    obj2 = ATS.AnchoredExact(h=h, tau=tau, n_anchors=n_anchors, n_slices=S, seed=seed + 2, visibility=visibility)
    ls, anc2 = obj2.log_scores(ev, m)
    assert torch.equal(anc2, anchors)
    save(f"exact_{kind}", kind=kind, xy=xy, t=t, b=b, B=B, H=H, W=W, h=h, tau=tau, S=S, visibility=visibility,
         theta=th, anchors=anchors, u=u, z=z, xs=xs, xa=xa, v=v, pair_S=Sv, Wn=Wn, vis=vis, ls=ls.detach(),
         loss=out["loss"].detach(), grad_theta=m.theta.grad)


def gen_sliced(name, kind, n, B, H, W, seed, S, sigma, K=3, masks=False, **obj_kw):
    """AnchoredSliced (ats.py:108-183) on a seeded window: per-anchor log scores, loss and the gradient of
    the loss w.r.t. the motion parameters (a PixelTrajectories coefficient grid, or theta / flow grid).
    ``obj_kw``: further constructor options (slices_per_step, n_anchors_per_slice, tau, smooth_anchors,
    dequantize, logdet, visibility); ``masks``: seeded held-out anchor / source masks (the split of
    heldout_score, ats.py:204-213)."""
    xy, t, b = synth_window(n, H, W, seed, B)
    ev = EventPacket(xy, t, torch.ones(n), b, B, H, W)
    g = torch.Generator().manual_seed(seed + 1)
    if kind == "trajectories":
        coeff = torch.nn.functional.avg_pool2d(torch.randn(B, 2 * K, H, W, generator=g), 9, 1, 4) * 12
        coeff.requires_grad_(True)
        m, param = PixelTrajectories(coeff, K, basis_kind="bezier", tile=4), coeff
    elif kind in ("affine_exact", "affine_linear"):
        th = torch.cat([(torch.rand(B, 2, generator=g) - 0.5) * 20, (torch.rand(B, 4, generator=g) - 0.5) * 0.1], 1)
        m = Affine(B, H, W, mode="exact" if kind == "affine_exact" else "linear", init=th)
        param = m.theta
    else:
        grid = torch.nn.functional.avg_pool2d(torch.randn(B, 2, H, W, generator=g), 7, 1, 3) * 30
        m = DenseLinearFlow(B, H, W, grid=(H, W), mode="linear", init=grid)
        param = m.grid
    init = param.detach().clone()
    obj = ATS.AnchoredSliced(n_slices=S, sigma=sigma, seed=seed + 2, **obj_kw)
    held = torch.rand(n, generator=torch.Generator().manual_seed(seed + 3)) < 0.3 if masks else None
    ls, idx = obj.log_scores(ev, m, anchor_mask=held, source_mask=None if held is None else ~held)
    loss = -ls.mean()
    loss.backward()
    extra = {"held": held} if masks else {}
    save(name, kind=kind, xy=xy, t=t, b=b, B=B, H=H, W=W, S=S, sigma=sigma, K=K, seed=seed + 2, param=init,
         ls=ls.detach(), idx=idx, loss=loss.detach(), grad=param.grad, obj_kw=repr(obj_kw), **extra)


class _MatrixExpF64:
    """Within the block, torch.linalg.matrix_exp (the reference's exact affine transport,
    atl/motion/parametric.py:64-70) is evaluated in float64 and returned in the input's dtype: the
    reference's math with an accurate exponential (its fp32 call is off by up to ~1e-4 px on these inputs)."""

    def __enter__(self):
        self.orig = torch.linalg.matrix_exp
        orig = self.orig
        torch.linalg.matrix_exp = lambda Z: orig(Z.double()).to(Z.dtype)
        return self

    def __exit__(self, *exc):
        torch.linalg.matrix_exp = self.orig


def gen_traj(name, K, basis_kind, per_event, seed, B=2, H=48, W=64, n=3000, scale=10.0):
    """PixelTrajectories.transport (atl/motion/trajectories.py:62-81) of seeded events: the transported
    positions and the gradient of sum(y * w) w.r.t. the coefficient grid, with positions spilling past the
    border (clamped coefficient samples) and scalar or per-event target times."""
    g = torch.Generator().manual_seed(seed)
    coeff = torch.nn.functional.avg_pool2d(torch.randn(B, 2 * K, H, W, generator=g), 9, 1, 4) * scale
    xy = torch.stack([torch.rand(n, generator=g) * (W + 16) - 8, torch.rand(n, generator=g) * (H + 16) - 8], 1)
    t = torch.rand(n, generator=g)
    b = torch.randint(0, B, (n,), generator=g)
    t_dst = torch.rand(n, generator=g) if per_event else torch.tensor(0.375)
    w = torch.randn(n, 2, generator=g)
    c = coeff.clone().requires_grad_(True)
    m = PixelTrajectories(c, K, basis_kind=basis_kind, tile=4)
    y = m.transport(xy, t, t_dst if per_event else 0.375, b)
    (y * w).sum().backward()
    save(name, K=K, basis=basis_kind, per_event=per_event, coeff=coeff, xy=xy, t=t, b=b, t_dst=t_dst, w=w,
         y=y.detach(), grad=c.grad)


def gen_exact_traj(name, n, B, H, W, seed, n_anchors=None, h=1.0):
    """AnchoredExact with PixelTrajectories(K=1, "polynomial") -- the trainer's loss call
    (atl/train/trainer.py:167; exact-path eligible by atl/motion/trajectories.py:54) -- on a seeded batch of
    windows: per-anchor log scores, loss, and the gradient w.r.t. the coefficient grid."""
    xy, t, b = synth_window(n, H, W, seed, B)
    ev = EventPacket(xy, t, torch.ones(n), b, B, H, W)
    g = torch.Generator().manual_seed(seed + 1)
    coeff = torch.nn.functional.avg_pool2d(torch.randn(B, 2, H, W, generator=g), 9, 1, 4) * 40
    init = coeff.clone()
    coeff.requires_grad_(True)
    m = PixelTrajectories(coeff, 1, basis_kind="polynomial", tile=4)
    assert m.linear_at_event
    obj = ATS.AnchoredExact(h=h, tau=1.0, n_anchors=n_anchors, n_slices=16, seed=seed + 2, visibility=True)
    ls, anchors = obj.log_scores(ev, m)
    loss = -ls.mean()
    loss.backward()
    save(name, xy=xy, t=t, b=b, B=B, H=H, W=W, h=h, seed=seed + 2, coeff=init, anchors=anchors, ls=ls.detach(),
         loss=loss.detach(), grad=coeff.grad)


if __name__ == "__main__":
    gen_ops()
    gen_plan("plan_tau1_s8", 600, 2, 20, 24, 3, 6.0, 1.0, 8, 1.5)
    gen_plan("plan_tau02_s16", 600, 2, 20, 24, 3, 6.0, 0.2, 16, 1.5)
    gen_plan("plan_tau005_s4", 600, 2, 20, 24, 3, 6.0, 0.05, 4, 1.5)
    gen_plan("plan_smooth_fast", 2500, 1, 48, 64, 7, 12.0, 1.0, 16, 1.0, anchor_step=2, smooth=True)
    gen_window()
    gen_motion()
    gen_exact("translation", 3000, 1, 48, 64, 40, None)
    gen_exact("affine", 3000, 2, 48, 64, 50, 2000, tau=0.5, S=8)
    gen_exact("dense", 4000, 1, 48, 64, 60, None, h=1.0)
    gen_sliced("sliced_trajectories", "trajectories", 3000, 2, 48, 64, 70, 4, 1.5)
    gen_sliced("sliced_affine_exact", "affine_exact", 3000, 1, 48, 64, 80, 5, 1.0)
    gen_sliced("sliced_dense", "dense", 3000, 1, 48, 64, 90, 4, 2.0)
    gen_sliced("sliced_traj_subsets", "trajectories", 3000, 2, 48, 64, 71, 6, 1.5, slices_per_step=4,
               n_anchors_per_slice=150, tau=0.3)
    gen_sliced("sliced_affine_plain", "affine_linear", 3000, 1, 48, 64, 81, 5, 1.0, smooth_anchors=False,
               logdet=False, dequantize=False, visibility=False)
    gen_sliced("sliced_dense_heldout", "dense", 3000, 2, 48, 64, 91, 4, 1.0, masks=True, tau=0.5)
    gen_traj("traj_k10_bezier", 10, "bezier", False, 101)
    gen_traj("traj_k3_poly_pe", 3, "polynomial", True, 102)
    gen_traj("traj_k1_poly", 1, "polynomial", False, 103)
    gen_traj("traj_k4_bezier_pe", 4, "bezier", True, 104)
    gen_exact_traj("exact_traj_k1", 4000, 4, 48, 64, 110)
    with _MatrixExpF64():
        gen_sliced("sliced_affine_exact_f64exp", "affine_exact", 3000, 1, 48, 64, 80, 5, 1.0)

