"""Host side of the multi-GPU path, on CPU: shard ranges, and the decomposition the sharded objective
relies on -- per-rank pair sums over a share of the sources, summed with an all-reduce over gloo
(world size 2, spawned ranks), equal the pair sums over all sources (C oracle)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from x_b200.distributed import allreduce_sum, shard_range


def test_shard_ranges_partition():
    for n in (0, 1, 7, 1000, 64_000_001):
        for world in (1, 2, 3, 8):
            rs = [shard_range(n, r, world) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            assert max(e - s for s, e in rs) - min(e - s for s, e in rs) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _window(n=3000, H=40, W=56, seed=3):
    rng = np.random.default_rng(seed)
    xy = np.stack([rng.integers(0, W, n), rng.integers(0, H, n)], 1).astype(np.float32)
    xy += rng.uniform(-0.5, 0.5, xy.shape).astype(np.float32)
    t = np.sort(rng.uniform(0, 1, n)).astype(np.float32)
    v = (rng.normal(size=(n, 2)) * 4).astype(np.float32)
    b = np.zeros(n, np.int64)
    return xy, t, v, b, H, W


def _restrict(plan, j0, j1):
    """The plan's entries whose source lies in [j0, j1), cells kept (what a rank's plan holds)."""
    keep = (plan["src_id"] >= j0) & (plan["src_id"] < j1)
    cs = plan["cell_start"]
    cell_of = np.repeat(np.arange(cs.shape[0] - 1), np.diff(cs))
    counts = np.bincount(cell_of[keep], minlength=cs.shape[0] - 1)
    out = dict(plan)
    for k in ("src_y", "src_v", "src_t", "src_id"):
        out[k] = np.ascontiguousarray(plan[k][keep])
    out["cell_start"] = np.concatenate([[0], np.cumsum(counts)]).astype(cs.dtype)
    return out


def _rank(rank, world, port, q):
    import torch.distributed as dist
    from oracle import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        xy, t, v, b, H, W = _window()
        n = t.shape[0]
        anchors = np.arange(n, dtype=np.int64)
        plan = O.build_pair_plan(xy, t, v, b, 1, H, W, anchors, 1.0, 1.0, 3.0, 8)
        j0, j1 = shard_range(n, rank, world)
        S_part, _ = O.pair_fwd(_restrict(plan, j0, j1), 1.0, 1.0, 3.0)
        S = allreduce_sum(torch.as_tensor(np.asarray(S_part, np.float64)))
        if rank == 0:
            S_full, _ = O.pair_fwd(plan, 1.0, 1.0, 3.0)
            q.put(float(np.abs(S.numpy() - np.asarray(S_full, np.float64)).max() / np.abs(S_full).max()))
    finally:
        dist.destroy_process_group()


def test_partial_pair_sums_allreduce_to_full_sums_gloo():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=10) < 1e-6


def _rank_sliced(rank, world, port, q):
    """The sliced path's decomposition over gloo: each rank splats its share of the points (the C oracle's
    Gaussian splat), the partial density stacks are summed by the differentiable all-reduce, and each
    rank's loss reads the full stack; the summed position gradients equal the single-process ones."""
    import torch.distributed as dist
    from oracle import oracle as O
    from x_b200.distributed import allreduce_sum_autograd
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        n, B, H, W, sigma, R = 4000, 2, 24, 40, 1.5, 5
        pos = np.stack([rng.uniform(-3, W + 3, n), rng.uniform(-3, H + 3, n)], 1).astype(np.float32)
        w = rng.uniform(0.5, 1.5, n).astype(np.float32)
        b = np.sort(rng.integers(0, B, n)).astype(np.int64)
        gimg = [rng.normal(size=(B, H, W)).astype(np.float32) for _ in range(world)]  # each rank's dL/dimg
        j0, j1 = shard_range(n, rank, world)
        part = torch.as_tensor(np.asarray(O.splat_gauss_fwd(pos[j0:j1], w[j0:j1], b[j0:j1], B, H, W, sigma, R),
                                          np.float32)).requires_grad_(True)
        img = allreduce_sum_autograd(part)
        (img * torch.as_tensor(gimg[rank])).sum().backward()
        # what the rank's splat backward receives: the sum over the ranks of dL/dimg
        g_total = np.sum(gimg, 0)
        full = np.asarray(O.splat_gauss_fwd(pos, w, b, B, H, W, sigma, R), np.float32)
        gp_rank, _ = O.splat_gauss_bwd(part.grad.numpy(), pos[j0:j1], w[j0:j1], b[j0:j1], sigma, R)
        gp_full, _ = O.splat_gauss_bwd(g_total, pos, w, b, sigma, R)
        gp_all = allreduce_sum(torch.zeros(n, 2).index_copy_(0, torch.arange(j0, j1),
                                                             torch.as_tensor(np.asarray(gp_rank, np.float32))))
        if rank == 0:
            q.put((float(np.abs(img.detach().numpy() - full).max() / np.abs(full).max()),
                   float(np.abs(part.grad.numpy() - g_total).max()),
                   float(np.abs(gp_all.numpy() - np.asarray(gp_full, np.float32)).max() /
                         np.abs(np.asarray(gp_full)).max())))
    finally:
        dist.destroy_process_group()


def test_sliced_density_allreduce_decomposition_gloo():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_sliced, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs)
    e_img, e_g, e_gp = q.get(timeout=10)
    assert e_img < 1e-6 and e_g < 1e-5 and e_gp < 1e-6
