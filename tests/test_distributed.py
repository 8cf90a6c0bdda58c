"""Views data-parallel host logic with 2 gloo ranks on the CPU: the gradient
all-reduce and its 1/world scale, the view assignment, identical densify noise
on every rank, the statistics reduction, and — with the CPU oracle standing in
for the per-view GPU computation — that a data-parallel Adam step equals the
single-process step on the mean gradient and leaves the replicas identical."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(fn, world=2):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r, ok, payload = q.get(timeout=240)
        results[r] = (ok, payload)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        ok, payload = results[r]
        assert ok, f"rank {r}: {payload}"
    return [results[r][1] for r in range(world)]


def _entry(fn, rank, world, port, q):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        out = fn(rank, world)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, True, out))
    except Exception as e:  # report, never hang the parent
        import traceback
        q.put((rank, False, traceback.format_exc()))


def _reduce_views_noise(rank, world):
    from mlx_gsplat_b200 import distributed as D
    pg = dist.group.WORLD
    g = torch.from_numpy(np.random.default_rng(rank).normal(0, 1, (100, 60)).astype(np.float32))
    mine = g.clone()
    scale = D.reduce_gradient_rows(g, pg)
    views = [D.view_for(7, r, world, 160) for r in range(world)]
    noise = D.densify_noise(300, 50, "cpu")
    g2 = torch.full((10,), float(rank + 1))
    c2 = torch.ones(10)
    D.reduce_densify_stats(g2, c2, pg)
    return {"sum": g.numpy(), "mine": mine.numpy(), "scale": scale, "views": views,
            "noise": {k: v.numpy() for k, v in noise.items()}, "g2": g2.numpy(), "c2": c2.numpy()}


def test_gradient_reduction_views_and_noise():
    a, b = _run(_reduce_views_noise)
    np.testing.assert_allclose(a["sum"], a["mine"] + b["mine"], rtol=1e-6)
    np.testing.assert_array_equal(a["sum"], b["sum"])
    assert a["scale"] == b["scale"] == 0.5
    assert len(set(a["views"])) == 2 and a["views"] == b["views"]
    for k in a["noise"]:
        np.testing.assert_array_equal(a["noise"][k], b["noise"][k])
    np.testing.assert_array_equal(a["g2"], np.full(10, 3.0, np.float32))
    np.testing.assert_array_equal(a["c2"], np.full(10, 2.0, np.float32))


def _scene():
    from mlx_gsplat_b200 import synthetic
    wl = synthetic.WORKLOADS["tiny-3k"]
    g = synthetic.make_gaussians(wl, seed=3, n=40)
    views, _ = synthetic.make_cameras(wl, seed=2, num_views=4)
    K = np.array([[30.0, 0, 16.0], [0, 30.0, 12.0], [0, 0, 1]], np.float32)
    return g, views, K


def _view_grads(g, vm, K):
    """Per-view gradient rows [N, 14] (quats, means, opacity, scales, sh0) from the oracle."""
    from oracle import rendering as orend
    ids = orend.cull(g["means"], g["opacities"], vm, K, 32, 24).astype(np.int64)
    C, _ = orend.rasterize_dense(g["means"][ids], g["quats"][ids], g["scales"][ids], g["opacities"][ids],
                                 g["sh0"][ids], vm, K, 32, 24, 32, 24)
    dC = np.full_like(C, 1.0 / (3 * 32 * 24))
    _, _, gr = orend.rasterize_dense_vjp(g["means"][ids], g["quats"][ids], g["scales"][ids], g["opacities"][ids],
                                         g["sh0"][ids], vm, K, 32, 24, 32, 24, dL_dC=dC)
    rows = np.zeros((g["means"].shape[0], 14), np.float32)
    for name, off, d in (("quats", 0, 4), ("means", 4, 3), ("opacities", 7, 1), ("scales", 8, 3)):
        rows[ids, off:off + d] = gr[name]
    rows[ids, 11:14] = gr["colors"]
    return rows


def _adam_rows(theta, g, scale):
    from oracle import adam as oadam
    th = theta.copy()
    m = np.zeros_like(th)
    v = np.zeros_like(th)
    gg = (g * np.float32(scale)).astype(np.float32)
    oadam.fused_adam_a1(th, gg, m, v, np.arange(th.shape[0], dtype=np.int32), 1e-3, 0.9, 0.999, 1e-15, 0.0, 1,
                        -1e10, 1e10)
    return th


def _dp_step(rank, world):
    from mlx_gsplat_b200 import distributed as D
    g, views, K = _scene()
    v = D.view_for(0, rank, world, len(views))
    rows = torch.from_numpy(_view_grads(g, views[v], K))
    scale = D.reduce_gradient_rows(rows, dist.group.WORLD)
    theta = np.concatenate([g["quats"], g["means"], g["opacities"], g["scales"], g["sh0"]], 1).astype(np.float32)
    return {"theta": _adam_rows(theta, rows.numpy(), scale), "view": v}


def test_data_parallel_step_equals_mean_gradient_step():
    a, b = _run(_dp_step)
    np.testing.assert_array_equal(a["theta"], b["theta"])  # replicas stay identical
    g, views, K = _scene()
    total = _view_grads(g, views[a["view"]], K) + _view_grads(g, views[b["view"]], K)
    theta = np.concatenate([g["quats"], g["means"], g["opacities"], g["scales"], g["sh0"]], 1).astype(np.float32)
    ref = _adam_rows(theta, total, 0.5)
    np.testing.assert_allclose(a["theta"], ref, rtol=1e-6, atol=1e-7)


def _rank_failure(rank, world):
    """A rank that raises before the collective: the other rank's collective
    must end with an error inside the process-group timeout, not hang."""
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    from mlx_gsplat_b200 import distributed as D
    t = torch.ones(4)
    try:
        D.reduce_gradient_rows(t, dist.group.WORLD)
    except Exception:
        return "collective failed as expected"
    return "collective returned"


def test_rank_failure_surfaces_as_error():
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(_rank_failure, r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, ok, payload = q.get(timeout=240)
        got[r] = (ok, payload)
    for p in procs:
        p.join(timeout=90)
        if p.is_alive():
            p.kill()
    assert got[1][0] is False and "injected failure" in got[1][1]
    # rank 0 either saw its collective fail or failed at the final barrier; it did not hang
    assert got[0][0] is False or got[0][1] == "collective failed as expected"


def _narrow_rows(rank, world):
    """Each rank's gradient rows for the Gaussians its view saw, full width and
    narrow (23 gradient columns + a view-count column), summed over ranks."""
    from mlx_gsplat_b200 import distributed as D
    rng = np.random.default_rng(10 + rank)
    n, ncols, reg = 64, 59, 1e-5
    seen = rng.uniform(0, 1, n) < 0.6
    full = np.zeros((n, 60), np.float32)
    full[seen, :23] = rng.normal(0, 1, (int(seen.sum()), 23))
    full[seen, 11:23] += np.float32(reg)   # colour columns the rasterizer reads carry reg + gradient
    full[seen, 23:ncols] = np.float32(reg)  # the rest only the regulariser
    narrow = np.zeros((n, 24), np.float32)
    narrow[:, :23] = full[:, :23]
    narrow[seen, 23] = 1.0
    F, N = torch.from_numpy(full), torch.from_numpy(narrow)
    D.reduce_gradient_rows(F, dist.group.WORLD)
    D.reduce_gradient_rows(N, dist.group.WORLD)
    return {"full": F.numpy(), "narrow": N.numpy()}


def test_narrow_gradient_rows_sum_like_full_rows():
    """The all-reduce of narrow rows, expanded as Adam expands them (column
    c >= 23 = view count * reg), equals the all-reduce of full rows."""
    a, b = _run(_narrow_rows)
    np.testing.assert_array_equal(a["narrow"], b["narrow"])
    nar, full = a["narrow"], a["full"]
    expanded = np.concatenate([nar[:, :23], nar[:, 23:24] * np.float32(1e-5) * np.ones((1, 36), np.float32)], 1)
    np.testing.assert_allclose(expanded, full[:, :59], rtol=1e-6, atol=0)
    assert nar[:, 23].max() <= 2 and nar[:, 23].sum() > 0


def _gather_owned(rank, world):
    """gather_owned_rows on gloo ranks: each rank holds the true rows of the
    slots it owns (slot % world == rank) and garbage (NaN included) elsewhere
    in the columns the owners keep; the broadcast columns are identical."""
    from mlx_gsplat_b200 import distributed as D
    rows, cols, hot = 40, 12, 4
    truth = np.random.default_rng(0).normal(0, 1, (rows, cols)).astype(np.float32)
    t = torch.from_numpy(truth.copy())
    owned = (torch.arange(rows) % world) == rank
    junk = torch.from_numpy(np.random.default_rng(100 + rank).normal(0, 1, (rows, cols)).astype(np.float32))
    junk[3, 7] = float("nan")
    t[~owned, hot:] = junk[~owned, hot:]
    outside = t[:10].clone()
    D.gather_owned_rows(t, owned, dist.group.WORLD, slice(10, rows), first_col=hot)
    return {"t": t.numpy(), "truth": truth, "outside": outside.numpy()}


def test_gather_owned_rows_moves_only_the_used_range_and_owner_columns():
    a, b = _run(_gather_owned)
    for r in (a, b):
        np.testing.assert_array_equal(r["t"][10:], r["truth"][10:])  # used slots: the owners' rows
        np.testing.assert_array_equal(r["t"][:10], r["outside"])     # outside the range: untouched
    np.testing.assert_array_equal(a["t"][10:], b["t"][10:])


def test_row_blocks_cover_every_row_once():
    from mlx_gsplat_b200 import distributed as D
    for n in (0, 1, 7, 8, 9, 1000, 1001):
        for w in (1, 2, 3, 8):
            seen = []
            for r in range(w):
                first, count, per = D.block_of(n, r, w)
                assert count <= per and per * w >= n
                seen += list(range(first, first + count))
            assert seen == list(range(n)), (n, w)


def test_nccl_path_choice():
    """The NCCL gradient path: the replicated Adam on 2 GPUs, the sharded one
    from 4 up, either forced by the setting, neither on one GPU or with the
    NVLink multicast sum."""
    from mlx_gsplat_b200 import distributed as D
    assert [D.use_sharded_nccl_adam(None, w) for w in (1, 2, 3, 4, 8)] == [False, False, False, True, True]
    assert D.use_sharded_nccl_adam(True, 2) and not D.use_sharded_nccl_adam(False, 8)
    assert not D.use_sharded_nccl_adam(True, 1)
    assert not D.use_sharded_nccl_adam(None, 8, multicast=True) and not D.use_sharded_nccl_adam(True, 4, True)
