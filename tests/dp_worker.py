"""Worker for the multi-GPU parity test (run under torch.distributed.run, one
process per GPU).  From the same start, trains a few steps of the outdoor
scene (SH degree 3 stored) five ways and checks that all give the same
parameters and moments on every GPU, before and after a densify step:

* the multicast sharded Adam: each GPU updates the pool slots it owns, fused
  with the gradient sum (multimem.ld_reduce) and the broadcast of the
  rasterizer's columns (multimem.st) — narrow gradient rows;
* the multicast row sum, then a replicated Adam — narrow rows;
* an NCCL all-reduce, then a replicated Adam — narrow rows;
* an NCCL all-reduce of full-width rows;
* the NCCL sharded Adam: a reduce-scatter of the rows, Adam on each GPU's
  block of active ids, an all-gather of the rasterizer's columns.

Then the same for an SH degree 0 scene (16-float rows, where the broadcast
columns are the whole row): both sharded Adams against the NCCL all-reduce.

Finally one data-parallel step of each NCCL path (the default all-reduce and
the sharded Adam) against the CPU oracle's single-process step: every rank renders its own view of a
small SH-3 outdoor scene; after the step, Adam's first moment (0.1 times the
gradient Adam applied) must equal 0.1 times the oracle's mean over both views
of the dense rasterizer's gradients plus the regulariser, within the gradient
tolerance (the L1 cotangent is taken from each rank's rendered image, as the
single-GPU parity tests do).
"""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from mlx_gsplat_b200 import distributed  # noqa: E402
from mlx_gsplat_b200.trainer import runner_for_workload  # noqa: E402

# workload, name, multicast, narrow rows, multicast sharded Adam, NCCL sharded Adam
CONFIGS = [("outdoor-1m", "sharded", True, True, True, False),
           ("outdoor-1m", "multicast sum", True, True, False, False),
           ("outdoor-1m", "nccl", False, True, True, False), ("outdoor-1m", "nccl full rows", False, False, True, False),
           ("outdoor-1m", "nccl sharded", False, True, False, True),
           ("mid-200k", "sharded sh0", True, True, True, False), ("mid-200k", "nccl sh0", False, True, True, False),
           ("mid-200k", "nccl sharded sh0", False, True, False, True)]


def state(r):
    r.gather_sharded_state()
    al = r.allocator
    torch.cuda.synchronize(r.device)
    t = al.indirection_table.cpu().numpy()
    return [al.theta.cpu().numpy()[t], al.adam_m.cpu().numpy()[t], al.adam_v.cpu().numpy()[t]]


def oracle_step_check(rank, world, dev, pg, nccl_sharded):
    """Returns (ok, worst relative error) of the data-parallel step against the oracle."""
    import dataclasses
    from gsutil import GRAD_RTOL
    from mlx_gsplat_b200 import synthetic
    from mlx_gsplat_b200.trainer import sh_cols_for
    from oracle import rendering as orend
    wl = dataclasses.replace(synthetic.WORKLOADS["outdoor-1m"], name="outdoor-small", num_gaussians=8000,
                             width=216, height=140, focal=1150.0 / 6)
    synthetic.WORKLOADS[wl.name] = wl
    r = runner_for_workload(wl.name, max_steps=50, device=dev, num_views=8, lr=1e-3, eps=1e-15, process_group=pg,
                            nccl_sharded_adam=nccl_sharded)
    al, L = r.allocator, r.layout
    theta0 = al.theta.cpu().numpy().copy()
    table = al.indirection_table.cpu().numpy()
    view = distributed.view_for(1, rank, world, 8)
    frame = r.train_step(view, 1)
    torch.cuda.synchronize(dev)
    mine = (view, frame.color.cpu().numpy(), frame.ids[:frame.V].cpu().numpy().astype(np.int64))
    views = [None] * world
    dist.all_gather_object(views, mine, group=pg)
    r.gather_sharded_state()  # the sharded Adam leaves each block's moments with its owner
    m_after = al.adam_m.cpu().numpy()[table]
    if rank != 0:
        return True, 0.0
    N, reg = table.shape[0], r.cfg.param_reg
    act = {k: theta0[table][:, o:o + L.dims[k]] for k, o in L.offsets.items()}
    ncols = sh_cols_for(1, r.cfg)
    colors = np.concatenate([act["sh0"], act["shN"]], 1)[:, :ncols]
    G = np.zeros((N, L.ncols), np.float64)
    P = wl.pixels
    for v, C, ids in views:
        tf = r.targets[v].cpu().numpy().astype(np.float32) / np.float32(255.0)
        dC = np.sign(C.astype(np.float64) - tf) / (3.0 * P)
        _, _, gr = orend.rasterize_dense_vjp(act["means"][ids], act["quats"][ids], act["scales"][ids],
                                             act["opacities"][ids], colors[ids], r.viewmats[v], r.K, wl.width,
                                             wl.height, wl.width, wl.height, dL_dC=dC)
        for k in ("means", "quats", "scales", "opacities"):
            o = L.offsets[k]
            G[:, o:o + L.dims[k]] += reg
            G[ids, o:o + L.dims[k]] += gr[k]
        G[ids, L.color_col:L.color_col + ncols] += gr["colors"] + reg
    G /= world
    worst, ok = 0.0, True
    for k, o in L.offsets.items():
        d = L.dims[k]
        got = m_after[:, o:o + d].astype(np.float64) / 0.1
        ref = G[:, o:o + d]
        nref = np.linalg.norm(ref)
        rel = np.linalg.norm(got - ref) / nref if nref > 0 else np.abs(got).max()
        floor = 1e-4 * np.abs(ref).max()
        bad = np.abs(got - ref) > GRAD_RTOL * np.abs(ref) + floor
        worst = max(worst, float(rel))
        ok = ok and rel <= GRAD_RTOL and not bad.any()
    return ok, worst


def main():
    rank, world, local, pg = distributed.init_from_env("nccl", timeout_s=120.0)
    dev = torch.device("cuda", local)
    out = {}
    for wl, name, fused, compact, sharded, nccl_sharded in CONFIGS:
        r = runner_for_workload(wl, n=20_000, max_steps=100, device=dev, num_views=8, process_group=pg,
                                fused_reduce=fused, compact_grad_rows=compact, sharded_adam=sharded,
                                nccl_sharded_adam=nccl_sharded, max_gaussians=60_000)
        if fused and r.fused_reduce is None:
            print("SKIP: no multicast support", flush=True)
            dist.destroy_process_group()
            return
        assert wl != "outdoor-1m" or (r.g_stride == 24) == compact
        assert r.sharded == (fused and sharded) and r.sharded_nccl == nccl_sharded
        for step in range(1, 4):
            r.train_step(distributed.view_for(step, rank, world, 8), step)
        before = state(r)
        # densify from fixed statistics (the same on every rank and in every run)
        al = r.allocator
        g = torch.Generator(device=dev)
        g.manual_seed(9)
        al.grad2d.copy_(torch.rand(al.max_gaussians, generator=g, device=dev) * 4e-4)
        al.count.fill_(1.0)
        r.densify(4)
        r.train_step(distributed.view_for(4, rank, world, 8), 4)
        if r.fused_reduce is not None:
            r.fused_reduce.check()
        out[name] = before + state(r)
    groups = {"sharded": [k for k in out if not k.endswith("sh0")], "sharded sh0": ["nccl sh0", "nccl sharded sh0"]}
    err, ok = 0.0, True
    for refname, others in groups.items():
        ref = out[refname]
        for o in (out[k] for k in others):
            err = max([err] + [float(np.abs(a - b).max()) for a, b in zip(ref, o) if a.shape == b.shape])
            ok = ok and len(o) == len(ref) and all(a.shape == b.shape and np.allclose(a, b, rtol=1e-5, atol=1e-6)
                                                   for a, b in zip(ref, o))
    ok_oracle, err_oracle = True, 0.0
    for nccl_sharded in (False, True):
        o, e = oracle_step_check(rank, world, dev, pg, nccl_sharded)
        ok_oracle, err_oracle = ok_oracle and o, max(err_oracle, e)
    ok = ok and ok_oracle
    gathered = [None] * world
    dist.all_gather_object(gathered, (bool(ok), float(err), ("oracle", bool(ok_oracle), float(err_oracle)),
                                      {k: [x.shape for x in v] for k, v in out.items()}), group=pg)
    if rank == 0:
        print("RESULT", gathered, flush=True)
    dist.barrier(group=pg)
    dist.destroy_process_group()
    if not ok:
        sys.exit(1)


if __name__ == "__main__":
    main()
