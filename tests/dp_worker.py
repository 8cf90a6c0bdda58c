"""Worker for the multi-GPU parity test (run under torch.distributed.run, one
process per GPU).  From the same start, trains a few steps of the outdoor
scene (SH degree 3 stored) four ways and checks that all give the same
parameters and moments on every GPU, before and after a densify step:

* the sharded Adam: each GPU updates the pool slots it owns, fused with the
  gradient sum (multimem.ld_reduce) and the broadcast of the rasterizer's
  columns (multimem.st) — narrow gradient rows;
* the multicast row sum, then a replicated Adam — narrow rows;
* an NCCL all-reduce, then a replicated Adam — narrow rows;
* an NCCL all-reduce of full-width rows.

Then the same for an SH degree 0 scene (16-float rows, where the broadcast
columns are the whole row): the sharded Adam against the NCCL all-reduce.
"""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from mlx_gsplat_b200 import distributed  # noqa: E402
from mlx_gsplat_b200.trainer import runner_for_workload  # noqa: E402

CONFIGS = [("outdoor-1m", "sharded", True, True, True), ("outdoor-1m", "multicast sum", True, True, False),
           ("outdoor-1m", "nccl", False, True, True), ("outdoor-1m", "nccl full rows", False, False, True),
           ("mid-200k", "sharded sh0", True, True, True), ("mid-200k", "nccl sh0", False, True, True)]


def state(r):
    r.gather_sharded_state()
    al = r.allocator
    torch.cuda.synchronize(r.device)
    t = al.indirection_table.cpu().numpy()
    return [al.theta.cpu().numpy()[t], al.adam_m.cpu().numpy()[t], al.adam_v.cpu().numpy()[t]]


def main():
    rank, world, local, pg = distributed.init_from_env("nccl", timeout_s=120.0)
    dev = torch.device("cuda", local)
    out = {}
    for wl, name, fused, compact, sharded in CONFIGS:
        r = runner_for_workload(wl, n=20_000, max_steps=100, device=dev, num_views=8, process_group=pg,
                                fused_reduce=fused, compact_grad_rows=compact, sharded_adam=sharded,
                                max_gaussians=60_000)
        if fused and r.fused_reduce is None:
            print("SKIP: no multicast support", flush=True)
            dist.destroy_process_group()
            return
        assert wl != "outdoor-1m" or (r.g_stride == 24) == compact
        assert r.sharded == (fused and sharded)
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
    groups = {"sharded": [k for k in out if not k.endswith("sh0")], "sharded sh0": ["nccl sh0"]}
    err, ok = 0.0, True
    for refname, others in groups.items():
        ref = out[refname]
        for o in (out[k] for k in others):
            err = max([err] + [float(np.abs(a - b).max()) for a, b in zip(ref, o) if a.shape == b.shape])
            ok = ok and len(o) == len(ref) and all(a.shape == b.shape and np.allclose(a, b, rtol=1e-5, atol=1e-6)
                                                   for a, b in zip(ref, o))
    gathered = [None] * world
    dist.all_gather_object(gathered, (bool(ok), float(err), {k: [x.shape for x in v] for k, v in out.items()}),
                           group=pg)
    if rank == 0:
        print("RESULT", gathered, flush=True)
    dist.barrier(group=pg)
    dist.destroy_process_group()
    if not ok:
        sys.exit(1)


if __name__ == "__main__":
    main()
