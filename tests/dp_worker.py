"""Worker for the multi-GPU parity test (run under torch.distributed.run, one
process per GPU): trains a few steps of the outdoor scene (SH degree 3
stored) with the gradient rows summed over GPUs by the NVLink multicast
kernels and, from the same start, by an NCCL all-reduce — both with narrow
gradient rows (23 columns + the view count) — and by an NCCL all-reduce of
full-width rows, and checks that all three give the same parameters on every
GPU."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from mlx_gsplat_b200 import distributed  # noqa: E402
from mlx_gsplat_b200.trainer import runner_for_workload  # noqa: E402


def main():
    rank, world, local, pg = distributed.init_from_env("nccl", timeout_s=120.0)
    dev = torch.device("cuda", local)
    out = {}
    for fused, compact in ((True, True), (False, True), (False, False)):
        r = runner_for_workload("outdoor-1m", n=20_000, max_steps=100, device=dev, num_views=8, process_group=pg,
                                fused_reduce=fused, compact_grad_rows=compact)
        if fused and r.fused_reduce is None:
            print("SKIP: no multicast support", flush=True)
            dist.destroy_process_group()
            return
        assert (r.g_stride == 24) == compact
        for step in range(1, 4):
            r.train_step(distributed.view_for(step, rank, world, 8), step)
        torch.cuda.synchronize(dev)
        if r.fused_reduce is not None:
            r.fused_reduce.check()
        n = r.allocator.num_active
        out[(fused, compact)] = r.allocator.theta[:n].cpu().numpy()
    a = out[(True, True)]
    err = max(float(np.abs(a - b).max()) for b in out.values())
    # same gradients up to the summation order of the cross-GPU sum
    ok = all(np.allclose(a, b, rtol=1e-5, atol=1e-6) for b in out.values())
    gathered = [None] * world
    dist.all_gather_object(gathered, (bool(ok), float(err)), group=pg)
    if rank == 0:
        print("RESULT", gathered, flush=True)
    dist.barrier(group=pg)
    dist.destroy_process_group()
    if not ok:
        sys.exit(1)


if __name__ == "__main__":
    main()
