"""Worker for the multi-GPU parity test (run under torch.distributed.run, one
process per GPU): trains a few steps with the gradient rows summed over GPUs
by the NVLink multicast kernels and, from the same start, by an NCCL
all-reduce, and checks that both give the same parameters on every GPU."""
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
    for fused in (True, False):
        r = runner_for_workload("mid-200k", n=20_000, max_steps=100, device=dev, num_views=8, process_group=pg,
                                fused_reduce=fused)
        if fused and r.fused_reduce is None:
            print("SKIP: no multicast support", flush=True)
            dist.destroy_process_group()
            return
        for step in range(1, 4):
            r.train_step(distributed.view_for(step, rank, world, 8), step)
        torch.cuda.synchronize(dev)
        if r.fused_reduce is not None:
            r.fused_reduce.check()
        n = r.allocator.num_active
        out[fused] = r.allocator.theta[:n].cpu().numpy()
    a, b = out[True], out[False]
    err = np.abs(a - b).max()
    # same gradients up to the summation order of the cross-GPU sum
    ok = np.allclose(a, b, rtol=1e-5, atol=1e-6)
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
