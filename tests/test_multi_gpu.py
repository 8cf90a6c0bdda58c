"""The multi-GPU paths of the training step on two GPUs (``tests/dp_worker.py``):
the sharded Adam fused with the NVLink multicast gradient sum and parameter
broadcast, the multicast row sum with a replicated Adam, and the NCCL
all-reduce of narrow and of full-width gradient rows give the same parameters
and moments after a few steps and after a densify step (rtol 1e-5; the sums
differ only in their order).  Needs at least two GPUs of one NVSwitch
domain."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_multicast_row_sum_matches_allreduce():
    env = dict(os.environ, NCCL_NVLS_ENABLE=os.environ.get("NCCL_NVLS_ENABLE", "1"))
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29533",
           os.path.join(HERE, "dp_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    print(r.stdout[-4000:])
    tail = (r.stdout + r.stderr)[-3000:]
    if "SKIP: no multicast support" in r.stdout:
        pytest.skip("no NVLink multicast on this machine")
    assert r.returncode == 0, tail
    assert "RESULT" in r.stdout, tail
