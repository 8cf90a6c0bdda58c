"""Gradient rows summed over GPUs by this library's NVLink multicast kernels
(bounded device barrier, multimem load-reduce + store of each GPU's slice)
against the NCCL all-reduce path: a few training steps from the same start
give the same parameters (rtol 1e-5; the two sums differ only in their
order).  Needs at least two GPUs of one NVSwitch domain."""
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
    tail = (r.stdout + r.stderr)[-3000:]
    if "SKIP: no multicast support" in r.stdout:
        pytest.skip("no NVLink multicast on this machine")
    assert r.returncode == 0, tail
    assert "RESULT" in r.stdout, tail
