"""The bounded device barrier of the multi-GPU step (gs_group_barrier) on one
GPU, through the C ABI.

The barrier's waits are bounded: a peer that never signals makes the wait
give up after ``max_polls`` polls, set the error flag and return, so the GPU
never spins forever and the context stays usable.  Here a group of two is
emulated on one GPU: the absent peer's signal pad is a second buffer on this
GPU that nothing writes, so the wait for it runs out.  Then the same barrier
with the peer's signal already in place passes without an error.
"""
import time

import pytest
import torch

from mlx_gsplat_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _barrier(lib, ptrs, rank, world, channel, epoch, err, max_polls):
    _lib.check(lib.gs_group_barrier(ptrs.data_ptr(), rank, world, channel, epoch, err.data_ptr(), max_polls,
                                    _lib.stream_ptr()), "group barrier")


def test_group_barrier_wait_runs_out_and_sets_the_error_flag():
    lib = _lib.lib()
    world, channels = 2, 2
    own = torch.zeros(channels * world, dtype=torch.int32, device=DEV)    # this GPU's pad [channel][rank]
    peer = torch.zeros(channels * world, dtype=torch.int32, device=DEV)   # stands in for the absent peer's pad
    ptrs = torch.tensor([own.data_ptr(), peer.data_ptr()], dtype=torch.int64, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _barrier(lib, ptrs, 0, world, 1, 7, err, 2000)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(err.item()) == 1, "the wait for a peer that never signals must set the error flag"
    assert dt < 5.0, f"a 2000-poll wait took {dt:.2f} s"
    # this GPU's signal to the peer (pad [channel 1][rank 0]) was written before the wait
    assert peer.cpu().tolist() == [0, 0, 7, 0]
    # the context is still usable, and a barrier whose peer has signalled passes
    err.zero_()
    own[1 * world + 1] = 8  # the peer's signal for epoch 8 on channel 1
    _barrier(lib, ptrs, 0, world, 1, 8, err, 2000)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert peer.cpu().tolist() == [0, 0, 8, 0]
    x = torch.arange(1000, device=DEV, dtype=torch.float32)
    assert float(x.sum()) == 499500.0


def test_group_barrier_rejects_bad_arguments():
    lib = _lib.lib()
    pads = torch.zeros(4, dtype=torch.int32, device=DEV)
    ptrs = torch.tensor([pads.data_ptr(), pads.data_ptr()], dtype=torch.int64, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = _lib.stream_ptr()
    assert lib.gs_group_barrier(ptrs.data_ptr(), 2, 2, 0, 1, err.data_ptr(), 10, st) == _lib.GS_ERR_INVALID
    assert lib.gs_group_barrier(ptrs.data_ptr(), 0, 2, 0, 1, err.data_ptr(), 0, st) == _lib.GS_ERR_INVALID
    assert lib.gs_group_barrier(None, 0, 2, 0, 1, err.data_ptr(), 10, st) == _lib.GS_ERR_INVALID
    # a group of one has nothing to wait for
    assert lib.gs_group_barrier(ptrs.data_ptr(), 0, 1, 0, 1, err.data_ptr(), 10, st) == _lib.GS_OK
    torch.cuda.synchronize()
    assert int(err.item()) == 0
