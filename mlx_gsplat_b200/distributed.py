"""Views data-parallel training across the GPUs of one box.

Every rank holds the whole pool (the Gaussians are replicated); each step every
rank renders its own camera view and stores the gradient rows of the
Gaussians it saw (without the geometry regulariser) into a zeroed slab, the
rows are summed over ranks (an NCCL all-reduce over NVLink, or the multicast
kernels of ``FusedRowReduce``), and every rank runs the same fused Adam on the
summed rows plus ``world * reg`` scaled by 1/world, so the replicas stay
bit-identical without any parameter broadcast.  The densification statistics
(grad2d, count) are summed before each densify step, and the densify noise is
drawn from a generator seeded by the step, identically on every rank.

The functions here hold that host-side logic; they work with any
``torch.distributed`` backend (NCCL on GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.distributed as dist


def world_of(pg) -> int:
    return 1 if pg is None else dist.get_world_size(pg)


def rank_of(pg) -> int:
    return 0 if pg is None else dist.get_rank(pg)


def view_for(step: int, rank: int, world: int, num_views: int) -> int:
    """The camera view rank ``rank`` trains on at ``step``: the world's ranks
    take consecutive views, and consecutive steps advance by ``world``."""
    return (rank + world * step) % num_views


def reduce_gradient_rows(grad_rows: torch.Tensor, pg) -> float:
    """Sums the gradient rows of all ranks in place; returns the scale Adam
    applies to them (1/world, so the update follows the mean over views)."""
    w = world_of(pg)
    if w > 1:
        dist.all_reduce(grad_rows, op=dist.ReduceOp.SUM, group=pg)
    return 1.0 / w


def reduce_densify_stats(grad2d: torch.Tensor, count: torch.Tensor, pg) -> None:
    """Sums the per-slot densification statistics over ranks in place."""
    if world_of(pg) > 1:
        dist.all_reduce(grad2d, op=dist.ReduceOp.SUM, group=pg)
        dist.all_reduce(count, op=dist.ReduceOp.SUM, group=pg)


def densify_noise(step: int, n: int, device) -> Dict[str, torch.Tensor]:
    """The normal draws of one densify step (child means x2, child quaternion),
    from a generator seeded by the step so every rank draws the same values."""
    gen = torch.Generator(device=device)
    gen.manual_seed(1_000_003 * int(step) + 17)
    return {"means1": torch.randn((n, 3), generator=gen, device=device),
            "means2": torch.randn((n, 3), generator=gen, device=device),
            "quats2": torch.randn((n, 4), generator=gen, device=device)}


class FusedRowReduce:
    """Gradient rows summed over the GPUs of one NVSwitch domain by the GPUs
    themselves through NVLink multicast, instead of by an NCCL all-reduce.

    The row slab lives in symmetric memory with a multicast mapping.  Each GPU
    stores its visible rows locally (without the geometry regulariser, which
    Adam adds once for every row: ``world * reg`` before the ``1/world`` scale)
    into a slab that is zero elsewhere.  ``sum_rows`` then waits until every
    GPU has written (barrier), sums this GPU's 1/world slice of the rows across
    all copies and stores the sums to all of them (``multimem.ld_reduce`` +
    ``multimem.st``: one writer per element, so every replica gets the same
    bits), and waits until every slice is done (barrier).  After Adam each GPU
    zeroes its own copy; the next step's first barrier keeps peers from
    summing before that.  Barrier waits are bounded; a timeout sets ``error``
    (``check`` raises), it never stalls the GPU.

    Use ``available`` first: it needs NCCL, more than one GPU and multicast
    support; otherwise the trainer keeps the all-reduce path.
    """

    MAX_POLLS = 1 << 25  # about 3 s of polling per wait

    def __init__(self, rows: int, cols: int, device, pg, theta_cols: Optional[int] = None):
        """``theta_cols``: also allocate the ``[rows, theta_cols]`` parameter
        slab in symmetric memory with a multicast mapping (``theta``,
        ``theta_multicast``) for the sharded Adam (``gs_fused_adam_slab_sharded``)."""
        import torch.distributed._symmetric_memory as symm
        from . import _lib
        self.device = torch.device(device)
        self.pg = pg
        self.rank = rank_of(pg)
        self.world = world_of(pg)
        name = pg.group_name
        try:
            symm.enable_symm_mem_for_group(name)
        except Exception:
            pass  # newer releases enable groups on first rendezvous
        self.rows = symm.empty((rows, cols), dtype=torch.float32, device=self.device)
        self.rows.zero_()
        self._rows_hdl = symm.rendezvous(self.rows, name)
        self.multicast = int(self._rows_hdl.multicast_ptr)
        if self.multicast == 0:
            raise RuntimeError("no NVLink multicast mapping for the gradient rows")
        self.theta = None
        self.theta_multicast = 0
        if theta_cols is not None:
            self.theta = symm.empty((rows, theta_cols), dtype=torch.float32, device=self.device)
            self._theta_hdl = symm.rendezvous(self.theta, name)
            self.theta_multicast = int(self._theta_hdl.multicast_ptr)
            if self.theta_multicast == 0:
                raise RuntimeError("no NVLink multicast mapping for the parameter slab")
        self.pads = symm.empty((2 * self.world,), dtype=torch.int32, device=self.device)
        self.pads.zero_()
        self._pads_hdl = symm.rendezvous(self.pads, name)
        self.peer_pads = torch.tensor([int(p) for p in self._pads_hdl.buffer_ptrs], dtype=torch.int64,
                                      device=self.device)
        self.error = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.epoch = [0, 0]
        self._lib = _lib
        torch.cuda.synchronize(self.device)
        dist.barrier(group=pg)

    @staticmethod
    def available(device, pg) -> bool:
        if pg is None or world_of(pg) < 2 or dist.get_backend(pg) != "nccl":
            return False
        try:
            import torch.distributed._symmetric_memory as symm
            return bool(symm._SymmetricMemory.has_multicast_support(symm.DeviceType.CUDA,
                                                                     torch.device(device).index or 0))
        except Exception:
            return False

    def _barrier(self, channel: int) -> None:
        self.epoch[channel] = (self.epoch[channel] + 1) & 0xFFFFFFFF
        lib = self._lib.lib()
        self._lib.check(lib.gs_group_barrier(self.peer_pads.data_ptr(), self.rank, self.world, channel,
                                             self.epoch[channel], self.error.data_ptr(), self.MAX_POLLS,
                                             self._lib.stream_ptr(self.device)), "group barrier")

    def barrier(self, channel: int) -> None:
        """Group barrier on ``channel`` (0 or 1), enqueued on the current stream."""
        self._barrier(channel)

    def owned_slots(self, rows: int) -> torch.Tensor:
        """Boolean mask of the physical slots whose rows this GPU updates in the
        sharded Adam (slot % world == rank)."""
        return (torch.arange(rows, device=self.device) % self.world) == self.rank

    def gather_owned_rows(self, t: torch.Tensor, owned: torch.Tensor, rows: Optional[slice] = None,
                          first_col: int = 0) -> None:
        """``gather_owned_rows`` over this group."""
        gather_owned_rows(t, owned, self.pg, rows, first_col)

    def slice_of(self, n_rows: int):
        """This GPU's rows of the sum: a contiguous 1/world share."""
        per = -(-n_rows // self.world)
        first = min(self.rank * per, n_rows)
        return first, min(per, n_rows - first)

    def sum_rows(self, n_rows: int) -> None:
        """Rows [0, n_rows) of every GPU's copy become the sum over GPUs."""
        self._barrier(0)
        first, count = self.slice_of(n_rows)
        lib = self._lib.lib()
        self._lib.check(lib.gs_rows_sum_multicast(self.multicast, first, count, self.rows.shape[1],
                                                  self.error.data_ptr(), self._lib.stream_ptr(self.device)),
                        "multicast row sum")
        self._barrier(1)

    def check(self) -> None:
        """Raises if a group barrier of this GPU gave up waiting for a peer (a
        host sync).  The row sum and the sharded Adam read the flag and skip
        their work on that GPU, so no partial sum is applied there, but the
        replicas are no longer in step and training cannot go on."""
        if int(self.error.item()) != 0:
            raise RuntimeError("multi-GPU barrier timed out (a peer did not arrive)")


def gather_owned_rows(t: torch.Tensor, owned: torch.Tensor, pg, rows: Optional[slice] = None,
                      first_col: int = 0) -> None:
    """Every rank's copy of the slot-indexed rows of ``t`` becomes the owners'
    rows: the rows this rank does not own are zeroed, then summed over the
    group (an all-reduce).  The sharded Adams leave some columns and the
    moments current only on the rank that owns a slot; densify, export and
    checkpoints call this first.  Only the slot range ``rows`` (default: all)
    and the columns from ``first_col`` on move: the columns every rank already
    holds identically (the broadcast ones) and unused slots need no exchange."""
    rows = rows if rows is not None else slice(0, t.shape[0])
    part = t[rows, first_col:]
    if part.numel() == 0:
        return
    buf = part.contiguous()
    buf.masked_fill_(~owned[rows].unsqueeze(1), 0.0)
    dist.all_reduce(buf, group=pg)
    part.copy_(buf)


def block_of(n_rows: int, rank: int, world: int):
    """The contiguous block of rows [first, first + count) rank ``rank`` owns when
    ``n_rows`` rows are cut into ``world`` equal blocks of ``per`` rows (the
    last ones padded): returns (first, count, per)."""
    per = -(-n_rows // world) if n_rows > 0 else 0
    first = min(rank * per, n_rows)
    return first, max(0, min(per, n_rows - first)), per


SHARDED_NCCL_ADAM_MIN_WORLD = 4


def use_sharded_nccl_adam(setting, world: int, multicast: bool = False) -> bool:
    """Which NCCL path sums the gradient rows of a group of ``world`` GPUs:
    True — reduce-scatter, Adam on this GPU's block of rows, all-gather of the
    rasterizer's columns; False — an all-reduce with a replicated Adam.
    ``setting`` True / False forces one; None picks the sharded Adam from
    SHARDED_NCCL_ADAM_MIN_WORLD GPUs up (on 2 GPUs the replicated Adam measured
    faster, 705 against 682 steps/s; on 4 the sharded one, 1387 against 1354).
    Neither runs on one GPU or with the NVLink multicast sum."""
    if world <= 1 or multicast:
        return False
    return bool(setting) if setting is not None else world >= SHARDED_NCCL_ADAM_MIN_WORLD


def init_from_env(backend: str = "nccl", timeout_s: float = 180.0):
    """Initialise the default process group from torchrun's environment
    (RANK, WORLD_SIZE, LOCAL_RANK, MASTER_ADDR/PORT); returns (rank, world,
    local_rank, group or None for a single process)."""
    import datetime
    import os
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world == 1:
        return rank, world, local, None
    kw = {}
    if backend == "nccl":
        torch.cuda.set_device(local)
        kw["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world, local, dist.group.WORLD


def max_over_ranks(x: float, pg, device: Optional[torch.device] = None) -> float:
    if world_of(pg) == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=pg)
    return float(t.item())
