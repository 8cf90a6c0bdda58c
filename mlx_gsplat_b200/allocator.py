"""``PointerStableChunkedAllocator`` (mlx_gsplat/allocator.py:8-307) on B200.

The pool is one fixed-capacity **slab** per state (parameters, Adam m, Adam v):
``[max_gaussians, stride]`` float32 in HBM, one 16-byte-aligned row per
physical slot holding every group side by side::

    cols  0-3   quats (w, x, y, z)      -> one float4, renormalised inside Adam
    cols  4-6   means
    col   7     opacities (logit)
    cols  8-10  scales (log)
    cols 11-13  sh0
    cols 14-    shN (3 * ((d+1)^2 - 1) floats), then zero padding to stride % 4 == 0

``physical_pools[name]`` / ``adam_m_pools[name]`` / ``adam_v_pools[name]`` are
``[max_gaussians, dim]`` strided views of the slabs, so the reference's
per-group interface keeps working, while the hot path reads a Gaussian's
parameters as one contiguous row and updates all groups in one vectorised
Adam launch.  The indirection table (logical id -> physical slot, int32) and
the LIFO free list live on the device; nothing is ever reallocated.
"""
from __future__ import annotations

import time
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from . import _lib

GROUP_ORDER = ("quats", "means", "opacities", "scales", "sh0", "shN")


class SlabLayout:
    def __init__(self, sh_degree: int = 3, feature_dim: Optional[int] = None):
        if feature_dim is None:
            dims = {"quats": 4, "means": 3, "opacities": 1, "scales": 3, "sh0": 3,
                    "shN": ((sh_degree + 1) ** 2 - 1) * 3}
        else:
            dims = {"quats": 4, "means": 3, "opacities": 1, "scales": 3, "colors": 3, "features": int(feature_dim)}
        self.dims = dims
        self.offsets: Dict[str, int] = {}
        off = 0
        for name, d in dims.items():
            self.offsets[name] = off
            off += d
        self.ncols = off
        self.stride = (off + 3) // 4 * 4
        self.quat_col = self.offsets["quats"]
        self.color_col = self.offsets.get("sh0", self.offsets.get("colors"))
        self.color_cols = self.ncols - self.color_col

    def group_of_col(self) -> List[str]:
        out = []
        for name, d in self.dims.items():
            out += [name] * d
        return out

    def col_bounds(self) -> Tuple[np.ndarray, np.ndarray]:
        lo = np.full(self.ncols, -1e10, np.float32)
        hi = np.full(self.ncols, 1e10, np.float32)
        for c, name in enumerate(self.group_of_col()):
            if name == "scales":
                lo[c], hi[c] = -10.0, -2.0
            elif name == "opacities":
                lo[c], hi[c] = -5.0, 2.0
        return lo, hi

    def init_row(self) -> np.ndarray:
        """Initial parameter values of an unused slot (allocator.py:61-73)."""
        row = np.zeros(self.stride, np.float32)
        for c, name in enumerate(self.group_of_col()):
            if name == "scales":
                row[c] = -10.0
            elif name == "opacities":
                row[c] = -5.0
        return row

    def reset_row(self) -> np.ndarray:
        """Values written into pruned slots (allocator.py:248-256): same as init."""
        return self.init_row()


class PointerStableChunkedAllocator:
    def __init__(self, max_gaussians: int, sh_degree: int = 3, feature_dim: Optional[int] = None,
                 device: Optional[torch.device] = None, theta_storage: Optional[torch.Tensor] = None):
        """``theta_storage``: a caller-owned ``[max_gaussians, stride]`` float32
        device tensor to hold the parameter slab (e.g. symmetric memory with a
        multicast mapping for the sharded multi-GPU Adam)."""
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.max_gaussians = int(max_gaussians)
        self.sh_degree = sh_degree
        self.feature_dim = feature_dim
        self.layout = SlabLayout(sh_degree, feature_dim)
        self.realloc_count = 0
        self.allocation_latency_ms = 0.0
        self.fragmentation_ratio = 0.0
        self.sh0_dim = 3
        self.shN_dim = ((sh_degree + 1) ** 2 - 1) * 3

        L = self.layout
        if theta_storage is not None:
            if tuple(theta_storage.shape) != (self.max_gaussians, L.stride) or theta_storage.dtype != torch.float32:
                raise ValueError(f"theta_storage must be float32 [{self.max_gaussians}, {L.stride}]")
            self.theta = theta_storage
        else:
            self.theta = torch.empty((self.max_gaussians, L.stride), dtype=torch.float32, device=self.device)
        self.theta.copy_(torch.from_numpy(L.init_row()).to(self.device).expand_as(self.theta))
        self.adam_m = torch.zeros_like(self.theta)
        self.adam_v = torch.zeros_like(self.theta)
        self.physical_pools = {n: self.theta[:, o:o + L.dims[n]] for n, o in L.offsets.items()}
        self.adam_m_pools = {n: self.adam_m[:, o:o + L.dims[n]] for n, o in L.offsets.items()}
        self.adam_v_pools = {n: self.adam_v[:, o:o + L.dims[n]] for n, o in L.offsets.items()}

        # LIFO free list: the stack's top is at free_top; pops take free_stack[free_top - 1]
        self.free_stack = torch.arange(self.max_gaussians, dtype=torch.int32, device=self.device)
        self.free_top = self.max_gaussians
        self.active_mask = torch.zeros(self.max_gaussians, dtype=torch.int8, device=self.device)
        self.indirection_table = torch.zeros(0, dtype=torch.int32, device=self.device)
        self.indirection_mx = None
        self.cached_pointers = None
        self.cached_indices_addr = None
        self.grad2d = torch.zeros(self.max_gaussians, dtype=torch.float32, device=self.device)
        self.count = torch.zeros(self.max_gaussians, dtype=torch.float32, device=self.device)
        self._ws = None  # density-step buffers, allocated at the first density step

    # ------------------------------------------------------------------ properties / metrics
    @property
    def num_active(self) -> int:
        return int(self.indirection_table.shape[0])

    @property
    def free_slots(self) -> List[int]:
        """The free list, bottom to top (a host copy, for inspection)."""
        return self.free_stack[:self.free_top].tolist()

    def update_metrics(self) -> None:
        self.fragmentation_ratio = self.free_top / self.max_gaussians if self.max_gaussians > 0 else 0.0

    def update_cached_pointers(self) -> None:
        if self.num_active == 0:
            return
        self.indirection_mx = self.indirection_table
        self.cached_indices_addr = self.indirection_table.data_ptr()
        self.cached_pointers = {n: {"theta_addr": self.physical_pools[n].data_ptr(),
                                    "m_addr": self.adam_m_pools[n].data_ptr(),
                                    "v_addr": self.adam_v_pools[n].data_ptr()} for n in self.physical_pools}

    # ------------------------------------------------------------------ population
    def set_initial_gaussians(self, initial_params: Dict[str, object]) -> None:
        """allocator.py:124-147: pops ``n`` slots (max-1, max-2, ...) and writes the rows."""
        first = next(iter(initial_params.values()))
        n = int(first.shape[0])
        if n > self.max_gaussians:
            raise ValueError(f"initialization ({n}) exceeds pool capacity ({self.max_gaussians})")
        if n > self.free_top:
            raise MemoryError("not enough free slots")
        allocated = self.free_stack[self.free_top - n:self.free_top].flip(0).clone()
        self.free_top -= n
        self.active_mask[allocated.long()] = 1
        self.indirection_table = allocated
        rows = allocated.long()
        for name, val in initial_params.items():
            t = torch.as_tensor(np.asarray(val) if not isinstance(val, torch.Tensor) else val)
            t = t.to(self.device, torch.float32).reshape(n, -1)
            self.physical_pools[name].index_copy_(0, rows, t)
        self.update_metrics()
        self.update_cached_pointers()

    def get_active_parameters(self) -> Dict[str, torch.Tensor]:
        idx = self.indirection_table.long()
        return {n: p.index_select(0, idx) for n, p in self.physical_pools.items()}

    def get_active_adam_states(self) -> Tuple[Dict[str, torch.Tensor], Dict[str, torch.Tensor]]:
        idx = self.indirection_table.long()
        return ({n: p.index_select(0, idx) for n, p in self.adam_m_pools.items()},
                {n: p.index_select(0, idx) for n, p in self.adam_v_pools.items()})

    def update_physical_pool(self, param_name: str, active_updated_val: torch.Tensor) -> None:
        self.physical_pools[param_name].index_copy_(0, self.indirection_table.long(),
                                                    active_updated_val.to(torch.float32))

    def update_adam_states(self, m_dict: Dict[str, torch.Tensor], v_dict: Dict[str, torch.Tensor]) -> None:
        idx = self.indirection_table.long()
        for n in self.physical_pools:
            self.adam_m_pools[n].index_copy_(0, idx, m_dict[n])
            self.adam_v_pools[n].index_copy_(0, idx, v_dict[n])

    # ------------------------------------------------------------------ split / prune
    FLAG_PRUNE, FLAG_REFINE, FLAG_SPLIT = 1, 2, 4

    def workspace(self) -> Dict[str, object]:
        """Buffers of the density step, sized for the whole pool and allocated
        once (the first density step): the row flags, the compacted slot and row
        lists, two indirection-table buffers that alternate (the new table is
        compacted into the one the current table does not use, and the child
        slots are popped straight behind its kept entries), the compaction
        scratch and the counts with their pinned host copy."""
        if self._ws is None:
            lib = _lib.lib()
            M = self.max_gaussians
            dev = self.device

            def i32(n):
                return torch.empty(max(n, 1), dtype=torch.int32, device=dev)

            self._ws = {"flags": torch.empty(max(M, 1), dtype=torch.uint8, device=dev),
                        "prune": i32(M), "split": i32(M), "refine": i32(M), "tables": (i32(M), i32(M)),
                        "counts": i32(4), "counts_host": torch.empty(4, dtype=torch.int32, pin_memory=True),
                        "scratch": torch.empty(max(lib.gs_cull_scratch_bytes(M), 16), dtype=torch.uint8,
                                               device=dev)}
        return self._ws

    def _compact(self, flags: torch.Tensor, n: int, mask: int, value: int, gather: Optional[torch.Tensor],
                 out: torch.Tensor, count_at: int) -> None:
        lib = _lib.lib()
        ws = self.workspace()
        sb = ws["scratch"]
        _lib.check(lib.gs_compact_flags(flags.data_ptr(), n, mask, value, None if gather is None else gather.data_ptr(),
                                        out.data_ptr(), ws["counts"][count_at:].data_ptr(), sb.data_ptr(), sb.numel(),
                                        _lib.stream_ptr(self.device)), "gs_compact_flags")

    def apply_flags(self, flags: torch.Tensor, make_children) -> Tuple[int, int]:
        """The realloc-free density step of allocator.py:185-292 driven by
        per-row GS flags (bit 0 prune, bit 1 refine).  ``make_children(split_slots,
        refine_rows, n)`` returns the child rows ``(child1, child2)`` as
        ``[n, stride]`` tensors.  Slot order is the reference's: pruned slots are
        pushed in ascending logical order and children pop from the same end, so
        a child can land in a just-pruned slot and is then reset by the prune.
        Every buffer comes from ``workspace()``; the three counts come back to
        the host in one read."""
        start = time.perf_counter()
        lib = _lib.lib()
        st = _lib.stream_ptr(self.device)
        L = self.layout
        ws = self.workspace()
        n = self.num_active
        table = self.indirection_table
        t0, t1 = ws["tables"]
        dst = t1 if table.data_ptr() == t0.data_ptr() else t0  # the buffer the current table does not use
        P, R = self.FLAG_PRUNE, self.FLAG_REFINE
        prune_slots, split_slots, refine_rows = ws["prune"], ws["split"], ws["refine"]
        self._compact(flags, n, P, P, table, prune_slots, 0)
        self._compact(flags, n, R, R, table, split_slots, 1)
        self._compact(flags, n, R, R, None, refine_rows, 3)
        self._compact(flags, n, P, 0, table, dst, 2)  # kept entries, in order, at the head of the new table
        host = ws["counts_host"]
        host.copy_(ws["counts"], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        n_p, n_s, n_keep = [int(x) for x in host[:3].tolist()]
        # 1. prune: slots go back on the free list (allocator.py:209-211)
        if n_p:
            self.free_stack[self.free_top:self.free_top + n_p].copy_(prune_slots[:n_p])
            _lib.check(lib.gs_mark_slots(self.active_mask.data_ptr(), self.max_gaussians, prune_slots.data_ptr(), n_p,
                                         0, st), "active mask")
        self.free_top += n_p
        # 2. children pop from the same end (allocator.py:213-220), straight behind the kept entries
        if self.free_top < n_s:
            raise MemoryError(f"pool capacity reached: {self.free_top} free slots, {n_s} children requested")
        children = dst[n_keep:n_keep + n_s]
        _lib.check(lib.gs_free_pop_reversed(self.free_stack.data_ptr(), self.free_top, n_s, children.data_ptr(), st),
                   "free list pop")
        self.free_top -= n_s
        if n_s:
            _lib.check(lib.gs_mark_slots(self.active_mask.data_ptr(), self.max_gaussians, children.data_ptr(), n_s, 1,
                                         st), "active mask")
        # 3. rows: child 1 -> parent slot, child 2 -> popped slot, then the prune reset (allocator.py:229-273)
        if n_s:
            child1, child2 = make_children(split_slots[:n_s], refine_rows[:n_s], n_s)
            for slots, vals in ((split_slots, child1), (children, child2)):
                _lib.check(lib.gs_pool_write_rows(self.theta.data_ptr(), self.adam_m.data_ptr(),
                                                  self.adam_v.data_ptr(), L.stride, slots.data_ptr(), n_s,
                                                  vals.data_ptr(), vals.stride(0), None, self.grad2d.data_ptr(),
                                                  self.count.data_ptr(), st), "child rows")
        if n_p:
            _lib.check(lib.gs_pool_write_rows(self.theta.data_ptr(), self.adam_m.data_ptr(), self.adam_v.data_ptr(),
                                              L.stride, prune_slots.data_ptr(), n_p, None, 0,
                                              _lib.fptr(L.reset_row()), self.grad2d.data_ptr(),
                                              self.count.data_ptr(), st), "prune reset")
        # 4. indirection table: kept entries in order, then the children (allocator.py:275-281)
        self.indirection_table = dst[:n_keep + n_s]
        self.allocation_latency_ms = (time.perf_counter() - start) * 1000.0
        self.update_metrics()
        self.update_cached_pointers()
        return n_p, n_s

    def split_and_prune(self, prune_mask, split_mask, split_params: Dict[str, torch.Tensor]) -> Tuple[int, int]:
        """allocator.py:185-292 with the reference's arguments: boolean masks over
        the active rows and ``{name}_child1`` / ``{name}_child2`` values per group."""
        pm = torch.as_tensor(np.asarray(prune_mask) if not isinstance(prune_mask, torch.Tensor) else prune_mask,
                             device=self.device).to(torch.uint8)
        sm = torch.as_tensor(np.asarray(split_mask) if not isinstance(split_mask, torch.Tensor) else split_mask,
                             device=self.device).to(torch.uint8)
        n = self.num_active
        flags = self.workspace()["flags"][:max(n, 1)]
        flags[:n].copy_(pm * self.FLAG_PRUNE + sm * self.FLAG_REFINE)
        L = self.layout

        def make_children(split_slots, refine_rows, n):
            rows = []
            for suffix in ("_child1", "_child2"):
                buf = torch.zeros((n, L.stride), dtype=torch.float32, device=self.device)
                for name, off in L.offsets.items():
                    val = split_params[name + suffix]
                    val = torch.as_tensor(np.asarray(val) if not isinstance(val, torch.Tensor) else val)
                    buf[:, off:off + L.dims[name]] = val.to(self.device, torch.float32).reshape(n, -1)
                rows.append(buf)
            return rows[0], rows[1]

        return self.apply_flags(flags, make_children)

    # ------------------------------------------------------------------ opacity reset
    def reset_opacities(self, value: float = -4.59) -> None:
        """trainer.py:416-419: every slot's opacity logit set to ``value``."""
        lib = _lib.lib()
        _lib.check(lib.gs_fill_column(self.theta.data_ptr(), self.max_gaussians, self.layout.stride,
                                      self.layout.offsets["opacities"], value, _lib.stream_ptr(self.device)),
                   "opacity reset")

    def log_instrumentation_metrics(self) -> str:
        return (f"Active: {self.num_active} | Reallocs: {self.realloc_count} | "
                f"Latency: {self.allocation_latency_ms:.4f} ms | Fragmentation: {self.fragmentation_ratio * 100:.2f}%")
