"""Pool allocator oracle — TEST INFRASTRUCTURE ONLY.

NumPy restatement of ``PointerStableChunkedAllocator`` (mlx_gsplat/allocator.py:8-292):

* pools per group ``[max, dim]`` for theta, m, v (:61-80); init theta:
  scales -10, opacities -5, the rest 0; moments 0;
* a LIFO free list ``list(range(max))`` (:46); ``set_initial_gaussians`` pops
  ``n`` slots (so slots ``max-1, max-2, ...``) (:124-147);
* ``split_and_prune`` (:185-292): pruned slots are pushed in ascending logical
  order, children pop from the same end, then per group: child 1 -> parent
  slot, child 2 -> popped slot, moments 0, and finally the prune reset
  (scales -10, opacities -5, others 0; moments 0), which overwrites any child
  that landed in a just-pruned slot; grad2d/count are zeroed at all touched
  slots; ``table = table[~prune] ++ children``; ``MemoryError`` when the free
  list is shorter than the number of splits.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import numpy as np

GROUPS_SH = ("means", "scales", "quats", "opacities", "sh0", "shN")


def group_dims(sh_degree: int) -> Dict[str, int]:
    return {"means": 3, "scales": 3, "quats": 4, "opacities": 1, "sh0": 3,
            "shN": ((sh_degree + 1) ** 2 - 1) * 3}


def reset_value(name: str) -> float:
    return -10.0 if name == "scales" else (-5.0 if name == "opacities" else 0.0)


class PoolOracle:
    def __init__(self, max_gaussians: int, sh_degree: int = 3):
        self.max_gaussians = max_gaussians
        self.sh_degree = sh_degree
        self.dims = group_dims(sh_degree)
        self.pools = {n: np.full((max_gaussians, d), reset_value(n) if n in ("scales", "opacities") else 0.0,
                                 np.float32) for n, d in self.dims.items()}
        self.m = {n: np.zeros((max_gaussians, d), np.float32) for n, d in self.dims.items()}
        self.v = {n: np.zeros((max_gaussians, d), np.float32) for n, d in self.dims.items()}
        self.free_slots: List[int] = list(range(max_gaussians))
        self.active_mask = np.zeros(max_gaussians, np.int8)
        self.table = np.zeros(0, np.int32)
        self.grad2d = np.zeros(max_gaussians, np.float32)
        self.count = np.zeros(max_gaussians, np.float32)

    @property
    def num_active(self) -> int:
        return int(self.table.shape[0])

    def set_initial_gaussians(self, init: Dict[str, np.ndarray]) -> None:
        n = init["means"].shape[0]
        if n > self.max_gaussians:
            raise ValueError("initialization exceeds pool capacity")
        allocated = [self.free_slots.pop() for _ in range(n)]
        self.active_mask[allocated] = 1
        self.table = np.array(allocated, np.int32)
        for name, val in init.items():
            self.pools[name][allocated] = np.asarray(val, np.float32).reshape(n, -1)

    def active(self, name: str) -> np.ndarray:
        return self.pools[name][self.table]

    def split_and_prune(self, prune_mask: np.ndarray, split_mask: np.ndarray,
                        split_params: Dict[str, np.ndarray]) -> Tuple[int, int]:
        prune_idx = np.where(prune_mask)[0]
        split_idx = np.where(split_mask)[0]
        prune_slots = self.table[prune_idx]
        split_slots = self.table[split_idx]
        n_p, n_s = len(prune_slots), len(split_slots)
        self.active_mask[prune_slots] = 0
        self.free_slots.extend(prune_slots.tolist())
        if len(self.free_slots) < n_s:
            # the reference raises after pushing the pruned slots (allocator.py:211-217)
            raise MemoryError("pool capacity reached")
        children = np.array([self.free_slots.pop() for _ in range(n_s)], np.int32)
        self.active_mask[children] = 1
        for name in self.pools:
            pool, m, v = self.pools[name], self.m[name], self.v[name]
            if n_s > 0:
                pool[split_slots] = split_params[f"{name}_child1"]
                m[split_slots] = 0.0
                v[split_slots] = 0.0
                pool[children] = split_params[f"{name}_child2"]
                m[children] = 0.0
                v[children] = 0.0
            if n_p > 0:
                pool[prune_slots] = reset_value(name)
                m[prune_slots] = 0.0
                v[prune_slots] = 0.0
        for slots in (split_slots, children, prune_slots):
            if len(slots):
                self.grad2d[slots] = 0.0
                self.count[slots] = 0.0
        keep = ~np.asarray(prune_mask, bool)
        new_table = self.table[keep]
        if n_s > 0:
            new_table = np.concatenate([new_table, children])
        self.table = new_table.astype(np.int32)
        return n_p, n_s

    def free_list_array(self) -> np.ndarray:
        return np.array(self.free_slots, np.int32)
