"""``FusedMLXAdam`` (mlx_gsplat/optimizer.py:11-175) on B200.

* ``step(..., use_metal_fusion=True, physical_pools=...)`` — the fused path the
  trainer uses: in place on the pools through the indirection table, with the
  Metal kernel's semantics (NaN scrubbing, per-group clamps, float32 bias
  corrections, no ``lr_scales``), one launch per group as the reference does.
* ``step(..., use_metal_fusion=False)`` — the pure path (optimizer.py:146-175):
  out of place, ``lr_scales`` applied, float64 bias corrections, no scrubbing
  or clamping.  It runs on the GPU too (there is no CPU fallback).
* ``step_slab`` — all groups of a pooled slab in one float4-vectorised launch,
  with the trainer's quaternion renormalisation fused in.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import numpy as np
import torch

from . import _lib

CLAMPS = {"scales": (-10.0, -2.0), "opacities": (-5.0, 2.0)}


def group_clamp(name: str) -> Tuple[float, float]:
    return CLAMPS.get(name, (-1e10, 1e10))


class FusedMLXAdam:
    def __init__(self, lr: float = 0.001, betas: Tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, lr_scales: Optional[Dict[str, float]] = None):
        self.lr = lr
        self.beta1, self.beta2 = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.t = 0
        self.lr_scales = lr_scales or {"means": 1.0, "scales": 2.0, "quats": 1.0, "opacities": 5.0, "sh0": 1.0,
                                       "shN": 0.05}

    # ------------------------------------------------------------------ reference API
    def step(self, active_params: Dict[str, torch.Tensor], grads: Dict[str, torch.Tensor],
             active_m: Dict[str, torch.Tensor], active_v: Dict[str, torch.Tensor], use_metal_fusion: bool = False,
             physical_pools: Optional[Dict[str, torch.Tensor]] = None,
             adam_m_pools: Optional[Dict[str, torch.Tensor]] = None,
             adam_v_pools: Optional[Dict[str, torch.Tensor]] = None, indirection_table=None,
             cached_pointers: Optional[Dict[str, Dict[str, int]]] = None, cached_indices_addr: Optional[int] = None,
             grad_scale: float = 1.0):
        self.t += 1
        lib = _lib.lib()
        st = _lib.stream_ptr()
        if use_metal_fusion and physical_pools is not None:
            keep = None
            if cached_indices_addr is not None:
                idx_addr = cached_indices_addr
            elif indirection_table is not None:
                keep = torch.as_tensor(np.asarray(indirection_table.cpu() if isinstance(indirection_table, torch.Tensor)
                                                  else indirection_table), dtype=torch.int32)
                keep = keep.to(next(iter(physical_pools.values())).device)
                idx_addr = keep.data_ptr()
            else:
                raise ValueError("Neither cached_indices_addr nor indirection_table provided for the fused optimizer.")
            for name in active_params.keys():
                g = grads.get(name)
                if g is None:
                    continue
                pool = physical_pools[name]
                if cached_pointers is not None and name in cached_pointers:
                    ptrs = cached_pointers[name]
                    th, m, v = ptrs["theta_addr"], ptrs["m_addr"], ptrs["v_addr"]
                else:
                    th, m, v = pool.data_ptr(), adam_m_pools[name].data_ptr(), adam_v_pools[name].data_ptr()
                dim = int(pool.shape[1])
                n = int(len(indirection_table)) if indirection_table is not None else int(active_params[name].shape[0])
                g2 = g.reshape(g.shape[0], -1)
                if g2.stride(1) != 1:
                    g2 = g2.contiguous()
                lo, hi = group_clamp(name)
                _lib.check(lib.gs_fused_adam_group(th, g2.data_ptr(), m, v, idx_addr, n, dim, pool.stride(0),
                                                   g2.stride(0), self.lr, self.beta1, self.beta2, self.eps,
                                                   self.weight_decay, self.t, lo, hi, 1.0, grad_scale,
                                                   _lib.GS_ADAM_FUSED, st), "fused adam (" + name + ")")
            del keep
            return active_params, active_m, active_v

        up, um, uv = {}, {}, {}
        for name, theta in active_params.items():
            g = grads.get(name)
            if g is None:
                up[name], um[name], uv[name] = theta, active_m[name], active_v[name]
                continue
            th = theta.detach().clone().contiguous()
            m = active_m[name].detach().clone().contiguous()
            v = active_v[name].detach().clone().contiguous()
            g2 = g.detach().contiguous()
            n, dim = int(th.shape[0]), int(th.reshape(th.shape[0], -1).shape[1])
            idx = torch.arange(n, dtype=torch.int32, device=th.device)
            _lib.check(lib.gs_fused_adam_group(th.data_ptr(), g2.data_ptr(), m.data_ptr(), v.data_ptr(),
                                               idx.data_ptr(), n, dim, dim, dim, self.lr, self.beta1, self.beta2,
                                               self.eps, self.weight_decay, self.t, -1e10, 1e10,
                                               float(self.lr_scales.get(name, 1.0)), grad_scale, _lib.GS_ADAM_PURE,
                                               st), "pure adam (" + name + ")")
            up[name], um[name], uv[name] = th, m, v
        return up, um, uv

    # ------------------------------------------------------------------ pooled fast path
    def step_slab(self, theta: torch.Tensor, g: torch.Tensor, m: torch.Tensor, v: torch.Tensor,
                  table: torch.Tensor, num_active: int, ncols: int, col_lo, col_hi, quat_col: int = -1,
                  grad_scale: float = 1.0, pure: bool = False, col_lr_scale=None, visible_words: Optional[int] = None,
                  unseen_grad=None, exact: bool = False, grad_bias=None, g_cols: Optional[int] = None,
                  count_col: int = 0, count_coef=None, row_select: int = 0, advance: bool = True) -> None:
        """One launch over every group of a ``[max, stride]`` slab (fused semantics).
        With ``visible_words`` (device address of the cull's visibility bitmask) rows
        the bitmask marks unseen take ``unseen_grad`` (ncols floats) as their gradient
        instead of reading ``g``.  The step uses the hardware approximate square
        root and reciprocal (relative error below 1e-6) unless ``exact``.
        ``grad_bias`` (ncols floats) is added to every row's gradient before
        ``grad_scale``.  Narrow gradient rows: only the first ``g_cols`` columns
        of ``g`` hold gradients; column c >= g_cols is ``g[count_col] *
        count_coef[c]`` (the regulariser of each view that saw the row).
        ``row_select`` (with ``visible_words``) updates only the seen
        (``GS_ROWS_SEEN``) or unseen (``GS_ROWS_UNSEEN``) rows; the second
        launch of such a pair passes ``advance=False`` to keep the step count."""
        if advance:
            self.t += 1
        lib = _lib.lib()
        _lib.check(lib.gs_fused_adam_slab(theta.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(),
                                          table.data_ptr(), num_active, ncols, theta.stride(0), g.stride(0),
                                          _lib.fptr(col_lo), _lib.fptr(col_hi),
                                          None if col_lr_scale is None else _lib.fptr(col_lr_scale), quat_col,
                                          self.lr, self.beta1, self.beta2, self.eps, self.weight_decay, self.t,
                                          grad_scale, (_lib.GS_ADAM_PURE if pure else _lib.GS_ADAM_FUSED) |
                                          (_lib.GS_ADAM_EXACT if exact else 0),
                                          visible_words, None if unseen_grad is None else _lib.fptr(unseen_grad),
                                          None if grad_bias is None else _lib.fptr(grad_bias),
                                          ncols if g_cols is None else int(g_cols), int(count_col),
                                          None if count_coef is None else _lib.fptr(count_coef), int(row_select),
                                          _lib.stream_ptr(theta.device)), "fused adam (slab)")

    def step_slab_sharded(self, theta: torch.Tensor, theta_multicast: int, g_multicast: int, g_stride: int,
                          m: torch.Tensor, v: torch.Tensor, table: torch.Tensor, num_active: int, ncols: int,
                          col_lo, col_hi, rank: int, world: int, hot_cols: int, quat_col: int = -1,
                          grad_scale: float = 1.0, grad_bias=None, g_cols: Optional[int] = None, count_col: int = 0,
                          count_coef=None, error_flag: Optional[int] = None) -> None:
        """``step_slab`` for one GPU of a multicast group: the rows whose slot
        this GPU owns (slot % world == rank), their gradient summed over the
        group through the multicast address ``g_multicast``, the first
        ``hot_cols`` columns of the new parameters stored to every GPU through
        ``theta_multicast`` (``gs_fused_adam_slab_sharded``).  ``error_flag``:
        device address of the group barriers' error flag; once a barrier wait
        has given up the update is skipped on the GPU."""
        self.t += 1
        lib = _lib.lib()
        _lib.check(lib.gs_fused_adam_slab_sharded(theta.data_ptr(), theta_multicast, g_multicast, m.data_ptr(),
                                                  v.data_ptr(), table.data_ptr(), num_active, ncols, theta.stride(0),
                                                  g_stride, _lib.fptr(col_lo), _lib.fptr(col_hi), quat_col, self.lr,
                                                  self.beta1, self.beta2, self.eps, self.weight_decay, self.t,
                                                  grad_scale, None if grad_bias is None else _lib.fptr(grad_bias),
                                                  ncols if g_cols is None else int(g_cols), int(count_col),
                                                  None if count_coef is None else _lib.fptr(count_coef), rank, world,
                                                  hot_cols, error_flag, _lib.stream_ptr(theta.device)),
                   "sharded fused adam")
