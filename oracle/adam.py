"""Adam oracles — TEST INFRASTRUCTURE ONLY.

* ``fused_adam_a1`` — the fused Metal kernel's semantics (src/mlx_extensions.cpp:102-152),
  through the C restatement ``oracle/adam_a1.c`` (built by ``oracle/Makefile``).
* ``ref_fused_adam_a1`` — the reference's own MSL kernel text compiled for the CPU
  (``oracle/build_ref.py`` -> ``oracle/_ref/libref_adam.so``), when built.
* ``pure_adam_a2`` — the pure-MLX path (mlx_gsplat/optimizer.py:146-175): per-group
  ``lr_scales``, bias corrections in float64 Python scalars, no scrubbing, no clamp.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Dict, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

DEFAULT_LR_SCALES = {"means": 1.0, "scales": 2.0, "quats": 1.0, "opacities": 5.0, "sh0": 1.0, "shN": 0.05}


def _lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle_adam.so")
        if not os.path.exists(path):
            subprocess.check_call(["make", "-s", "-C", HERE])
        _LIB = ctypes.CDLL(path)
        f = _LIB.oracle_fused_adam_a1
        f.restype = None
        f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                              ctypes.c_float, ctypes.c_int, ctypes.c_float, ctypes.c_float]
    return _LIB


def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libref_adam.so"))


def _ref():
    global _REF
    if _REF is None:
        _REF = ctypes.CDLL(os.path.join(HERE, "_ref", "libref_adam.so"))
        f = _REF.ref_fused_adam_step
        f.restype = None
        f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_long, ctypes.c_int] + [ctypes.c_float] * 5 + \
                     [ctypes.c_int, ctypes.c_float, ctypes.c_float]
    return _REF


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _check(theta, g, m, v, idx):
    for a in (theta, g, m, v):
        assert a.dtype == np.float32 and a.flags.c_contiguous
    assert idx.dtype == np.int32 and idx.flags.c_contiguous


def fused_adam_a1(theta: np.ndarray, g: np.ndarray, m: np.ndarray, v: np.ndarray, indices: np.ndarray,
                  lr: float, beta1: float, beta2: float, eps: float, weight_decay: float, step: int,
                  a_min: float, a_max: float, num_active: Optional[int] = None) -> None:
    """In place on ``theta/m/v [max, dim]``; ``g [num_active, dim]``."""
    _check(theta, g, m, v, indices)
    dim = theta.shape[1]
    n = indices.shape[0] if num_active is None else num_active
    _lib().oracle_fused_adam_a1(_p(theta), _p(g), _p(m), _p(v), _p(indices), n, dim, dim, dim,
                                lr, beta1, beta2, eps, weight_decay, step, a_min, a_max)


def ref_fused_adam_a1(theta, g, m, v, indices, lr, beta1, beta2, eps, weight_decay, step, a_min, a_max,
                      num_active: Optional[int] = None) -> None:
    """The reference's MSL kernel text run on the CPU (same arguments as ``fused_adam_a1``)."""
    _check(theta, g, m, v, indices)
    dim = theta.shape[1]
    n = indices.shape[0] if num_active is None else num_active
    _ref().ref_fused_adam_step(_p(theta), _p(g), _p(m), _p(v), _p(indices), n, dim,
                               lr, beta1, beta2, eps, weight_decay, step, a_min, a_max)


def group_clamp(name: str):
    """optimizer.py:123-130."""
    if name == "scales":
        return -10.0, -2.0
    if name == "opacities":
        return -5.0, 2.0
    return -1e10, 1e10


def pure_adam_a2(params: Dict[str, np.ndarray], grads: Dict[str, np.ndarray], m: Dict[str, np.ndarray],
                 v: Dict[str, np.ndarray], t: int, lr: float, beta1: float = 0.9, beta2: float = 0.999,
                 eps: float = 1e-8, weight_decay: float = 0.0, lr_scales: Optional[Dict[str, float]] = None):
    """optimizer.py:146-175 (``t`` is the already-incremented step).  Returns new dicts."""
    f32 = np.float32
    lr_scales = DEFAULT_LR_SCALES if lr_scales is None else lr_scales
    bc1 = 1.0 - beta1 ** t
    bc2 = 1.0 - beta2 ** t
    out_p, out_m, out_v = {}, {}, {}
    for name, theta in params.items():
        g = grads.get(name)
        if g is None:
            out_p[name], out_m[name], out_v[name] = theta, m[name], v[name]
            continue
        g = g.astype(f32)
        if weight_decay != 0.0:
            g = g + f32(weight_decay) * theta
        m_new = f32(beta1) * m[name] + f32(1.0 - beta1) * g
        v_new = f32(beta2) * v[name] + f32(1.0 - beta2) * (g * g)
        scale = lr_scales.get(name, 1.0)
        step_size = f32((lr * scale) / bc1)
        denom = (np.sqrt(v_new) / f32(np.sqrt(bc2))) + f32(eps)
        out_p[name] = (theta - step_size * (m_new / denom)).astype(f32)
        out_m[name] = m_new.astype(f32)
        out_v[name] = v_new.astype(f32)
    return out_p, out_m, out_v
