"""Drop-in for the reference's native module ``mlx_gsplat_ext``
(src/mlx_extensions.cpp:238-248): the same two functions, the same argument
names and meaning, backed by ``libgsplat_b200.so``.

``launch_fused_adam_step`` takes device addresses (``tensor.data_ptr()``) of
caller-owned buffers — contiguous ``theta/m/v [max_gaussians, dim]`` pools,
dense ``g [num_active, dim]`` and int32 ``indices [num_active]`` — and updates
the pools in place, enqueued on the current CUDA stream.  Errors raise
``RuntimeError`` as the pybind11 module's ``std::runtime_error`` did.
"""
from __future__ import annotations

from . import _lib


def launch_fused_adam_step(theta_addr: int, g_addr: int, m_addr: int, v_addr: int, indices_addr: int,
                           max_gaussians: int, num_active: int, dim: int, lr: float, beta1: float, beta2: float,
                           eps: float, weight_decay: float, step: int, a_min: float, a_max: float) -> None:
    lib = _lib.lib()
    _lib.check(lib.gs_launch_fused_adam_step(theta_addr, g_addr, m_addr, v_addr, indices_addr, max_gaussians,
                                             num_active, dim, lr, beta1, beta2, eps, weight_decay, step, a_min, a_max,
                                             _lib.stream_ptr()), "launch_fused_adam_step")


def clear_buffer_cache() -> None:
    _lib.check(_lib.load().gs_clear_buffer_cache(), "clear_buffer_cache")
