"""ctypes binding of ``libgsplat_b200.so`` (C ABI in ``include/gsplat_b200.h``).

The product has no CPU fallback: every call goes to the CUDA library, and
loading fails loudly when the library is missing or CUDA is unavailable.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libgsplat_b200.so")

GS_OK, GS_ERR_INVALID, GS_ERR_CUDA, GS_ERR_CAPACITY = 0, 1, 2, 3
GS_ADAM_FUSED, GS_ADAM_PURE, GS_ADAM_EXACT = 0, 1, 0x100
GS_LOSS_NONE, GS_LOSS_L1_U8, GS_LOSS_L1_F32, GS_LOSS_MEAN = 0, 1, 2, 3
GS_SH_REFERENCE, GS_SH_FULL = 0, 1
GS_ROWS_ALL, GS_ROWS_SEEN, GS_ROWS_UNSEEN = 0, 1, 2

c_float_p = ctypes.POINTER(ctypes.c_float)
c_vp = ctypes.c_void_p
i64 = ctypes.c_int64
i32 = ctypes.c_int32


class GsGaussians(ctypes.Structure):
    _fields_ = [("means", c_vp), ("means_stride", i64),
                ("quats", c_vp), ("quats_stride", i64),
                ("scales", c_vp), ("scales_stride", i64),
                ("opac", c_vp), ("opac_stride", i64),
                ("colors", c_vp), ("colors_stride", i64),
                ("colors_dim", i32), ("colors_by_visible", i32),
                ("table", c_vp), ("sh_mode", i32)]


class GsGaussianGrads(ctypes.Structure):
    _fields_ = [("means", c_vp), ("means_stride", i64),
                ("quats", c_vp), ("quats_stride", i64),
                ("scales", c_vp), ("scales_stride", i64),
                ("opac", c_vp), ("opac_stride", i64),
                ("colors", c_vp), ("colors_stride", i64),
                ("colors_write", i32), ("colors_by_visible", i32), ("accumulate", i32),
                ("reg", ctypes.c_float), ("reg_color_cols", i32), ("reg_geometry", i32), ("count_col", i32)]


class GsCamera(ctypes.Structure):
    _fields_ = [("viewmat", ctypes.c_float * 16),
                ("fx", ctypes.c_float), ("fy", ctypes.c_float), ("cx", ctypes.c_float), ("cy", ctypes.c_float),
                ("width", i32), ("height", i32), ("render_width", i32), ("render_height", i32)]


class GsRasterSettings(ctypes.Structure):
    _fields_ = [("alpha_cutoff", ctypes.c_float), ("transmittance_min", ctypes.c_float), ("alpha_mask", i32)]


_SIGS = {
    "gs_last_error": (ctypes.c_char_p, []),
    "gs_abi_version": (ctypes.c_int, []),
    "gs_kernel_launches": (ctypes.c_ulonglong, []),
    "gs_launch_fused_adam_step": (ctypes.c_int, [ctypes.c_uint64] * 5 + [ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int,
                                                                        ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                                                        ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                                                        ctypes.c_float, ctypes.c_float, c_vp]),
    "gs_clear_buffer_cache": (ctypes.c_int, []),
    "gs_fused_adam_group": (ctypes.c_int, [c_vp] * 5 + [i64, ctypes.c_int, i64, i64] + [ctypes.c_double] * 3 +
                            [ctypes.c_float] * 2 + [ctypes.c_int] + [ctypes.c_float] * 4 + [ctypes.c_int, c_vp]),
    "gs_fused_adam_slab": (ctypes.c_int, [c_vp] * 5 + [i64, ctypes.c_int, i64, i64, c_float_p, c_float_p, c_float_p,
                                                       ctypes.c_int] + [ctypes.c_double] * 3 + [ctypes.c_float] * 2 +
                           [ctypes.c_int, ctypes.c_float, ctypes.c_int, c_vp, c_float_p, c_float_p,
                            ctypes.c_int, ctypes.c_int, c_float_p, ctypes.c_int, c_vp]),
    "gs_cull_scratch_bytes": (ctypes.c_size_t, [i64]),
    "gs_cull": (ctypes.c_int, [ctypes.POINTER(GsGaussians), i64, ctypes.POINTER(GsCamera), ctypes.c_float,
                               ctypes.c_float, ctypes.c_float, c_vp, c_vp, c_vp, ctypes.c_size_t, c_vp]),
    "gs_cull_noalloc": (ctypes.c_int, [ctypes.POINTER(GsGaussians), i64, ctypes.POINTER(GsCamera), ctypes.c_float,
                                       ctypes.c_float, ctypes.c_float, c_vp, c_vp, c_vp]),
    "gs_radix_sort_scratch_bytes": (ctypes.c_size_t, [i64]),
    "gs_radix_sort_pairs": (ctypes.c_int, [c_vp] * 4 + [i64, ctypes.c_int, ctypes.c_int, c_vp, ctypes.c_size_t, c_vp]),
    "gs_scan_scratch_bytes": (ctypes.c_size_t, [i64]),
    "gs_exclusive_scan_u32": (ctypes.c_int, [c_vp, c_vp, i64, c_vp, ctypes.c_size_t, c_vp]),
    "gs_project_forward": (ctypes.c_int, [ctypes.POINTER(GsGaussians), c_vp, i64, ctypes.POINTER(GsCamera),
                                          ctypes.POINTER(GsRasterSettings), c_vp, c_vp, c_vp, c_vp, c_vp]),
    "gs_bin_scratch_bytes": (ctypes.c_size_t, [i64]),
    "gs_bin_offsets_scratch_bytes": (ctypes.c_size_t, [i64]),
    "gs_bin_offsets": (ctypes.c_int, [c_vp, c_vp, i64, c_vp, c_vp, ctypes.c_size_t, c_vp]),
    "gs_bin_emit": (ctypes.c_int, [c_vp] * 4 + [i64, ctypes.POINTER(GsCamera), ctypes.POINTER(GsRasterSettings),
                                                c_vp, c_vp, i64, c_vp, c_vp, c_vp]),
    "gs_tile_ranges": (ctypes.c_int, [c_vp, i64, ctypes.c_int32, c_vp, c_vp]),
    "gs_tile_order": (ctypes.c_int, [c_vp, ctypes.c_int32, c_vp, c_vp]),
    "gs_render_forward": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, i64, ctypes.POINTER(GsCamera),
                                         ctypes.POINTER(GsRasterSettings), c_vp, c_vp, c_vp, c_vp, ctypes.c_int,
                                         c_vp, c_vp, c_vp]),
    "gs_render_pair_count": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, i64, ctypes.POINTER(GsCamera),
                                             ctypes.POINTER(GsRasterSettings), c_vp, c_vp]),
    "gs_fp32_peak_probe": (ctypes.c_int, [c_vp, i64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_double), c_vp]),
    "gs_apply_sorted_mask": (ctypes.c_int, [c_vp, c_vp, c_vp, i64, ctypes.POINTER(GsRasterSettings), c_vp]),
    "gs_render_backward": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, i64, ctypes.POINTER(GsCamera),
                                          ctypes.POINTER(GsRasterSettings), c_vp, c_vp, c_vp, ctypes.c_int, c_vp,
                                          c_vp, c_vp, c_vp, c_vp]),
    "gs_project_backward": (ctypes.c_int, [ctypes.POINTER(GsGaussians), c_vp, i64, ctypes.POINTER(GsCamera), c_vp,
                                           ctypes.POINTER(GsGaussianGrads), c_vp, c_vp, c_vp]),
    "gs_export_rows": (ctypes.c_int, [c_vp, i64, c_vp, i64] + [ctypes.c_int] * 6 + [c_vp, i64, c_vp]),
    "gs_l1_dssim_scratch_bytes": (ctypes.c_size_t, [i32, i32]),
    "gs_l1_dssim_loss": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int, i32, i32, ctypes.c_float, ctypes.c_float, c_vp,
                                        c_vp, c_vp, c_vp, ctypes.c_size_t, c_vp]),
    "gs_resize_bilinear": (ctypes.c_int, [c_vp, ctypes.c_int, i32, i32, i32, c_vp, i32, i32, c_vp]),
    "gs_group_barrier": (ctypes.c_int, [c_vp, i32, i32, i32, ctypes.c_uint32, c_vp, i64, c_vp]),
    "gs_rows_sum_multicast": (ctypes.c_int, [c_vp, i64, i64, i64, c_vp, c_vp]),
    "gs_fused_adam_slab_sharded": (ctypes.c_int, [c_vp] * 6 + [i64, ctypes.c_int, i64, i64, c_float_p, c_float_p,
                                                               ctypes.c_int] + [ctypes.c_double] * 3 +
                                   [ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_float, c_float_p,
                                    ctypes.c_int, ctypes.c_int, c_float_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    c_vp, c_vp]),
    "gs_compact_flags": (ctypes.c_int, [c_vp, i64, ctypes.c_uint8, ctypes.c_uint8, c_vp, c_vp, c_vp, c_vp,
                                        ctypes.c_size_t, c_vp]),
    "gs_densify_masks": (ctypes.c_int, [ctypes.POINTER(GsGaussians), c_vp, c_vp, i64] + [ctypes.c_float] * 5 +
                         [ctypes.c_int, c_vp, c_vp]),
    "gs_densify_children": (ctypes.c_int, [c_vp, i64, ctypes.c_int] + [c_vp] * 6 + [i64] + [ctypes.c_int] * 4 +
                            [c_vp, c_vp, c_vp]),
    "gs_pool_write_rows": (ctypes.c_int, [c_vp, c_vp, c_vp, i64, c_vp, i64, c_vp, i64, c_float_p, c_vp, c_vp, c_vp]),
    "gs_free_pop_reversed": (ctypes.c_int, [c_vp, i64, i64, c_vp, c_vp]),
    "gs_fill_rows": (ctypes.c_int, [c_vp, i64, i64, c_float_p, c_vp]),
    "gs_fill_column": (ctypes.c_int, [c_vp, i64, i64, ctypes.c_int, ctypes.c_float, c_vp]),
    "gs_mark_slots": (ctypes.c_int, [c_vp, i64, c_vp, i64, ctypes.c_int, c_vp]),
    "gs_copy_rows": (ctypes.c_int, [c_vp, i64, c_vp, c_vp, i64, c_vp, i64, ctypes.c_int, c_vp]),
}

_LIB: Optional[ctypes.CDLL] = None


class GsplatError(RuntimeError):
    pass


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library and declare every signature (no CUDA needed to load)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise GsplatError(f"{path} is missing: build it with `python -m mlx_gsplat_b200.build` "
                          "(there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in _SIGS.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    _LIB = lib
    return lib


def exported_names():
    return list(_SIGS.keys())


def lib() -> ctypes.CDLL:
    """The library, for compute calls: also requires a CUDA device."""
    if not torch.cuda.is_available():
        raise GsplatError("libgsplat_b200 needs a CUDA device; there is no CPU fallback")
    return load()


def check(status: int, what: str = "") -> None:
    if status == GS_OK:
        return
    msg = load().gs_last_error().decode(errors="replace")
    if status == GS_ERR_CAPACITY:
        raise MemoryError(f"{what}: {msg}")
    raise GsplatError(f"{what} failed ({status}): {msg}")


def stream_ptr(device: Optional[torch.device] = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def fptr(arr) -> "ctypes.Array":
    """Host float32 array argument."""
    vals = [float(x) for x in arr]
    return (ctypes.c_float * len(vals))(*vals)
