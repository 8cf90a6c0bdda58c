"""Cull and differentiable rasterization on B200, with the reference's entry
points (``mlx_gsplat/rendering.py``): ``frustum_culling_mlx`` and
``rasterize_gaussians_mlx`` keep their names, arguments and return shapes.

Underneath, the dense pixel-chunked evaluator of the reference
(rendering.py:246-308) is replaced by a 16x16-tile rasterizer:

    cull (bitmask + ordered compaction)
    -> projection + tile count per visible Gaussian
    -> stable radix sort of depth keys
    -> per-Gaussian entry offsets (scan, in depth order) -> tile binning
    -> stable radix sort of the entries by tile -> per-tile ranges
    -> compositing forward (shared-memory staged, warp-level early stop)
    -> compositing backward (back-to-front, warp-reduced vector atomics)
    -> projection backward (chain rule to the Gaussian parameters)

Parity with the dense evaluator: a Gaussian is binned into a tile only when
some pixel centre of that tile can see ``alpha >= alpha_cutoff`` and a pixel
stops once its transmittance is below ``transmittance_min``; at the defaults
the contribution left out is far below 1e-4 per pixel.

All tensors are CUDA float32; there is no CPU fallback.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import GsCamera, GsGaussianGrads, GsGaussians, GsRasterSettings, check

TILE = 16


@dataclass
class RasterSettings:
    alpha_cutoff: float = 1e-7
    transmittance_min: float = 1e-6

    def cstruct(self, alpha_mask: bool = False) -> GsRasterSettings:
        return GsRasterSettings(self.alpha_cutoff, self.transmittance_min, int(alpha_mask))


DEFAULT_SETTINGS = RasterSettings()


def _host(x) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        return x.detach().to("cpu", torch.float32).numpy()
    return np.asarray(x, np.float32)


def camera_struct(viewmat, K, width: int, height: int, render_width: int, render_height: int) -> GsCamera:
    vm = _host(viewmat).reshape(4, 4)
    Kh = _host(K)
    cam = GsCamera()
    for i, v in enumerate(vm.reshape(-1)):
        cam.viewmat[i] = float(v)
    cam.fx, cam.fy, cam.cx, cam.cy = float(Kh[0, 0]), float(Kh[1, 1]), float(Kh[0, 2]), float(Kh[1, 2])
    cam.width, cam.height = int(width), int(height)
    cam.render_width, cam.render_height = int(render_width), int(render_height)
    return cam


def num_tiles(render_width: int, render_height: int) -> Tuple[int, int]:
    return (render_width + TILE - 1) // TILE, (render_height + TILE - 1) // TILE


def _rows(t: Optional[torch.Tensor], cols: int, name: str):
    if t is None:
        return None, 0
    if not t.is_cuda or t.dtype != torch.float32:
        raise TypeError(f"{name} must be a CUDA float32 tensor")
    t2 = t.reshape(t.shape[0], -1) if t.dim() != 2 else t
    if t2.shape[1] < cols or (t2.shape[0] > 1 and t2.stride(1) != 1) or (t2.shape[1] > 1 and t2.stride(1) != 1):
        raise ValueError(f"{name}: need rows of >= {cols} contiguous floats, got shape {tuple(t.shape)}")
    return t2.data_ptr(), t2.stride(0)


SH_MODES = {"reference": _lib.GS_SH_REFERENCE, "full": _lib.GS_SH_FULL}


def sh_mode_code(sh_mode) -> int:
    """``"reference"`` (mlx_gsplat/rendering.py:229-244: SH degree <= 1) or
    ``"full"`` (real SH up to the degree the colour rows hold, at most 3)."""
    if isinstance(sh_mode, str):
        if sh_mode not in SH_MODES:
            raise ValueError(f"sh_mode must be one of {sorted(SH_MODES)}, got {sh_mode!r}")
        return SH_MODES[sh_mode]
    return int(sh_mode)


def gaussians_struct(means, quats=None, scales=None, opacities=None, colors=None, colors_dim: Optional[int] = None,
                     colors_by_visible: bool = False, table: Optional[torch.Tensor] = None,
                     sh_mode="reference") -> GsGaussians:
    g = GsGaussians()
    g.means, g.means_stride = _rows(means, 3, "means")
    g.quats, g.quats_stride = _rows(quats, 4, "quats")
    g.scales, g.scales_stride = _rows(scales, 3, "scales")
    g.opac, g.opac_stride = _rows(opacities, 1, "opacities")
    g.colors, g.colors_stride = _rows(colors, 3, "colors")
    if colors is not None:
        g.colors_dim = int(colors_dim if colors_dim is not None else colors.reshape(colors.shape[0], -1).shape[1])
    g.colors_by_visible = int(colors_by_visible)
    g.table = None if table is None else table.data_ptr()
    g.sh_mode = sh_mode_code(sh_mode)
    return g


def grads_struct(means=None, quats=None, scales=None, opacities=None, colors=None, colors_write: int = 0,
                 colors_by_visible: bool = False, accumulate: bool = True, reg: float = 0.0,
                 reg_color_cols: int = 0, reg_geometry: bool = True, count_col: int = 0) -> GsGaussianGrads:
    o = GsGaussianGrads()
    o.means, o.means_stride = _rows(means, 3, "grad means")
    o.quats, o.quats_stride = _rows(quats, 4, "grad quats")
    o.scales, o.scales_stride = _rows(scales, 3, "grad scales")
    o.opac, o.opac_stride = _rows(opacities, 1, "grad opacities")
    o.colors, o.colors_stride = _rows(colors, 0, "grad colors")
    o.colors_write = int(colors_write)
    o.colors_by_visible = int(colors_by_visible)
    o.accumulate = int(accumulate)
    o.reg = float(reg)
    o.reg_color_cols = int(reg_color_cols)
    o.reg_geometry = int(bool(reg_geometry))
    o.count_col = int(count_col)
    return o


def _scratch(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


def _i32(n: int, device) -> torch.Tensor:
    return torch.empty(max(int(n), 1), dtype=torch.int32, device=device)


# ----------------------------------------------------------------------------- target image
def bilinear_resize_mlx(img: torch.Tensor, H_out: int, W_out: int) -> torch.Tensor:
    """mlx_gsplat/rendering.py:6-38 on the GPU (``gs_resize_bilinear``): HWC
    float32 ``img`` resized to ``[H_out, W_out, C]``, bit-identical to the
    reference.  A uint8 ``img`` is taken as ``img / 255.0`` first (the
    trainer's target scaling), so a cached uint8 image becomes the float
    target in one pass.  The result is not differentiable (the trainer resizes
    targets only)."""
    if not img.is_cuda or img.dtype not in (torch.uint8, torch.float32) or img.dim() != 3:
        raise TypeError("bilinear_resize_mlx: img must be a CUDA uint8 or float32 HWC tensor")
    H, W, C = img.shape
    src = img.contiguous()
    out = torch.empty((int(H_out), int(W_out), C), dtype=torch.float32, device=img.device)
    check(_lib.lib().gs_resize_bilinear(src.data_ptr(), int(src.dtype == torch.uint8), W, H, C, out.data_ptr(),
                                        int(W_out), int(H_out), _lib.stream_ptr(img.device)), "gs_resize_bilinear")
    return out


# ----------------------------------------------------------------------------- cull
def cull_ids(g: GsGaussians, n: int, cam: GsCamera, device, near_plane: float = 0.01, far_plane: float = 1e10,
             opacity_threshold: float = -5.3, sync: bool = True, return_scratch: bool = False):
    """Ascending ids passing the cull; returns ``(ids_buffer, count_tensor, V or None)``
    (and the scratch buffer, whose first words are the visibility bitmask, when
    ``return_scratch``)."""
    lib = _lib.lib()
    ids = _i32(n, device)
    cnt = _i32(1, device)
    sb = lib.gs_cull_scratch_bytes(n)
    scratch = _scratch(sb, device)
    check(lib.gs_cull(g, n, cam, near_plane, far_plane, opacity_threshold, ids.data_ptr(), cnt.data_ptr(),
                      scratch.data_ptr(), scratch.numel(), _lib.stream_ptr(device)), "gs_cull")
    V = int(cnt.item()) if sync else None
    if return_scratch:
        return ids, cnt, V, scratch
    return ids, cnt, V


def frustum_culling_mlx(means, quats, scales, viewmat, K, width: int, height: int, near_plane: float = 0.01,
                        far_plane: float = 1e10, opacities=None, opacity_threshold: float = -5.3,
                        empty_quirk: bool = False) -> torch.Tensor:
    """mlx_gsplat/rendering.py:41-94.  Returns the ascending int32 ids of the
    Gaussians inside the frustum (with the 50 px tolerance) whose opacity
    logit is >= ``opacity_threshold``.  Like the reference this reads the
    count back to the host.  When nothing is visible the result is empty;
    ``empty_quirk=True`` instead returns the reference's ``sorted[-0:]``
    result (all N entries, each -1)."""
    n = int(means.shape[0])
    device = means.device
    g = gaussians_struct(means, opacities=opacities)
    cam = camera_struct(viewmat, K, width, height, width, height)
    ids, _, V = cull_ids(g, n, cam, device, near_plane, far_plane, opacity_threshold)
    if V == 0 and empty_quirk:
        return torch.full((n,), -1, dtype=torch.int32, device=device)
    return ids[:V]


# ----------------------------------------------------------------------------- tile pipeline
class TileFrame:
    """Forward state of one view (kept for the backward)."""

    def __init__(self):
        self.V = 0
        self.K = 0
        self.tile_order = None  # dispatch order of the compositing CTAs (None: tile index order)


def render_forward(g: GsGaussians, ids: torch.Tensor, V: int, cam: GsCamera, settings: RasterSettings,
                   device, loss_mode: int = _lib.GS_LOSS_NONE, target: Optional[torch.Tensor] = None,
                   out_color: Optional[torch.Tensor] = None, timer=None, v_count: Optional[torch.Tensor] = None,
                   k_hint: int = 0, mask: Optional[torch.Tensor] = None) -> TileFrame:
    """The forward of one view.  With ``v_count`` (the cull's device count, not
    yet read back) ``V`` is an upper bound of the visible count: every
    per-view buffer is allocated before the count is read, and the tile-entry
    buffers before the entry count is read (``k_hint`` entries, enlarged only
    when a view has more), so the host goes from each read-back straight to
    the next kernel launch.  ``mask`` (float32 [V] in [0, 1], device): the
    reference's alpha mask, entry j multiplying the clipped alpha of the j-th
    visible Gaussian in depth order (mlx_gsplat/rendering.py:289-290)."""
    lib = _lib.lib()
    st = _lib.stream_ptr(device)
    rs = settings.cstruct(alpha_mask=mask is not None)
    RW, RH = cam.render_width, cam.render_height
    tx, ty = num_tiles(RW, RH)
    T = tx * ty
    f = TileFrame()
    Vb = int(V)  # buffer bound
    f.cam, f.rs, f.ids, f.loss_mode, f.target = cam, rs, ids, loss_mode, target
    f.color = out_color if out_color is not None else torch.empty((RH, RW, 3), dtype=torch.float32, device=device)
    f.alpha = torch.empty((RH, RW, 1), dtype=torch.float32, device=device)
    f.final_T = torch.empty((RH, RW), dtype=torch.float32, device=device)
    f.n_contrib = torch.empty((RH, RW), dtype=torch.int32, device=device)
    f.loss_partials = torch.empty(T, dtype=torch.float32, device=device) if loss_mode != _lib.GS_LOSS_NONE else None
    f.splats = torch.empty((max(Vb, 1), 12), dtype=torch.float32, device=device)
    f.ranges = torch.empty((T, 2), dtype=torch.int32, device=device)
    if Vb > 0:
        depth_keys = _i32(Vb, device)
        tile_counts = _i32(Vb, device)
        bin_scratch = _scratch(lib.gs_bin_scratch_bytes(Vb), device)  # binning state for gs_bin_emit
        keys_sorted = _i32(Vb, device)
        order = _i32(Vb, device)
        sb = _scratch(lib.gs_radix_sort_scratch_bytes(Vb), device)
        offsets = _i32(Vb + 1, device)
        ob = _scratch(lib.gs_bin_offsets_scratch_bytes(Vb), device)
    V = int(v_count.item()) if v_count is not None else Vb
    f.V = V
    if V > 0:
        check(lib.gs_project_forward(g, ids.data_ptr(), V, cam, rs, f.splats.data_ptr(), depth_keys.data_ptr(),
                                     tile_counts.data_ptr(), bin_scratch.data_ptr(), st), "gs_project_forward")
        if timer:
            timer.mark("project_fwd")
        check(lib.gs_radix_sort_pairs(depth_keys.data_ptr(), None, keys_sorted.data_ptr(),
                                      order.data_ptr(), V, 0, 32, sb.data_ptr(), sb.numel(), st), "depth sort")
        if mask is not None:
            check(lib.gs_apply_sorted_mask(f.splats.data_ptr(), order.data_ptr(), mask.data_ptr(), V, rs, st),
                  "gs_apply_sorted_mask")
        check(lib.gs_bin_offsets(order.data_ptr(), tile_counts.data_ptr(), V, offsets.data_ptr(), ob.data_ptr(),
                                 ob.numel(), st), "gs_bin_offsets")
        if timer:
            timer.mark("depth_sort+offsets")

        def entry_buffers(cap):
            flag = torch.zeros(1, dtype=torch.int32, device=device)
            return (_i32(cap, device), _i32(cap, device), _i32(cap, device), _i32(cap, device),
                    _scratch(lib.gs_radix_sort_scratch_bytes(cap), device), flag)

        kcap = int(k_hint)
        bufs = entry_buffers(kcap) if kcap > 0 else None
        K = int(offsets[V].item())
        f.K = K
        f.order = order
        if K > 0:
            if bufs is None or K > kcap:
                bufs = entry_buffers(K)
            keys, vals, f.tile_keys, f.entry_vals, sb2, flag = bufs
            check(lib.gs_bin_emit(f.splats.data_ptr(), order.data_ptr(), offsets.data_ptr(), tile_counts.data_ptr(),
                                  V, cam, rs, keys.data_ptr(), vals.data_ptr(), K, flag.data_ptr(),
                                  bin_scratch.data_ptr(), st), "gs_bin_emit")
            tile_bits = max(1, int(T).bit_length())  # 2**bits - 1 >= T: the emit sentinel sorts last
            check(lib.gs_radix_sort_pairs(keys.data_ptr(), vals.data_ptr(), f.tile_keys.data_ptr(),
                                          f.entry_vals.data_ptr(), K, 0, tile_bits, sb2.data_ptr(), sb2.numel(), st),
                  "tile sort")
            check(lib.gs_tile_ranges(f.tile_keys.data_ptr(), K, T, f.ranges.data_ptr(), st), "gs_tile_ranges")
            # heaviest tiles first: the compositing launches then end evenly across the SMs
            f.tile_order = _i32(T, device)
            check(lib.gs_tile_order(f.ranges.data_ptr(), T, f.tile_order.data_ptr(), st), "gs_tile_order")
            if timer:
                timer.mark("bin+tile_sort")
        else:
            f.entry_vals = _i32(1, device)
            f.ranges.zero_()
    else:
        f.entry_vals = _i32(1, device)
        f.ranges.zero_()
    tptr = None if target is None else target.data_ptr()
    check(lib.gs_render_forward(f.ranges.data_ptr(), _lib.ptr(f.tile_order), f.entry_vals.data_ptr(),
                                f.splats.data_ptr(), V, cam, rs,
                                f.color.data_ptr(), f.alpha.data_ptr(), f.final_T.data_ptr(), f.n_contrib.data_ptr(),
                                loss_mode, tptr, None if f.loss_partials is None else f.loss_partials.data_ptr(), st),
          "gs_render_forward")
    if timer:
        timer.mark("render_fwd")
    return f


def render_backward(f: TileFrame, g: GsGaussians, out: GsGaussianGrads, device,
                    dL_dcolor: Optional[torch.Tensor] = None, dL_dalpha: Optional[torch.Tensor] = None,
                    grad2d: Optional[torch.Tensor] = None, count: Optional[torch.Tensor] = None,
                    timer=None) -> None:
    lib = _lib.lib()
    st = _lib.stream_ptr(device)
    if f.V == 0:
        return
    f.splat_grads = torch.zeros((f.V, 12), dtype=torch.float32, device=device)
    tptr = None if f.target is None else f.target.data_ptr()
    check(lib.gs_render_backward(f.ranges.data_ptr(), _lib.ptr(f.tile_order), f.entry_vals.data_ptr(),
                                 f.splats.data_ptr(), f.V, f.cam, f.rs,
                                 f.color.data_ptr(), f.final_T.data_ptr(), f.n_contrib.data_ptr(), f.loss_mode, tptr,
                                 None if dL_dcolor is None else dL_dcolor.data_ptr(),
                                 None if dL_dalpha is None else dL_dalpha.data_ptr(), f.splat_grads.data_ptr(), st),
          "gs_render_backward")
    if timer:
        timer.mark("render_bwd")
    check(lib.gs_project_backward(g, f.ids.data_ptr(), f.V, f.cam, f.splat_grads.data_ptr(), out,
                                  None if grad2d is None else grad2d.data_ptr(),
                                  None if count is None else count.data_ptr(), st), "gs_project_backward")
    if timer:
        timer.mark("project_bwd")


# ----------------------------------------------------------------------------- autograd entry
class _RasterizeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means, quats, scales, opacities, colors, ids, cam, settings, colors_by_visible, sh_mode,
                mask=None):
        device = means.device
        g = gaussians_struct(means, quats, scales, opacities, colors, colors_by_visible=colors_by_visible,
                             sh_mode=sh_mode)
        V = int(ids.shape[0])
        f = render_forward(g, ids, V, cam, settings, device, mask=mask)
        ctx.frame = f
        ctx.g = g
        ctx.colors_by_visible = colors_by_visible
        ctx.save_for_backward(means, quats, scales, opacities, colors, ids)
        return f.color, f.alpha

    @staticmethod
    def backward(ctx, dC, dA):
        means, quats, scales, opacities, colors, ids = ctx.saved_tensors
        device = means.device
        gm = torch.zeros_like(means, memory_format=torch.contiguous_format)
        gq = torch.zeros_like(quats, memory_format=torch.contiguous_format)
        gsc = torch.zeros_like(scales, memory_format=torch.contiguous_format)
        go = torch.zeros_like(opacities, memory_format=torch.contiguous_format)
        gc = torch.zeros_like(colors, memory_format=torch.contiguous_format)
        C = colors.reshape(colors.shape[0], -1).shape[1]
        out = grads_struct(gm, gq, gsc, go, gc.reshape(gc.shape[0], -1), colors_write=C,
                           colors_by_visible=ctx.colors_by_visible, accumulate=True)
        dC = torch.zeros_like(ctx.frame.color) if dC is None else dC.contiguous()
        dA = None if dA is None else dA.contiguous()
        render_backward(ctx.frame, ctx.g, out, device, dL_dcolor=dC, dL_dalpha=dA)
        return gm, gq, gsc, go, gc, None, None, None, None, None, None


def rasterize_gaussians_mlx(means, quats, scales, opacities, colors, viewmat, K, width: int, height: int,
                            active_indices, means_active=None, quats_active=None, scales_active=None,
                            opacities_active=None, render_width: int = 120, render_height: int = 90,
                            pixel_chunk_size: int = 1024, mask=None, raster_settings: Optional[RasterSettings] = None,
                            sh_mode: str = "reference", **kwargs):
    """mlx_gsplat/rendering.py:97-308.  Renders the Gaussians selected by
    ``active_indices`` (rows of ``means``/``quats``/``scales``/``opacities``, or
    of their ``*_active`` replacements when given) and returns
    ``(render_colors [RH, RW, 3], render_alphas [RH, RW, 1])``, differentiable
    with respect to the five parameter tensors.  ``colors`` is used row per
    visible Gaussian when it has one row per index, otherwise gathered too.
    ``pixel_chunk_size`` is accepted for compatibility (the tiled kernels need
    no pixel chunking).  ``mask`` ([V] values in [0, 1]) multiplies clipped
    alphas as the reference's does: entry j goes to the j-th visible Gaussian in
    depth order (the reference applies it after its depth sort without
    permuting it); no gradient flows to it.
    ``sh_mode="full"`` evaluates real spherical harmonics up to the degree the
    colour rows hold (3, 12, 27 or 48 floats: degree 0-3; the reference,
    ``"reference"``, stops at degree 1), with channel ch's coefficients at
    ``colors[:, 3 + k*ch : 3 + k*(ch+1)]``, k = (degree+1)**2 - 1."""
    m = means if means_active is None else means_active
    q = quats if quats_active is None else quats_active
    s = scales if scales_active is None else scales_active
    o = opacities if opacities_active is None else opacities_active
    ids = torch.as_tensor(active_indices, device=m.device).to(torch.int32).contiguous()
    V = int(ids.shape[0])
    if V == 0:
        return (torch.zeros((render_height, render_width, 3), dtype=torch.float32, device=m.device),
                torch.zeros((render_height, render_width, 1), dtype=torch.float32, device=m.device))
    cam = camera_struct(viewmat, K, width, height, render_width, render_height)
    by_visible = int(colors.shape[0]) == V
    mk = None
    if mask is not None:
        mk = torch.as_tensor(mask, device=m.device).detach().to(torch.float32).reshape(-1).contiguous()
        if mk.numel() != V:
            raise ValueError(f"rasterize_gaussians_mlx: mask has {mk.numel()} entries for {V} Gaussians")
        if bool(((mk < 0) | (mk > 1) | ~torch.isfinite(mk)).any()):
            raise ValueError("rasterize_gaussians_mlx: mask values must lie in [0, 1]")
    return _RasterizeFn.apply(m, q, s, o, colors, ids, cam, raster_settings or DEFAULT_SETTINGS, by_visible,
                              sh_mode_code(sh_mode), mk)
