"""Trainer loop (``MLXConfig`` / ``RunnerMLX``, mlx_gsplat/trainer.py:24-631) on B200.

One training step on one view (``train_step``) runs entirely on the GPU over
the pooled slab — no per-step gather of the active parameters:

    cull over the active ids (through the indirection table)
    -> tile rasterizer forward with the L1 loss fused into its epilogue
       (or the L1 + D-SSIM loss kernels after it)
    -> rasterizer backward writing one gradient row per visible Gaussian and
       accumulating the densification statistic (grad2d, count)
    -> [views data-parallel: sum of the gradient rows over GPUs]
    -> one fused Adam launch over the slab (+ quaternion renormalisation);
       unseen Gaussians' rows take the regulariser inside Adam
    -> periodic opacity reset and densify/prune (``densify``).

Loss: ``loss="l1"`` is mean |render - target| (the benchmark workloads);
``loss="l1+dssim"`` is the reference trainer's loss with a target,
0.8 * L1 + 0.2 * (1 - SSIM) / 2 (trainer.py:276-279, SSIM with its 11 x 11
box window); ``loss="mean"`` is the reference's target-less ``mean(render)``.  The
reference's ``1e-5 * sum(active params)`` term (trainer.py:283-292) is kept as
``param_reg``: +1e-5 on every means/quats/scales/opacities gradient of every
active Gaussian and on the gathered colour coefficients of visible ones.
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from . import _lib, distributed, synthetic
from .allocator import PointerStableChunkedAllocator, SlabLayout
from .optimizer import FusedMLXAdam
from .rendering import (DEFAULT_SETTINGS, RasterSettings, camera_struct, cull_ids, gaussians_struct, grads_struct,
                        render_backward, render_forward)


@dataclass
class MLXConfig:
    max_gaussians: int = 500000
    init_gaussians: Optional[int] = None
    max_steps: int = 300
    lr: float = 1.6e-4
    sh_degree: int = 3
    sh_degree_interval: int = 500
    refine_every: int = 100
    data_dir: str = "data/garden"
    data_factor: int = 8
    width: int = 800
    height: int = 600
    use_real_data: bool = True
    render_width: int = 200
    render_height: int = 150
    pixel_chunk_size: int = 1024
    preload_images: bool = True
    # B200 additions
    betas: Tuple[float, float] = (0.9, 0.999)
    eps: float = 1e-8
    # "l1+dssim": the reference trainer's loss with a target (trainer.py:276-279);
    # "l1": mean |render - target| (the benchmark workloads); "mean": mean(render)
    loss: str = "l1+dssim"
    param_reg: float = 1e-5
    densify: bool = True
    opacity_reset: bool = True
    alpha_cutoff: float = DEFAULT_SETTINGS.alpha_cutoff
    transmittance_min: float = DEFAULT_SETTINGS.transmittance_min
    near_plane: float = 0.01
    far_plane: float = 1e10
    opacity_threshold: float = -5.3
    # "reference": colour from SH degree <= 1 as the reference rasterizer does
    # (rendering.py:229-244); "full": real SH up to the scheduled degree (<= 3)
    sh_eval: str = "reference"
    # real-data mode: the reference passes the camera-to-world matrix where the
    # rasterizer expects world-to-camera (trainer.py:365); True reproduces that
    c2w_as_viewmat: bool = False
    # real-data mode: keep the uint8 training images in HBM (else each step
    # uploads its image from pinned host memory)
    images_on_device: bool = True
    seed: int = 0
    # narrow gradient rows (reference SH mode with SH degree > 1 stored): the
    # colour columns past SH degree 1 get only the regulariser, so the gradient
    # rows keep the 23 columns with gradients plus a view count and Adam
    # rebuilds the rest (2.5x fewer bytes summed over GPUs)
    compact_grad_rows: bool = True
    # with the multicast gradient sum (fused_reduce): each GPU runs Adam only for
    # the rows of the pool slots it owns, fused with the sum and the broadcast
    # of the updated parameters (else the rows are summed and Adam replicated)
    sharded_adam: bool = True
    # write ``<scene>_mlx_custom_3dgs.ply`` when train() finishes, as the
    # reference's train() does (trainer.py:566-568)
    export_ply_on_finish: bool = False
    # NCCL path across GPUs: True — the gradient rows are reduce-scattered, each
    # GPU runs Adam for its contiguous block of active ids and the columns the
    # rasterizer reads are all-gathered; False — an all-reduce pipelined with a
    # replicated Adam; None (default) — the sharded Adam from 4 GPUs up (measured
    # faster there; on two GPUs the replicated Adam is)
    nccl_sharded_adam: Optional[bool] = None
    # replicated-Adam NCCL path: the gradient rows are summed in this many row
    # ranges, each range's Adam running while the later ranges are reduced
    # (1: one all-reduce, then Adam)
    allreduce_buckets: int = 4


def lr_at(lr: float, step: int, max_steps: int) -> float:
    return lr * (0.01 ** (step / max_steps))


def sh_cols_for(step: int, cfg: MLXConfig) -> int:
    """Colour columns the rasterizer sees at ``step`` (trainer.py:242-250)."""
    d = min(step // cfg.sh_degree_interval, cfg.sh_degree)
    return 3 + 3 * ((d + 1) ** 2 - 1)


class StepTimer:
    """CUDA events between the phases of a step, on the step's stream."""

    PHASES = ("cull", "project_fwd", "depth_sort+offsets", "bin+tile_sort", "render_fwd", "grad_init",
              "render_bwd", "project_bwd", "allreduce", "adam")

    def __init__(self):
        self.events: List[Tuple[str, torch.cuda.Event]] = []

    def mark(self, name: str):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.events.append((name, e))

    def durations(self) -> Dict[str, float]:
        out: Dict[str, float] = {}
        for (n0, e0), (n1, e1) in zip(self.events[:-1], self.events[1:]):
            out[n1] = out.get(n1, 0.0) + e0.elapsed_time(e1)
        return out


def reference_init(cfg: MLXConfig):
    """The reference trainer's start (trainer.py:50-136) without MLX: with
    ``use_real_data`` and a COLMAP model under ``data_dir/sparse/0``, the
    normalised scene (``Parser(factor=data_factor, normalize=True)``), its train
    split and Gaussians initialised from the SfM points (log-scale log 0.01,
    random unit quaternions, opacity logit 0.1, SH DC from the point colours,
    higher SH zero; at most ``init_gaussians`` points, chosen with seed 42);
    otherwise the reference's synthetic mode (3,000 random Gaussians seen by
    an identity camera, K = [[500, 0, 400], [0, 500, 300]], no target).
    Returns ``(init_params, viewmats, Ks, sizes, scene_scale, train_dataset)``;
    random draws use ``cfg.seed`` (the reference uses the global NumPy state).
    A relative ``data_dir`` is taken from the current directory."""
    from . import dataset as D
    rng = np.random.default_rng(cfg.seed)
    data_dir = os.path.abspath(cfg.data_dir)
    shn_dim = ((cfg.sh_degree + 1) ** 2 - 1) * 3
    if cfg.use_real_data and os.path.exists(os.path.join(data_dir, "sparse/0")):
        parser = D.Parser(data_dir=data_dir, factor=cfg.data_factor, normalize=True)
        ds = D.Dataset(parser, split="train", preload_images=cfg.preload_images, seed=cfg.seed)
        points = np.array(parser.points, dtype=np.float32)
        rgbs = np.array(parser.points_rgb / 255.0, dtype=np.float32)
        n = len(points)
        if cfg.init_gaussians is not None and cfg.init_gaussians < n:
            keep = np.random.default_rng(42).choice(n, size=cfg.init_gaussians, replace=False)
            points, rgbs, n = points[keep], rgbs[keep], cfg.init_gaussians
        quats = rng.standard_normal((n, 4)).astype(np.float32)
        quats /= np.linalg.norm(quats, axis=-1, keepdims=True)
        init = {"means": points,
                "scales": np.full((n, 3), np.log(np.float32(0.01)), np.float32),
                "quats": quats,
                "opacities": np.full((n, 1), 0.1, np.float32),
                "sh0": ((rgbs - 0.5) / np.float32(synthetic.SH_C0)).astype(np.float32),
                "shN": np.zeros((n, shn_dim), np.float32)}
        viewmats, Ks, sizes = [], [], []
        for i in ds.indices:
            c2w = parser.camtoworlds[i]
            viewmats.append(c2w if cfg.c2w_as_viewmat else np.linalg.inv(c2w))
            cid = parser.camera_ids[i]
            Ks.append(parser.Ks_dict[cid])
            sizes.append(parser.imsize_dict[cid])
        return init, np.stack(viewmats), np.stack(Ks), sizes, float(parser.scene_scale), ds
    n = 3000
    init = {"means": rng.standard_normal((n, 3)).astype(np.float32),
            "scales": np.full((n, 3), np.log(np.float32(0.01)), np.float32),
            "quats": rng.standard_normal((n, 4)).astype(np.float32),
            "opacities": np.full((n, 1), 0.1, np.float32),
            "sh0": rng.standard_normal((n, 3)).astype(np.float32),
            "shN": rng.standard_normal((n, shn_dim)).astype(np.float32)}
    K = np.array([[500, 0, 400], [0, 500, 300], [0, 0, 1]], np.float32)
    return init, np.eye(4, dtype=np.float32)[None], K[None], [(cfg.width, cfg.height)], 1.0, None


class RunnerMLX:
    """The training loop of mlx_gsplat/trainer.py:44-631 on B200.
    ``RunnerMLX(cfg)`` starts as the reference does (``reference_init``: a
    COLMAP scene, or the synthetic mode); the other arguments give the scene
    directly (initial Gaussians, world-to-camera ``viewmats`` [V, 4, 4], one
    ``K`` [3, 3] or one per view, device targets [V, H, W, 3])."""

    def __init__(self, cfg: MLXConfig, init_params: Optional[Dict[str, np.ndarray]] = None,
                 viewmats: Optional[np.ndarray] = None, K: Optional[np.ndarray] = None,
                 targets: Optional[torch.Tensor] = None, device: Optional[torch.device] = None,
                 scene_scale: float = 1.0, process_group=None, fused_reduce: bool = False):
        self.cfg = cfg
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.train_dataset = None
        sizes = None
        if init_params is None:
            init_params, viewmats, K, sizes, scene_scale, self.train_dataset = reference_init(cfg)
            if self.train_dataset is not None and cfg.images_on_device and cfg.preload_images:
                self.train_dataset.to_device(self.device)
        L = SlabLayout(cfg.sh_degree)
        self.layout = L
        self.pg = process_group
        self.world = distributed.world_of(process_group)
        # Gradient rows: the layout of the pooled rows, or narrow rows — the
        # geometry and the 12 colour columns the reference rasterizer evaluates
        # (SH degree <= 1), then one view-count column; every colour column past
        # them has only the regulariser as gradient, which Adam rebuilds from the
        # count (g_cols, count_col, count_coef).
        if cfg.compact_grad_rows and cfg.sh_eval == "reference" and L.color_cols > 12:
            self.g_cols = L.color_col + 12
            self.count_col = self.g_cols
            self.g_stride = (self.g_cols + 1 + 3) // 4 * 4
        else:
            self.g_cols, self.count_col, self.g_stride = L.ncols, 0, L.stride
        # Across GPUs the gradient rows are summed by NCCL, or (``fused_reduce``)
        # through NVLink multicast: by this library's row-sum kernel before a
        # replicated Adam, or (``cfg.sharded_adam``) inside the sharded Adam,
        # which updates the rows of the slots this GPU owns and broadcasts the
        # columns the rasterizer reads (``hot_cols``) to every GPU.
        self.fused_reduce = None
        self.sharded = False
        self.sharded_nccl = False
        if fused_reduce and distributed.FusedRowReduce.available(self.device, process_group):
            self.sharded = bool(cfg.sharded_adam)
            self.fused_reduce = distributed.FusedRowReduce(cfg.max_gaussians, self.g_stride, self.device,
                                                           process_group,
                                                           theta_cols=L.stride if self.sharded else None)
        self.allocator = PointerStableChunkedAllocator(
            cfg.max_gaussians, cfg.sh_degree, device=self.device,
            theta_storage=self.fused_reduce.theta if self.sharded else None)
        self.allocator.set_initial_gaussians(init_params)
        self.optimizer = FusedMLXAdam(lr=cfg.lr, betas=cfg.betas, eps=cfg.eps)
        # columns every GPU needs each step: what the rasterizer reads (the
        # geometry and SH <= 1 colour in the reference mode), whole 16-byte chunks
        self.hot_cols = L.stride if cfg.sh_eval == "full" else min(L.stride, (L.color_col + 12 + 3) // 4 * 4)
        self._owned = self.fused_reduce.owned_slots(cfg.max_gaussians) if self.sharded else None
        # NCCL across GPUs with a sharded Adam: rank r updates the active ids of
        # block r (distributed.block_of); the row buffers have room for the
        # padding of the last block
        self.sharded_nccl = distributed.use_sharded_nccl_adam(cfg.nccl_sharded_adam, self.world,
                                                              multicast=self.fused_reduce is not None)
        if self.fused_reduce is not None:
            self.grad = self.fused_reduce.rows
        else:
            pad = self.world if self.sharded_nccl else 0
            self.grad = torch.zeros((cfg.max_gaussians + pad, self.g_stride), dtype=torch.float32,
                                    device=self.device)
        if self.sharded_nccl:
            rows = cfg.max_gaussians + self.world
            self._grad_shard = torch.empty((-(-rows // self.world), self.g_stride), dtype=torch.float32,
                                           device=self.device)
            self._hot_rows = torch.empty((rows, self.hot_cols), dtype=torch.float32, device=self.device)
        lo, hi = L.col_bounds()
        self.col_lo, self.col_hi = lo.tolist(), hi.tolist()
        self.viewmats = np.asarray(viewmats, np.float32)
        self.K = np.asarray(K, np.float32)
        Ks = self.K if self.K.ndim == 3 else [self.K] * len(self.viewmats)
        if self.K.ndim == 3 and len(self.K) == 1:
            self.K = self.K[0]
            Ks = [self.K] * len(self.viewmats)
        sizes = sizes or [(cfg.width, cfg.height)] * len(self.viewmats)
        self.cams = [camera_struct(vm, k, w, h, cfg.render_width, cfg.render_height)
                     for vm, k, (w, h) in zip(self.viewmats, Ks, sizes)]
        self.targets = targets
        self.rng = np.random.default_rng(cfg.seed)
        self.settings = RasterSettings(cfg.alpha_cutoff, cfg.transmittance_min)
        self.scene_scale = scene_scale
        self.last_frame = None
        self._child_rows = None  # [2, capacity, stride] child rows of the density step
        self.step_count = 0
        self._k_hint = 0  # tile-entry buffer size for the next view (grows with the views seen)
        # How gradient rows of unseen Gaussians are formed: "sparse" (one GPU:
        # Adam takes the regulariser row for them from the cull's visibility
        # bits), "dense" (every row filled with the regulariser first), "summed"
        # (rows summed over GPUs from a zeroed slab; Adam adds world * reg).
        self.row_mode = "summed" if self.world > 1 else "sparse"

    # ------------------------------------------------------------------ helpers
    def _reg_pattern(self, n: Optional[int] = None) -> List[float]:
        """``n`` columns (default: a gradient row) with the regulariser on the
        geometry columns and zero elsewhere."""
        L = self.layout
        pat = [0.0] * (self.g_stride if n is None else n)
        for name in ("quats", "means", "opacities", "scales"):
            o = L.offsets[name]
            for c in range(o, o + L.dims[name]):
                pat[c] = self.cfg.param_reg
        return pat

    def count_coef(self, step: int) -> List[float]:
        """Per parameter column: the regulariser a view adds to a column that
        narrow gradient rows do not hold (the colour columns the rasterizer
        reads at this step's SH degree get it, the others nothing)."""
        L = self.layout
        reg_cols = sh_cols_for(step, self.cfg)
        return [self.cfg.param_reg if c >= self.g_cols and c - L.color_col < reg_cols else 0.0
                for c in range(L.ncols)]

    def full_gradient_rows(self, step: int, n: Optional[int] = None) -> torch.Tensor:
        """The gradient rows as ``[n, ncols]`` parameter columns, for inspection:
        narrow rows get their regulariser-only colour columns rebuilt from the
        view count as Adam rebuilds them (the cross-GPU bias and 1/world scale
        Adam also applies in the summed row mode are not)."""
        L = self.layout
        n = self.allocator.num_active if n is None else n
        G = self.grad[:n]
        if self.g_cols == L.ncols:
            return G[:, :L.ncols].clone()
        out = torch.zeros((n, L.ncols), dtype=torch.float32, device=self.device)
        out[:, :self.g_cols] = G[:, :self.g_cols]
        coef = torch.tensor(self.count_coef(step), dtype=torch.float32, device=self.device)
        out[:, self.g_cols:] = G[:, self.count_col:self.count_col + 1] * coef[self.g_cols:]
        return out

    def _gaussians(self, step: int):
        L = self.layout
        th = self.allocator.theta
        pools = self.allocator.physical_pools
        return gaussians_struct(pools["means"], pools["quats"], pools["scales"], pools["opacities"],
                                th[:, L.color_col:], colors_dim=sh_cols_for(step, self.cfg),
                                table=self.allocator.indirection_table, sh_mode=self.cfg.sh_eval)

    def _grad_out(self, step: int):
        L = self.layout
        gb = self.grad
        o = L.offsets
        # summed rows: Adam adds the geometry regulariser once for every row
        summed = self.row_mode == "summed"
        return grads_struct(gb[:, o["means"]:o["means"] + 3], gb[:, o["quats"]:o["quats"] + 4],
                            gb[:, o["scales"]:o["scales"] + 3], gb[:, o["opacities"]:o["opacities"] + 1],
                            gb[:, L.color_col:], colors_write=self.g_cols - L.color_col, colors_by_visible=False,
                            accumulate=False, reg=self.cfg.param_reg, reg_color_cols=sh_cols_for(step, self.cfg),
                            reg_geometry=not summed, count_col=self.count_col)

    # ------------------------------------------------------------------ one step
    def train_step(self, view_idx: int, step: int, target: Optional[torch.Tensor] = None,
                   timer: Optional[StepTimer] = None):
        """One view: forward, backward, (all-reduce), Adam.  ``target`` is a
        device uint8 HWC image (defaults to ``targets[view_idx]``)."""
        cfg = self.cfg
        lib = _lib.lib()
        st = _lib.stream_ptr(self.device)
        self.optimizer.lr = lr_at(cfg.lr, step, cfg.max_steps)
        N = self.allocator.num_active
        cam = self.cams[view_idx % len(self.cams)]
        if target is None and self.targets is not None:
            target = self.targets[view_idx % self.targets.shape[0]]
        elif target is None and self.train_dataset is not None:
            target = self.dataset_target(view_idx % len(self.train_dataset))
        ssim_loss = cfg.loss == "l1+dssim" and target is not None
        if cfg.loss not in ("l1", "mean", "l1+dssim"):
            raise ValueError(f"unknown loss {cfg.loss!r} (l1, mean or l1+dssim)")
        if ssim_loss:
            loss_mode = _lib.GS_LOSS_NONE  # the image loss and dL/dC come from gs_l1_dssim_loss
        elif cfg.loss == "mean" or target is None:
            loss_mode = _lib.GS_LOSS_MEAN
        else:
            loss_mode = _lib.GS_LOSS_L1_U8 if target.dtype == torch.uint8 else _lib.GS_LOSS_L1_F32
        g = self._gaussians(step)
        if timer:
            timer.mark("start")
        ids, vcount, _, cull_scratch = cull_ids(g, N, cam, self.device, cfg.near_plane, cfg.far_plane,
                                                cfg.opacity_threshold, sync=False, return_scratch=True)
        if timer:
            timer.mark("cull")
        # buffers are sized from N and the entry counts of earlier views, before
        # the counts are read back
        frame = render_forward(g, ids, N, cam, self.settings, self.device, loss_mode=loss_mode, target=target,
                               timer=timer, v_count=vcount, k_hint=self._k_hint)
        # 50% headroom: views differ in their entry counts, and a view that exceeds
        # the hint gets freshly allocated entry buffers
        self._k_hint = max(self._k_hint, frame.K + frame.K // 2)
        dL_dcolor = self._l1_dssim(frame, target) if ssim_loss else None
        if ssim_loss and timer:
            timer.mark("loss")
        # Gradient rows of Gaussians this view does not see hold only the
        # regulariser.  On one GPU Adam takes them from the cull's visibility bits
        # (no rows written).  Across GPUs every GPU stores only its visible rows
        # (without the geometry regulariser) into a slab that is zero elsewhere,
        # the rows are summed over GPUs, and Adam adds ``world * reg`` to every
        # row before the ``1/world`` scale.
        mode = self.row_mode
        fused = self.fused_reduce is not None
        if mode == "dense":
            _lib.check(lib.gs_fill_rows(self.grad.data_ptr(), N, self.g_stride, _lib.fptr(self._reg_pattern()),
                                        st), "grad init")
            if timer:
                timer.mark("grad_init")
        render_backward(frame, g, self._grad_out(step), self.device, dL_dcolor=dL_dcolor,
                        grad2d=self.allocator.grad2d, count=self.allocator.count, timer=timer)
        scale = 1.0
        bias = None
        sparse = mode == "sparse"
        vis = (cull_scratch.data_ptr() + 255) // 256 * 256 if sparse else None
        if mode == "summed":
            scale = 1.0 / self.world
            bias = [self.world * r for r in self._reg_pattern(self.layout.ncols)]
            if self.sharded:
                self._sharded_adam(N, step, scale, bias)
                if timer:
                    timer.mark("sharded_adam")
            elif fused:
                self.fused_reduce.sum_rows(N)
                if timer:
                    timer.mark("row_sum")
            elif self.sharded_nccl:
                self._nccl_sharded_adam(N, step, scale, bias, timer)
            elif cfg.allreduce_buckets > 1 and self.world > 1:
                self._bucketed_allreduce_adam(N, step, scale, bias, timer)
            else:
                distributed.reduce_gradient_rows(self.grad[:N], self.pg)
                if timer:
                    timer.mark("allreduce")
        if not self.sharded and not self.sharded_nccl and not (mode == "summed" and not fused and
                                                               cfg.allreduce_buckets > 1 and self.world > 1):
            self._adam_rows(0, N, step, scale, bias, vis=vis)
            if timer:
                timer.mark("adam")
        if mode == "summed":
            # this GPU's rows for the next step (with the multicast sum the
            # peers are past it: the next step's first barrier orders the rest)
            self.grad[:N].zero_()
            if timer:
                timer.mark("zero_rows")
        self.last_frame = frame
        self.step_count += 1
        return frame

    def _adam_rows(self, r0: int, r1: int, step: int, scale: float, bias, vis=None,
                   advance: bool = True, g: Optional[torch.Tensor] = None) -> None:
        """The slab Adam over the active ids [r0, r1), their gradient rows
        ``g`` (default: rows [r0, r1) of the gradient slab)."""
        L, al = self.layout, self.allocator
        if r1 <= r0:
            if advance:
                self.optimizer.t += 1  # every rank keeps the same step count
            return
        g = self.grad[r0:r1] if g is None else g
        self.optimizer.step_slab(al.theta, g, al.adam_m, al.adam_v, al.indirection_table[r0:r1],
                                 r1 - r0, L.ncols, self.col_lo, self.col_hi, quat_col=L.quat_col, grad_scale=scale,
                                 visible_words=vis, unseen_grad=self._reg_pattern(L.ncols) if vis is not None else None,
                                 grad_bias=bias, g_cols=self.g_cols, count_col=self.count_col,
                                 count_coef=self.count_coef(step) if self.g_cols < L.ncols else None, advance=advance)

    def _nccl_sharded_adam(self, N: int, step: int, scale: float, bias, timer=None) -> None:
        """The gradient rows reduce-scattered over the GPUs (NCCL), Adam on this
        GPU's block of active ids only, then the columns the rasterizer reads
        (``hot_cols``) of every block all-gathered and written into every GPU's
        parameter slab.  The same bytes cross NVLink as with an all-reduce, and
        Adam's HBM traffic is 1/N of a replicated one.  The other parameter
        columns and the moments are current only on the block's owner until
        ``gather_sharded_state``."""
        import torch.distributed as dist
        lib = _lib.lib()
        st = _lib.stream_ptr(self.device)
        al, L = self.allocator, self.layout
        W, r = self.world, distributed.rank_of(self.pg)
        first, count, per = distributed.block_of(N, r, W)
        shard = self._grad_shard[:per]
        dist.reduce_scatter_tensor(shard, self.grad[:per * W], op=dist.ReduceOp.SUM, group=self.pg)
        if timer:
            timer.mark("reduce_scatter")
        self._adam_rows(first, first + count, step, scale, bias, g=shard[:count])
        if timer:
            timer.mark("adam")
        hot, hc = self._hot_rows, self.hot_cols
        tab = al.indirection_table
        if count:
            _lib.check(lib.gs_copy_rows(al.theta.data_ptr(), L.stride, tab[first:].data_ptr(),
                                        hot[first:].data_ptr(), hc, None, count, hc, st), "pack columns")
        # rank r's block is its slice of the gathered rows (in place)
        dist.all_gather_into_tensor(hot[:per * W], hot[r * per:(r + 1) * per], group=self.pg)
        _lib.check(lib.gs_copy_rows(hot.data_ptr(), hc, None, al.theta.data_ptr(), L.stride, tab.data_ptr(), N, hc,
                                    st), "unpack columns")
        if timer:
            timer.mark("all_gather")

    def _owned_slots_of_block(self) -> torch.Tensor:
        """Boolean mask of the pool slots whose rows this GPU's sharded NCCL Adam
        updates (the slots of its block of active ids)."""
        al = self.allocator
        first, count, _ = distributed.block_of(al.num_active, distributed.rank_of(self.pg), self.world)
        owned = torch.zeros(al.max_gaussians, dtype=torch.bool, device=self.device)
        owned[al.indirection_table[first:first + count].long()] = True
        return owned

    def _bucketed_allreduce_adam(self, N: int, step: int, scale: float, bias, timer=None) -> None:
        """The sum of the gradient rows over GPUs pipelined with Adam: the rows
        are cut into ``cfg.allreduce_buckets`` ranges, every range's NCCL
        all-reduce is queued at once on NCCL's stream, and Adam updates range b
        as soon as range b is summed, while the later ranges are still being
        reduced."""
        nb = max(1, min(self.cfg.allreduce_buckets, N))
        edges = [N * b // nb for b in range(nb + 1)]
        works = [torch.distributed.all_reduce(self.grad[edges[b]:edges[b + 1]], group=self.pg, async_op=True)
                 for b in range(nb)]
        for b in range(nb):
            works[b].wait()  # this stream waits for bucket b's sum
            self._adam_rows(edges[b], edges[b + 1], step, scale, bias, advance=b == 0)
        if timer:
            timer.mark("allreduce+adam")

    def dataset_target(self, item: int) -> torch.Tensor:
        """The training image of dataset item ``item`` as this step's target:
        the uint8 image itself when it has the render size, else
        ``bilinear_resize_mlx(image / 255.0)`` to the render size
        (trainer.py:231-234, 369), both on the GPU."""
        from .rendering import bilinear_resize_mlx
        img = self.train_dataset.device_image(item, self.device)
        RH, RW = self.cfg.render_height, self.cfg.render_width
        if tuple(img.shape[:2]) == (RH, RW):
            return img
        return bilinear_resize_mlx(img, RH, RW)

    def _sharded_adam(self, N: int, step: int, scale: float, bias) -> None:
        """Barrier (every GPU wrote its gradient rows), the sharded Adam over the
        slots this GPU owns, barrier (every broadcast landed and every sum was
        read, so the rows may be zeroed and the next cull sees the parameters)."""
        fr = self.fused_reduce
        al, L = self.allocator, self.layout
        fr.barrier(0)
        self.optimizer.step_slab_sharded(al.theta, fr.theta_multicast, fr.multicast, self.g_stride, al.adam_m,
                                         al.adam_v, al.indirection_table, N, L.ncols, self.col_lo, self.col_hi,
                                         fr.rank, fr.world, self.hot_cols, quat_col=L.quat_col, grad_scale=scale,
                                         grad_bias=bias, g_cols=self.g_cols, count_col=self.count_col,
                                         count_coef=self.count_coef(step) if self.g_cols < L.ncols else None,
                                         error_flag=fr.error.data_ptr())
        fr.barrier(1)

    def gather_sharded_state(self, moments: bool = True) -> None:
        """With the sharded Adam, the parameter columns past ``hot_cols`` and the
        moments are current only on the GPU that owns each slot: every GPU's
        copy becomes the owners' (the parameters, and ``moments`` too).  The
        densify step, the PLY export and checkpoints call it first."""
        if not (self.sharded or self.sharded_nccl):
            return
        al = self.allocator
        self.check_group()
        if al.num_active == 0:
            return
        t = al.indirection_table
        used = slice(int(t.min()), int(t.max()) + 1)  # the slot range in use (the free list pops from the top)
        owned = self._owned if self.sharded else self._owned_slots_of_block()
        # theta: only the columns past the broadcast ones differ between GPUs
        distributed.gather_owned_rows(al.theta, owned, self.pg, used, first_col=self.hot_cols)
        if moments:
            distributed.gather_owned_rows(al.adam_m, owned, self.pg, used)
            distributed.gather_owned_rows(al.adam_v, owned, self.pg, used)

    def check_group(self) -> None:
        """Raises if a multi-GPU barrier wait gave up (``FusedRowReduce.check``;
        a host sync).  Called where the host syncs anyway: densify, export,
        checkpoints, the log lines and the end of ``train``."""
        if self.fused_reduce is not None:
            self.fused_reduce.check()

    # ------------------------------------------------------------------ densify / prune
    def densify(self, step: int, noise: Optional[Dict[str, torch.Tensor]] = None) -> Tuple[int, int]:
        """trainer.py:425-519 on the GPU: decisions from the pooled rows and the
        accumulated statistics, children built from the parents and seeded
        normal noise, the pool updated in place, then grad2d/count cleared.
        With views data-parallel the statistics are all-reduced first, and every
        rank draws the same noise (a generator seeded by the step), so every
        replica takes identical decisions."""
        cfg = self.cfg
        lib = _lib.lib()
        st = _lib.stream_ptr(self.device)
        al = self.allocator
        L = self.layout
        N = al.num_active
        self.check_group()
        # children copy whole parent rows; with blocks of active ids the blocks
        # move when the table changes, so the moments are gathered as well
        self.gather_sharded_state(moments=self.sharded_nccl)
        distributed.reduce_densify_stats(al.grad2d, al.count, self.pg)
        g = self._gaussians(step)
        flags = al.workspace()["flags"]
        f32 = np.float32
        _lib.check(lib.gs_densify_masks(g, al.grad2d.data_ptr(), al.count.data_ptr(), N, 0.0002,
                                        float(f32(0.01 * self.scene_scale)), float(f32(0.1 * self.scene_scale)),
                                        0.005, 5e-2, int(N >= 80000), flags.data_ptr(), st), "densify masks")
        self.last_densify = {"flags": flags[:N]}  # valid until the next density step

        def make_children(split_slots, refine_rows, n):
            nz = noise if noise is not None else distributed.densify_noise(step, n, self.device)
            self.last_densify["noise"] = nz
            # child rows: buffers kept between density steps, grown (with headroom) when a step needs more
            if self._child_rows is None or self._child_rows.shape[1] < n:
                cap = min(al.max_gaussians, n + n // 4 + 1024)
                self._child_rows = torch.empty((2, cap, L.stride), dtype=torch.float32, device=self.device)
            c1, c2 = self._child_rows[0, :n], self._child_rows[1, :n]
            o = L.offsets
            _lib.check(lib.gs_densify_children(al.theta.data_ptr(), L.stride, L.ncols, split_slots.data_ptr(),
                                               refine_rows.data_ptr(), flags.data_ptr(), nz["means1"].data_ptr(),
                                               nz["means2"].data_ptr(), nz["quats2"].data_ptr(), n, o["means"],
                                               o["scales"], o["quats"], o["opacities"], c1.data_ptr(), c2.data_ptr(),
                                               st), "densify children")
            return c1, c2

        n_p, n_s = al.apply_flags(flags, make_children)
        al.grad2d.zero_()
        al.count.zero_()
        return n_p, n_s

    def scale_densify_stats(self, fraction: float, threshold: float = 0.0002) -> float:
        """Stress knob for the density step (not part of the reference's
        schedule): scales the accumulated view-space gradients so that the
        ``fraction`` of active Gaussians with the largest average statistic
        exceed ``threshold``; returns the factor.  Large renders give small
        per-pixel gradients, whose statistics may never reach the reference's
        2e-4 otherwise."""
        al = self.allocator
        t = al.indirection_table.long()
        avg = al.grad2d[t] / al.count[t].clamp(min=1.0)
        q = float(torch.quantile(avg.float(), 1.0 - fraction)) if avg.numel() <= (1 << 24) else \
            float(avg.kthvalue(max(1, int(avg.numel() * (1.0 - fraction)))).values)
        factor = threshold / q * 1.0001 if q > 0 else 1.0
        al.grad2d.mul_(factor)
        return factor

    def _l1_dssim(self, frame, target: torch.Tensor) -> torch.Tensor:
        """The reference trainer's image loss 0.8 * L1 + 0.2 * (1 - SSIM) / 2
        (trainer.py:276-279) of the rendered frame; returns dL/dC (HWC) and
        keeps the loss (and SSIM) on the frame."""
        lib = _lib.lib()
        RW, RH = frame.cam.render_width, frame.cam.render_height
        key = (RW, RH)
        if getattr(self, "_ssim_key", None) != key:
            self._ssim_scratch = torch.empty(lib.gs_l1_dssim_scratch_bytes(RW, RH), dtype=torch.uint8,
                                             device=self.device)
            self._ssim_dc = torch.empty((RH, RW, 3), dtype=torch.float32, device=self.device)
            self._ssim_key = key
        frame.loss_scalar = torch.empty(2, dtype=torch.float32, device=self.device)  # loss, SSIM
        _lib.check(lib.gs_l1_dssim_loss(frame.color.data_ptr(), target.data_ptr(),
                                        int(target.dtype == torch.uint8), RW, RH, 0.8, 0.2,
                                        frame.loss_scalar.data_ptr(), frame.loss_scalar[1:].data_ptr(),
                                        self._ssim_dc.data_ptr(), self._ssim_scratch.data_ptr(),
                                        self._ssim_scratch.numel(), _lib.stream_ptr(self.device)),
                   "l1+dssim loss")
        return self._ssim_dc

    def loss_value(self, frame=None) -> torch.Tensor:
        f = frame or self.last_frame
        if getattr(f, "loss_scalar", None) is not None:
            return f.loss_scalar[0]
        P = f.cam.render_width * f.cam.render_height
        return f.loss_partials.sum() / (3.0 * P)

    # ------------------------------------------------------------------ export / checkpoint
    def export_to_ply(self, filepath: str) -> int:
        """trainer.py:570-631: the active Gaussians as a binary little-endian PLY
        (quaternions normalised, log-scales and opacity logits clipped).  The
        rows are gathered on the GPU (``gs_export_rows``); returns the count."""
        L = self.layout
        if "sh0" not in L.offsets:
            raise NotImplementedError("PLY export needs the SH colour layout (sh0 + shN)")
        lib = _lib.lib()
        al = self.allocator
        n = al.num_active
        self.gather_sharded_state(moments=False)
        cols = 14 + L.color_cols  # means 3, normals 3, colours, opacity 1, scales 3, quaternion 4
        out = torch.empty((max(n, 1), cols), dtype=torch.float32, device=self.device)
        _lib.check(lib.gs_export_rows(al.theta.data_ptr(), L.stride, al.indirection_table.data_ptr(), n,
                                      L.offsets["means"], L.offsets["opacities"], L.offsets["scales"], L.quat_col,
                                      L.color_col, L.color_cols, out.data_ptr(), cols,
                                      _lib.stream_ptr(self.device)), "export rows")
        rows = out[:n].cpu().numpy()
        if distributed.rank_of(self.pg) != 0:  # every rank holds the same rows; one writes the file
            self._group_barrier()
            return n
        head = [b"ply\n", b"format binary_little_endian 1.0\n", f"element vertex {n}\n".encode()]
        head += [f"property float {p}\n".encode() for p in ("x", "y", "z", "nx", "ny", "nz")]
        head += [f"property float f_dc_{j}\n".encode() for j in range(L.dims["sh0"])]
        head += [f"property float f_rest_{j}\n".encode() for j in range(L.dims["shN"])]
        head += [b"property float opacity\n"]
        head += [f"property float scale_{i}\n".encode() for i in range(3)]
        head += [f"property float rot_{i}\n".encode() for i in range(4)]
        head += [b"end_header\n"]
        with open(filepath, "wb") as f:
            f.write(b"".join(head))
            f.write(rows.astype("<f4").tobytes())
        self._group_barrier()
        return n

    def _group_barrier(self) -> None:
        """Host barrier of the process group (after rank 0 wrote a file)."""
        if self.world > 1:
            torch.distributed.barrier(group=self.pg)

    _CKPT_TENSORS = ("theta", "adam_m", "adam_v", "free_stack", "active_mask", "grad2d", "count")

    def save_checkpoint(self, filepath: str) -> None:
        """The whole training state: the pooled parameter and moment slabs, the
        indirection table, the free list, the densification statistics, the
        Adam step and the trainer's step count (``.npz``)."""
        al = self.allocator
        self.gather_sharded_state()
        torch.cuda.synchronize(self.device)
        state = {k: getattr(al, k).cpu().numpy() for k in self._CKPT_TENSORS}
        state["indirection_table"] = al.indirection_table.cpu().numpy()
        state["free_top"] = np.int64(al.free_top)
        state["adam_t"] = np.int64(self.optimizer.t)
        state["step_count"] = np.int64(self.step_count)
        state["layout"] = np.array([al.max_gaussians, al.layout.stride, al.layout.ncols], np.int64)
        if distributed.rank_of(self.pg) == 0:  # every rank holds the same state; one writes the file
            np.savez(filepath, **state)
        self._group_barrier()

    def load_checkpoint(self, filepath: str) -> None:
        """Restores a ``save_checkpoint`` state into this runner (same pool size
        and layout); the pools keep their device addresses."""
        al = self.allocator
        d = np.load(filepath)
        want = np.array([al.max_gaussians, al.layout.stride, al.layout.ncols], np.int64)
        if not np.array_equal(d["layout"], want):
            raise ValueError(f"checkpoint pool {d['layout'].tolist()} does not match {want.tolist()}")
        for k in self._CKPT_TENSORS:
            getattr(al, k).copy_(torch.from_numpy(d[k]))
        al.indirection_table = torch.from_numpy(d["indirection_table"]).to(self.device)
        al.free_top = int(d["free_top"])
        al.update_cached_pointers()
        self.optimizer.t = int(d["adam_t"])
        self.step_count = int(d["step_count"])

    # ------------------------------------------------------------------ full loop
    def train(self, log_every: int = 20):
        cfg = self.cfg
        t0 = time.time()
        for step in range(1, cfg.max_steps + 1):
            if self.train_dataset is not None:
                v = int(self.rng.integers(0, len(self.train_dataset)))  # trainer.py:362
            else:
                v = (step - 1) % len(self.cams)
            self.train_step(v, step)
            if cfg.opacity_reset:
                interval = 1000 if cfg.max_steps <= 3000 else 3000
                if step % interval == 0:
                    self.allocator.reset_opacities(-4.59)
            if cfg.densify:
                d0 = 300 if cfg.max_steps <= 3000 else 500
                d1 = 15000 if cfg.max_steps >= 30000 else int(cfg.max_steps * 0.7)
                if d0 <= step <= d1 and step % cfg.refine_every == 0:
                    n_p, n_s = self.densify(step)
                    if log_every:
                        print(f"[Step {step:4d} - Densification] Pruned: {n_p} | Split/Duplicated: {n_s} | "
                              f"Active GS: {self.allocator.num_active}")
            if log_every and (step % log_every == 0 or step == 1):
                self.check_group()
                print(f"Step {step:5d} | Active: {self.allocator.num_active} | loss {float(self.loss_value()):.5f}")
        torch.cuda.synchronize(self.device)
        self.check_group()
        elapsed = time.time() - t0
        if log_every:
            print(f"\n[Finished] 3DGS training complete in {elapsed:.2f} seconds.")
            print(f"Average speed: {elapsed / max(cfg.max_steps, 1) * 1000:.2f} ms/iter.")
        if cfg.export_ply_on_finish:
            name = os.path.basename(os.path.abspath(cfg.data_dir).rstrip("/\\"))
            self.export_to_ply(f"{name}_mlx_custom_3dgs.ply")
        return elapsed


def runner_for_workload(name: str, max_steps: int = 100, num_views: Optional[int] = None, device=None,
                        n: Optional[int] = None, lr: float = 1e-3, eps: float = 1e-15, seed: int = 0,
                        loss: str = "l1", upload_targets: bool = True, process_group=None,
                        fused_reduce: bool = False, **overrides) -> RunnerMLX:
    """A runner for one of the synthetic workloads (``synthetic.WORKLOADS``)."""
    wl = synthetic.WORKLOADS[name]
    g = synthetic.make_gaussians(wl, seed=seed, n=n)
    views, K = synthetic.make_cameras(wl, seed=2, num_views=num_views)
    cap = wl.capacity or g["means"].shape[0]
    cfg = MLXConfig(max_gaussians=cap, max_steps=max_steps, lr=lr, sh_degree=wl.sh_degree, sh_degree_interval=1,
                    width=wl.width, height=wl.height, render_width=wl.width, render_height=wl.height, eps=eps,
                    loss=loss)
    for k, v in overrides.items():
        setattr(cfg, k, v)
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    targets = None
    if upload_targets and wl.target_kind == "uint8":
        targets = torch.from_numpy(synthetic.make_uint8_targets(wl, min(len(views), 8), seed=1)).to(dev)
    elif upload_targets and wl.target_kind == "render":
        targets = render_targets(wl, views, K, dev, seed=1, n=n)
    return RunnerMLX(cfg, g, views, K, targets=targets, device=dev, scene_scale=synthetic.scene_scale(views),
                     process_group=process_group, fused_reduce=fused_reduce)


def render_targets(wl: synthetic.Workload, views: np.ndarray, K: np.ndarray, device, seed: int = 1,
                   n: Optional[int] = None) -> torch.Tensor:
    """Target images rendered from a second seeded Gaussian set (float32 HWC per view)."""
    from .rendering import frustum_culling_mlx, rasterize_gaussians_mlx
    g = synthetic.make_gaussians(wl, seed=seed, n=n)
    t = {k: torch.from_numpy(v).to(device) for k, v in g.items()}
    cols = torch.cat([t["sh0"], t["shN"]], 1)
    out = []
    with torch.no_grad():
        for vm in views:
            ids = frustum_culling_mlx(t["means"], None, None, vm, K, wl.width, wl.height, opacities=t["opacities"])
            C, _ = rasterize_gaussians_mlx(t["means"], t["quats"], t["scales"], t["opacities"], cols, vm, K,
                                           wl.width, wl.height, ids, render_width=wl.width, render_height=wl.height)
            out.append(C.contiguous())
    return torch.stack(out)
