#!/usr/bin/env python
"""Benchmark of the 3DGS training hot path on B200.

One *step* = one camera view per GPU: cull -> tile rasterizer forward with the
L1 loss fused in -> rasterizer backward -> the fused Adam over the pooled slab.
Across GPUs the gradient rows are summed over NCCL: from 4 GPUs up by a
reduce-scatter, Adam over each GPU's block of rows and an all-gather of the
columns the rasterizer reads; on 2 GPUs by an all-reduce in four row ranges,
each range's replicated Adam launched as soon as the range is summed.  Workload: the
``outdoor-1m`` scene (1,000,000 Gaussians, SH degree 3, 160 ring views at
1297x840, fx = fy = 1150, seeded uint8 targets).

``value`` = train steps/s summed over GPUs (views processed per second by the
whole job) with every input resident in HBM.  ``e2e`` = the same metric
through the public API with each step's target image copied from pinned host
memory and the loss read back.  ``roofline`` is for the dominant kernel,
timed live with CUDA events on the launching stream.  ``cpu_baseline`` times
the CPU oracle (dense O(pixels x Gaussians) rasterizer + Adam) on a bounded
sample and scales it to a full step.

Usage: ``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]``
(N > 1 under ``torch.distributed.run``, one process per GPU).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "src": "measured"}
    return {"hbm_gbs": PEAKS_FALLBACK["hbm_gbs"], "src": "fallback"}


# What actually limits each kernel (ncu summaries under profiles/): the compositing kernels keep
# their splat records in L2 and are bound by FP32 instruction issue, not by HBM.
LIMITERS = {"render_bwd": "fp32 instruction issue (ncu issue-active ~79%, DRAM ~1%; paired f32x2 math)",
            "render_fwd": "fp32 instruction issue (ncu issue-active ~75%, DRAM ~1%; paired f32x2 math)",
            "adam": "hbm"}


def measured_traffic(kernel: str, workload: str):
    """DRAM bytes per launch of ``kernel`` from the committed one-pass ncu capture
    of this workload (``profiles/dram_traffic.json``), or None."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if not os.path.exists(path):
        return None
    return json.load(open(path)).get(workload, {}).get("bytes_per_launch", {}).get(kernel)


def metric_name(workload: str) -> str:
    from mlx_gsplat_b200 import synthetic
    wl = synthetic.WORKLOADS[workload]
    return (f"train steps/s (1 view per GPU per step, fwd+bwd+Adam) @ {workload} "
            f"{wl.num_gaussians} Gaussians {wl.width}x{wl.height}")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="outdoor-1m")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the densify and 6M-row Adam measurements")
    ap.add_argument("--multicast", action="store_true",
                    help="N > 1: the sharded Adam fused with the NVLink multicast gradient sum and parameter "
                         "broadcast, instead of an NCCL all-reduce and a replicated Adam")
    ap.add_argument("--gaussians", type=int, default=None, help="override the workload's Gaussian count (profiling)")
    ap.add_argument("--views", type=int, default=None, help="override the workload's view count (profiling)")
    nccl_path = ap.add_mutually_exclusive_group()
    nccl_path.add_argument("--sharded-adam", action="store_true",
                           help="N > 1 over NCCL: reduce-scatter the gradient rows, run Adam on each GPU's block of "
                                "rows and all-gather the rasterizer's columns (the default from 4 GPUs up)")
    nccl_path.add_argument("--replicated-adam", action="store_true",
                           help="N > 1 over NCCL: an all-reduce pipelined with a replicated Adam (the default on 2 "
                                "GPUs)")
    ap.add_argument("--allreduce-buckets", type=int, default=4,
                    help="N > 1 over NCCL: row ranges of the gradient sum, each range's Adam overlapping the later "
                         "ranges' all-reduce (1: one all-reduce, then Adam)")
    ap.add_argument("--target-images", type=int, default=None,
                    help="distinct seeded uint8 target images, cycled over the views (default: one per view, "
                         "up to ~1 GB of them)")
    ap.add_argument("--train-run", type=int, default=0,
                    help="instead of the step benchmark, time a whole training run of this many steps with the "
                         "trainer's schedule (density steps every 100 steps in its window, opacity resets) and "
                         "report its steps/s")
    ap.add_argument("--densify-fraction", type=float, default=0.0,
                    help="--train-run stress knob: before each density step scale the accumulated statistics so "
                         "that this fraction of the Gaussians crosses the 2e-4 threshold (default: as trained)")
    ap.add_argument("--clocks-csv", default=None,
                    help="keep the nvidia-smi clock samples in this file ({rank} is replaced; default: a temp file)")
    return ap.parse_args()


# ----------------------------------------------------------------------------- distributed
def dist_setup():
    from mlx_gsplat_b200 import distributed as D
    rank, world, local, pg = D.init_from_env("nccl", timeout_s=180.0)
    torch.cuda.set_device(local)
    return world, rank, local, pg


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices, path: str = None, period_ms: int = 100):
        """One nvidia-smi poller for the GPUs ``gpu_indices`` (local rank 0 samples
        every GPU of the job; the other ranks sample nothing)."""
        self.gpus = list(gpu_indices)
        self.gpu = self.gpus[0] if self.gpus else 0
        self.period_ms = period_ms
        self.proc = None
        self.path = path

    def start(self):
        if not self.gpus:
            return
        try:
            if self.path is None:
                import tempfile
                fd, self.path = tempfile.mkstemp(prefix=f"clocks_gpu{self.gpu}_", suffix=".csv")
                os.close(fd)
            else:
                os.makedirs(os.path.dirname(os.path.abspath(self.path)), exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", ",".join(str(g) for g in self.gpus),
                                          f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms",
                                          str(self.period_ms)], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self, t0: float = None, t1: float = None):
        """Median SM clock and the active throttle reasons over the samples taken
        between host times t0 and t1 (the timed region)."""
        if not self.gpus:
            return None
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        import datetime
        sm, smax, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                mhz = float(parts[2])
                smax = float(parts[3])
                pw = float(parts[4])
            except ValueError:
                continue
            if t0 is not None and not (t0 - 0.06 <= ts <= t1 + 0.06):
                continue
            sm.append(mhz)
            power.append(pw)
            for n, v in zip(names, parts[6:10]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "gpus": self.gpus,
                "power_w_median": float(np.median(power)) if power else None}


# ----------------------------------------------------------------------------- byte model
def kernel_bytes(name: str, N: int, V: int, K: int, P: int, tiles: int, ncols: int, stride: int,
                 sparse_grad: bool = False, grad_row_bytes: float = None) -> float:
    """Algorithmic bytes per launch (what the kernel must move at minimum).  With
    ``sparse_grad`` Adam reads gradient rows only for the V rows the view saw
    (the rest take the regulariser, selected by the cull's visibility bits).
    ``grad_row_bytes``: bytes of one gradient row Adam reads (narrow rows: the
    23 gradient columns and the view count; default full rows)."""
    if name == "adam":
        gb = ncols * 4 if grad_row_bytes is None else grad_row_bytes
        if sparse_grad:
            return N * (ncols * 24 + 4) + V * gb + N / 8
        return N * (ncols * 24 + 4) + N * gb
    if name == "render_fwd":
        return K * (4 + 48) + tiles * 8 + P * (12 + 4 + 4 + 4 + 3)
    if name == "render_bwd":
        return K * (4 + 48) + tiles * 8 + P * (12 + 4 + 4 + 3) + V * 36
    if name == "project_bwd":
        return V * (4 + 4 + 92 + 36 + 4 * ncols + 8)
    if name == "project_fwd":
        return V * (4 + 4 + 92 + 48 + 4 + 4)
    if name == "cull":
        return N * (4 + 16) + V * 4
    if name == "grad_init":
        return N * stride * 4
    return 0.0


def adam_standalone(rows: int, layout, dev, iters: int = 10):
    """The fused slab Adam over ``rows`` pooled rows (one launch per step), timed
    with CUDA events; bytes = rows * (ncols * 28 + 4) (read theta, m, v, g, write
    theta, m, v, read the indirection entry)."""
    from mlx_gsplat_b200.optimizer import FusedMLXAdam
    S = layout.stride
    try:
        th = torch.randn((rows, S), device=dev)
        m = torch.zeros_like(th)
        v = torch.zeros_like(th)
        g = torch.randn_like(th) * 0.01
        table = torch.arange(rows - 1, -1, -1, dtype=torch.int32, device=dev)
    except torch.OutOfMemoryError:
        return None
    lo, hi = layout.col_bounds()
    opt = FusedMLXAdam(lr=1e-3, eps=1e-15)
    for _ in range(3):
        opt.step_slab(th, g, m, v, table, rows, layout.ncols, lo.tolist(), hi.tolist(), quat_col=layout.quat_col)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        opt.step_slab(th, g, m, v, table, rows, layout.ncols, lo.tolist(), hi.tolist(), quat_col=layout.quat_col)
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / iters
    b = rows * (layout.ncols * 28 + 4)
    pk = peaks()["hbm_gbs"]
    del th, m, v, g, table
    torch.cuda.empty_cache()
    return {"rows": rows, "ms": ms, "gbs": b / (ms * 1e-3) / 1e9, "frac": b / (ms * 1e-3) / 1e9 / pk,
            "bytes": b, "inputs": "5.8 GB of slabs > L2"}


def l1_dssim_timing(color, target, dev, iters: int = 20):
    """The L1 + D-SSIM loss kernels (loss and dL/dC) on one rendered image,
    timed with CUDA events; bytes = what they must move (image, target,
    gradient, the three partial maps written and read back)."""
    from mlx_gsplat_b200 import _lib
    lib = _lib.load()
    H, W, _ = color.shape
    out = torch.zeros(2, dtype=torch.float32, device=dev)
    dC = torch.empty_like(color)
    sb = torch.empty(lib.gs_l1_dssim_scratch_bytes(W, H), dtype=torch.uint8, device=dev)

    def run():
        _lib.check(lib.gs_l1_dssim_loss(color.data_ptr(), target.data_ptr(), int(target.dtype == torch.uint8),
                                        W, H, 0.8, 0.2, out.data_ptr(), out[1:].data_ptr(), dC.data_ptr(),
                                        sb.data_ptr(), sb.numel(), _lib.stream_ptr(dev)), "l1+dssim loss")
    for _ in range(3):
        run()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        run()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / iters
    P = H * W
    b = P * (12 + 3) * 2 + P * 12 + P * 36 * 2
    return {"ms": ms, "gbs": b / (ms * 1e-3) / 1e9, "loss": float(out[0]), "ssim": float(out[1]),
            "image": f"{W}x{H}"}


# ----------------------------------------------------------------------------- CPU baseline (oracle)
# fp32 operations one contributing (pixel, splat) pair costs in the compositing
# kernels (fused multiply-adds count 2; the ex2 / reciprocal special functions
# are not counted): forward 21 (offset, quadratic form, falloff argument,
# alpha, weight, colour and alpha sums, transmittance), backward 35 (the same
# recompute, transmittance recovery, the B recursion, colour sums, dL/dalpha
# and the five moments).
FWD_FLOPS_PER_PAIR = 21
BWD_FLOPS_PER_PAIR = 35


def oracle_train_run(wl_name: str = "tiny-3k", steps: int = 50):
    """The reference's training step restated on the CPU (the oracle), run in
    full for ``steps`` steps: cull -> dense rasterizer forward with the L1
    loss gradient in the same pass (fp32 torch-CPU on every host thread) ->
    the trainer's 1e-5 regulariser -> the fused-Adam restatement (C) per group
    with the reference's clamps and learning-rate schedule -> quaternion
    renormalisation.  Targets are rendered from the second seeded set, as the
    GPU runner's are."""
    from mlx_gsplat_b200 import synthetic
    from oracle import adam as oadam
    from oracle import densify as odens
    from oracle import rendering as orend
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    wl = synthetic.WORKLOADS[wl_name]
    g = synthetic.make_gaussians(wl, seed=0)
    views, K = synthetic.make_cameras(wl, seed=2)
    g2 = synthetic.make_gaussians(wl, seed=1)
    cols2 = np.concatenate([g2["sh0"], g2["shN"]], 1)[:, :12 if wl.sh_degree > 0 else 3]
    targets = []
    for vm in views:
        i2 = orend.cull(g2["means"], g2["opacities"], vm, K, wl.width, wl.height).astype(np.int64)
        C, _ = orend.rasterize_dense(g2["means"][i2], g2["quats"][i2], g2["scales"][i2], g2["opacities"][i2],
                                     cols2[i2], vm, K, wl.width, wl.height, wl.width, wl.height, dtype=torch.float32)
        targets.append(C)
    P = {"means": g["means"].copy(), "quats": g["quats"].copy(), "scales": g["scales"].copy(),
         "opacities": g["opacities"].copy(), "colors": np.concatenate([g["sh0"], g["shN"]], 1).astype(np.float32)}
    M = {k: np.zeros_like(v) for k, v in P.items()}
    Vv = {k: np.zeros_like(v) for k, v in P.items()}
    n = P["means"].shape[0]
    table = np.arange(n, dtype=np.int32)
    ncol = 12 if wl.sh_degree > 0 else 3
    reg = np.float32(1e-5)
    t0 = time.perf_counter()
    for step in range(1, steps + 1):
        vi = (step - 1) % len(views)
        ids = orend.cull(P["means"], P["opacities"], views[vi], K, wl.width, wl.height).astype(np.int64)
        _, _, gr = orend.rasterize_dense_vjp(P["means"][ids], P["quats"][ids], P["scales"][ids],
                                             P["opacities"][ids], P["colors"][ids][:, :ncol], views[vi], K,
                                             wl.width, wl.height, wl.width, wl.height, dL_dC=None,
                                             l1_target=targets[vi], dtype=torch.float32, chunk=256)
        grads = {}
        for k in ("means", "quats", "scales", "opacities"):
            gk = np.full_like(P[k], reg)
            gk[ids] += gr[k].astype(np.float32)
            grads[k] = gk
        gc = np.zeros_like(P["colors"])
        gc[ids, :ncol] = gr["colors"].astype(np.float32) + reg
        grads["colors"] = gc
        lr = 1e-3 * (0.01 ** (step / steps))
        for k in P:
            lo, hi = oadam.group_clamp(k if k != "colors" else "sh0")
            oadam.fused_adam_a1(P[k], grads[k], M[k], Vv[k], table, lr=np.float32(lr), beta1=0.9, beta2=0.999,
                                eps=1e-15, weight_decay=0.0, step=step, a_min=lo, a_max=hi)
        P["quats"] = odens.quat_renorm(P["quats"])
    dt = time.perf_counter() - t0
    return {"workload": wl_name, "steps": steps, "seconds": dt, "value": steps / dt, "unit": "train steps/s",
            "mpix_per_s": steps * wl.pixels / dt / 1e6, "cores": threads, "kind": "port",
            "sample": (f"{steps} full training steps of {wl_name} ({n} Gaussians, {len(views)} views at "
                       f"{wl.width}x{wl.height}, L1, fused Adam) through the CPU oracle, fp32 torch-CPU on "
                       f"{threads} threads")}


class OracleSampler:
    """A bounded sample of one training step of a full-size workload through
    the CPU oracle, scaled to the full step.  The dense rasterizer's cost is
    fitted as ``a + b * pixels`` from calls on two pixel-subset sizes over
    every Gaussian the view sees (``a`` is the per-view projection of all of
    them, ``b`` the dense compositing per pixel); Adam is timed on a row slice
    and scaled by rows."""

    def __init__(self, wl_name: str, pix_small: int = 8, pix_large: int = 72, adam_rows: int = 100_000):
        from mlx_gsplat_b200 import synthetic
        from oracle import rendering as orend
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.wl = wl = synthetic.WORKLOADS[wl_name]
        self.wl_name = wl_name
        g = synthetic.make_gaussians(wl, seed=0)
        views, self.K = synthetic.make_cameras(wl, seed=2, num_views=8)
        self.vm = views[0]
        ids = orend.cull(g["means"], g["opacities"], self.vm, self.K, wl.width, wl.height).astype(np.int64)
        cols = np.concatenate([g["sh0"], g["shN"]], 1)[:, :12 if wl.sh_degree > 0 else 3]
        self.rows = {k: np.ascontiguousarray(g[k][ids]) for k in ("means", "quats", "scales", "opacities")}
        self.rows["colors"] = np.ascontiguousarray(cols[ids])
        self.V = len(ids)
        self.ncols = sum(v.shape[1] for k, v in g.items())
        self.n_pix = (pix_small, pix_large)
        self.rng = np.random.default_rng(0)
        self.adam_rows = adam_rows
        r = self.rng
        self.adam = [r.normal(0, 1, (adam_rows, self.ncols)).astype(np.float32),
                     r.normal(0, 0.1, (adam_rows, self.ncols)).astype(np.float32),
                     np.zeros((adam_rows, self.ncols), np.float32), np.zeros((adam_rows, self.ncols), np.float32),
                     np.arange(adam_rows, dtype=np.int32)]
        self.t_small, self.t_large, self.t_adam, self.samples = 0.0, 0.0, 0.0, 0
        self.step = 0

    def _raster(self, n_pix: int) -> float:
        from oracle import rendering as orend
        wl = self.wl
        pix = np.sort(self.rng.choice(wl.pixels, n_pix, replace=False))
        dC = self.rng.uniform(-1, 1, (n_pix, 3)) / wl.pixels
        s = time.perf_counter()
        r = self.rows
        orend.rasterize_dense_vjp(r["means"], r["quats"], r["scales"], r["opacities"], r["colors"], self.vm, self.K,
                                  wl.width, wl.height, wl.width, wl.height, dL_dC=dC, dtype=torch.float32, chunk=8,
                                  pixel_ids=pix)
        return time.perf_counter() - s

    def sample_step(self) -> float:
        """One sample step; returns its seconds."""
        from oracle import adam as oadam
        s0 = time.perf_counter()
        self.t_small += self._raster(self.n_pix[0])
        self.t_large += self._raster(self.n_pix[1])
        self.step += 1
        th, g, m, v, idx = self.adam
        s = time.perf_counter()
        oadam.fused_adam_a1(th, g, m, v, idx, 1e-3, 0.9, 0.999, 1e-15, 0.0, self.step, -1e10, 1e10)
        self.t_adam += time.perf_counter() - s
        self.samples += 1
        return time.perf_counter() - s0

    def full_step_seconds(self) -> float:
        n = max(self.samples, 1)
        ps, pl = self.n_pix
        b = max((self.t_large - self.t_small) / n / (pl - ps), 0.0)
        a = max(self.t_small / n - b * ps, 0.0)
        return a + b * self.wl.pixels + self.t_adam / n * self.wl.num_gaussians / self.adam_rows

    def describe(self) -> str:
        ps, pl = self.n_pix
        return (f"{self.samples} sample steps of {self.wl_name}: the dense oracle fwd+bwd over all {self.V} visible "
                f"Gaussians of one view at {ps} and at {pl} random pixels (fp32 torch-CPU, {self.threads} threads), "
                f"cost fitted as projection + per-pixel compositing and scaled to {self.wl.pixels} pixels, plus the "
                f"C fused-Adam restatement on {self.adam_rows} rows x {self.ncols} columns scaled to "
                f"{self.wl.num_gaussians} rows; extrapolated seconds per full step "
                f"{self.full_step_seconds():.1f}")


def cpu_baseline(wl_name: str, seconds: float):
    """The CPU oracle on the host cores: a bounded sample of the benchmark
    workload scaled to full steps/s (``value``), and the reference's own
    CPU-sized workload (3,000 Gaussians at 120x90, 50 steps) measured in full
    (``config0_measured``)."""
    sampler = OracleSampler(wl_name)
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds or sampler.samples < 2:
        sampler.sample_step()
    t = sampler.full_step_seconds()
    return {"value": 1.0 / t, "unit": "train steps/s", "cores": sampler.threads, "kind": "port",
            "basis": "extrapolated from a bounded sample", "sample": sampler.describe(),
            "config0_measured": oracle_train_run("tiny-3k", 50)}


def workload_config(args, world: int) -> dict:
    """The ``config`` of the JSON line (both arms print the same one)."""
    from mlx_gsplat_b200 import synthetic
    wl = synthetic.WORKLOADS[args.workload]
    return {"workload": args.workload, "gaussians": args.gaussians or wl.num_gaussians,
            "image": f"{wl.width}x{wl.height}", "sh_degree": wl.sh_degree, "views": args.views or wl.num_views,
            "views_per_gpu_per_step": 1, "parallelism": f"views-dp{world}", "loss": "l1",
            "l2": "working set > L2: Adam streams the 1M x 60-float theta/m/v slabs (0.72 GB) and the seen "
                  "gradient rows every step"}


def run_reference(args, world, rank):
    """The reference arm: the reference's training step restated on the CPU
    (the oracle; MLX itself cannot be installed here) on the host cores.
    Each step is a bounded sample of the workload's step (see OracleSampler);
    ``ms_per_step`` is the measured time of one sample step, ``value`` the
    full-step rate the samples extrapolate to."""
    if rank != 0:
        return
    sampler = OracleSampler(args.workload)
    for _ in range(args.warmup):
        sampler.sample_step()
    sampler.t_small = sampler.t_large = sampler.t_adam = 0.0
    sampler.samples = 0
    t_samples = 0.0
    for _ in range(args.steps):
        t_samples += sampler.sample_step()
    full = sampler.full_step_seconds()
    value = 1.0 / full
    base = {"value": value, "unit": "train steps/s", "cores": sampler.threads, "kind": "port",
            "basis": "extrapolated from bounded sample steps", "sample": sampler.describe()}
    if not args.no_cpu_baseline:
        base["config0_measured"] = oracle_train_run("tiny-3k", 50)
    line = {"metric": metric_name(args.workload), "value": value, "unit": "train steps/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * t_samples / args.steps,
            "ms_per_full_step_extrapolated": 1000.0 * full,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference", "config": workload_config(args, world), "cpu_baseline": base,
            "e2e": {"value": value, "unit": "train steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def fp32_peak(dev) -> dict:
    """The GPU's fp32 fused multiply-add throughput (``gs_fp32_peak_probe``, paired
    and scalar forms, best of 5 launches each, CUDA events)."""
    import ctypes
    from mlx_gsplat_b200 import _lib
    lib = _lib.load()
    blocks, iters = 148 * 16, 4096
    out = torch.empty(blocks * 256, dtype=torch.float32, device=dev)
    res = {}
    for paired in (1, 0):
        fl = ctypes.c_double()
        best = None
        for _ in range(6):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            _lib.check(lib.gs_fp32_peak_probe(out.data_ptr(), out.numel(), blocks, iters, paired, ctypes.byref(fl),
                                              _lib.stream_ptr(dev)), "fp32 peak probe")
            e1.record()
            torch.cuda.synchronize(dev)
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        res["paired" if paired else "scalar"] = fl.value / (best * 1e-3) / 1e12
    return {"tflops": max(res.values()), "by_form_tflops": res,
            "how": "gs_fp32_peak_probe: 16 independent FMA chains per thread, 148x16 CTAs of 256 threads"}


def pair_counts(frames, dev) -> float:
    """Mean number of contributing (pixel, splat) pairs per view (the work both
    compositing kernels do) over the given step frames (gs_render_pair_count
    on each frame's staged splats and tile lists)."""
    from mlx_gsplat_b200 import _lib
    lib = _lib.load()
    cnt = torch.zeros(1, dtype=torch.int64, device=dev)
    n = 0
    for f in frames:
        if f.V > 0:
            _lib.check(lib.gs_render_pair_count(f.ranges.data_ptr(), _lib.ptr(f.tile_order), f.entry_vals.data_ptr(),
                                                f.splats.data_ptr(), f.V, f.cam, f.rs, cnt.data_ptr(),
                                                _lib.stream_ptr(dev)), "pair count")
        n += 1
    torch.cuda.synchronize(dev)
    return float(cnt.item()) / max(n, 1)


def train_run(args, runner, targets_dev, n_tgt, view_of, world, rank, dev, clocks):
    """A whole training run with the trainer's schedule (mlx_gsplat/trainer.py:416-425):
    every step a train step, the opacity reset every 1000 (3000) steps, a density
    step every ``refine_every`` steps inside the densify window.  Timed end to
    end with CUDA events (density steps, with their host count read-backs,
    included); one JSON line."""
    import torch.distributed as dist
    from mlx_gsplat_b200 import _lib
    S = args.train_run
    runner.cfg.max_steps = S
    interval = 1000 if S <= 3000 else 3000
    d0 = 300 if S <= 3000 else 500
    d1 = 15000 if S >= 30000 else int(S * 0.7)
    lib = _lib.load()
    for w in range(args.warmup):  # warm-up on a copy-free path: steps of the first view, then restart the count
        runner.train_step(view_of(0), 1, target=targets_dev[view_of(0) % n_tgt])
    runner.allocator.grad2d.zero_()
    runner.allocator.count.zero_()
    barrier(world)
    torch.cuda.synchronize(dev)
    clocks.start()
    launches0 = lib.gs_kernel_launches()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    t_start = time.time()
    e0.record()
    dens = []
    for step in range(1, S + 1):
        runner.train_step(view_of(step), step, target=targets_dev[view_of(step) % n_tgt])
        if step % interval == 0:
            runner.allocator.reset_opacities(-4.59)
        if d0 <= step <= d1 and step % runner.cfg.refine_every == 0:
            if args.densify_fraction > 0:
                runner.scale_densify_stats(args.densify_fraction)
            t0 = time.perf_counter()
            n_p, n_s = runner.densify(step)
            dens.append({"step": step, "pruned": n_p, "refined": n_s, "active": runner.allocator.num_active,
                         "host_ms": (time.perf_counter() - t0) * 1e3})
    e1.record()
    torch.cuda.synchronize(dev)
    t_end = time.time()
    barrier(world)
    clk = clocks.stop(t_start, t_end)
    runner.check_group()
    ms = e0.elapsed_time(e1) / S
    ms_max = max_over_ranks(ms, world)
    if rank == 0:
        from mlx_gsplat_b200 import synthetic
        wl = synthetic.WORKLOADS[args.workload]
        line = {"metric": f"train steps/s over a {S}-step run incl. densify/prune @ {args.workload}",
                "densify_fraction": args.densify_fraction or "as trained",
                "value": world * 1000.0 / ms_max, "unit": "train steps/s", "n_gpus": world, "steps": S,
                "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_config(args, world),
                "pool_slots": runner.allocator.max_gaussians, "density_steps": len(dens),
                "density_host_ms_mean": float(np.mean([d["host_ms"] for d in dens])) if dens else None,
                "active_first_last": [dens[0]["active"], dens[-1]["active"]] if dens else None,
                "densify": dens, "clocks": clk, "gpu_launches": int(lib.gs_kernel_launches() - launches0)}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- main
def main():
    args = parse()
    world, rank, local, pg = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    from mlx_gsplat_b200 import _lib, synthetic
    from mlx_gsplat_b200.rendering import num_tiles
    from mlx_gsplat_b200.trainer import StepTimer, runner_for_workload

    dev = torch.device("cuda", local)
    wl = synthetic.WORKLOADS[args.workload]
    nv = args.views or wl.num_views
    n_init = args.gaussians or wl.num_gaussians
    # a pool with headroom (the trainer's max_gaussians), so a densify step has free slots
    runner = runner_for_workload(args.workload, max_steps=10_000, device=dev, upload_targets=False, lr=1.6e-4,
                                 eps=1e-15, n=args.gaussians, num_views=nv,
                                 max_gaussians=max(wl.capacity or 0, (3 * n_init) // 2),
                                 process_group=pg, fused_reduce=args.multicast,
                                 allreduce_buckets=args.allreduce_buckets,
                                 nccl_sharded_adam=(True if args.sharded_adam else
                                                    (False if args.replicated_adam else None)))
    # the targets: seeded uint8 images, one per view up to ~1 GB of pinned host memory
    # per process, cycled over the views beyond that (the large scene's 512 3840x2160
    # targets alone would take 12.7 GB per process)
    n_tgt = args.target_images or max(1, min(nv, int(1e9 // (wl.pixels * 3))))
    targets_host = torch.from_numpy(synthetic.make_uint8_targets(wl, n_tgt, seed=1)).pin_memory()
    targets_dev = targets_host.to(dev)
    L = runner.layout
    P = wl.pixels
    tx, ty = num_tiles(wl.width, wl.height)

    def view_of(step):
        return (rank + world * step) % nv

    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    clocks = ClockSampler(range(local_world) if local == 0 else [],
                          args.clocks_csv.format(rank=local) if args.clocks_csv else None)
    if args.train_run:
        return train_run(args, runner, targets_dev, n_tgt, view_of, world, rank, dev, clocks)
    clocks.start()
    step = 0
    for _ in range(args.warmup):
        step += 1
        runner.train_step(view_of(step), step, target=targets_dev[view_of(step) % n_tgt])
    torch.cuda.synchronize(dev)

    # ---- timed region: inputs resident in HBM
    lib = _lib.load()
    launches0 = lib.gs_kernel_launches()
    timers = []
    stats = []
    barrier(world)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    t_start = time.time()
    e0.record()
    for _ in range(args.steps):
        step += 1
        tm = StepTimer()
        f = runner.train_step(view_of(step), step, target=targets_dev[view_of(step) % n_tgt], timer=tm)
        timers.append(tm)
        stats.append((f.V, f.K))
    e1.record()
    torch.cuda.synchronize(dev)
    t_end = time.time()
    barrier(world)
    clk = clocks.stop(t_start, t_end)
    if runner.fused_reduce is not None:
        runner.fused_reduce.check()  # a barrier that timed out invalidates the run
    launches = lib.gs_kernel_launches() - launches0
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(ms, world)
    value = world * 1000.0 / ms_max

    # per-kernel durations over the timed steps
    phase = {}
    for tm in timers:
        for k, v in tm.durations().items():
            phase[k] = phase.get(k, 0.0) + v / len(timers)
    Vm = float(np.mean([s[0] for s in stats]))
    Km = float(np.mean([s[1] for s in stats]))
    N = runner.allocator.num_active
    # the part of each step before the gradient sum, per rank: the sum waits for
    # the slowest rank's view, so the spread is part of the collective's phase
    pre = ("cull", "project_fwd", "depth_sort+offsets", "bin+tile_sort", "render_fwd", "render_bwd", "project_bwd")
    pre_steps = [sum(tm.durations().get(k, 0.0) for k in pre) for tm in timers]
    per_rank = {"mean_ms": float(np.mean(pre_steps))}
    if world > 1:
        import torch.distributed as dist
        allr = [None] * world
        dist.all_gather_object(allr, pre_steps)
        arr = np.array(allr)  # [rank, step]
        per_rank = {"mean_ms_by_rank": [round(float(x), 4) for x in arr.mean(1)],
                    "mean_over_steps_of_max_minus_mean_ms": float(np.mean(arr.max(0) - arr.mean(0)))}
    kernels = ["render_fwd", "render_bwd", "project_bwd", "project_fwd", "adam", "cull", "grad_init"]
    per = {}
    for k in kernels:
        if k in phase and phase[k] > 0:
            b = kernel_bytes(k, N, Vm, Km, P, tx * ty, L.ncols, L.stride,
                             sparse_grad=runner.row_mode == "sparse", grad_row_bytes=4 * (runner.g_cols + 1)
                             if runner.g_cols < L.ncols else None)
            per[k] = {"ms": phase[k], "gbs": b / (phase[k] * 1e-3) / 1e9, "bytes": b}
    pk = peaks()
    dom = max(per, key=lambda k: per[k]["ms"])
    full_size = args.gaussians is None and args.views is None
    roof = {"bound": "hbm", "kernel": dom, "achieved": per[dom]["gbs"], "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": per[dom]["gbs"] / pk["hbm_gbs"], "peak_src": pk["src"] + " MEASURED_PEAKS.json hbm_gbs",
            "traffic": measured_traffic(dom, args.workload) if full_size else None,
            "bytes_per_launch": per[dom]["bytes"],
            "limiter": LIMITERS.get(dom, "hbm")}
    if "adam" in per:
        roof["adam"] = {"achieved": per["adam"]["gbs"], "frac": per["adam"]["gbs"] / pk["hbm_gbs"],
                        "traffic": measured_traffic("adam", args.workload) if full_size else None}
    # compute roofline of the compositing kernels: contributing (pixel, splat) pairs
    # times the fp32 operations per pair, against the measured fp32 throughput
    # (on four more steps' frames, after the timed region)
    pairs = 0.0
    for _ in range(4):
        step += 1
        f = runner.train_step(view_of(step), step, target=targets_dev[view_of(step) % n_tgt])
        pairs += pair_counts([f], dev) / 4
        del f
    fp = fp32_peak(dev)
    comp = {"pairs_per_view": pairs, "peak_tflops": fp["tflops"], "peak_by_form_tflops": fp["by_form_tflops"],
            "peak_how": fp["how"], "flops_per_pair": {"render_fwd": FWD_FLOPS_PER_PAIR,
                                                      "render_bwd": BWD_FLOPS_PER_PAIR}}
    for k, fl in (("render_fwd", FWD_FLOPS_PER_PAIR), ("render_bwd", BWD_FLOPS_PER_PAIR)):
        if k in per:
            tf = pairs * fl / (per[k]["ms"] * 1e-3) / 1e12
            comp[k] = {"ms": per[k]["ms"], "gpairs_per_s": pairs / (per[k]["ms"] * 1e-3) / 1e9,
                       "achieved_tflops": tf, "frac": tf / fp["tflops"]}
    roof["fp32"] = comp

    # ---- end to end through the public API (host target in, loss out)
    e2e = None
    if not args.no_e2e:
        # Each step's target comes from pinned host memory into one of two device
        # staging buffers on a copy stream, issued one step ahead so that the
        # upload overlaps the previous step's compute (the compute stream waits
        # for the copy; the copy into a buffer waits until the step two back,
        # which read it, is done).
        stages = [torch.empty_like(targets_dev[0]) for _ in range(2)]
        copy_stream = torch.cuda.Stream(dev)
        copied = [torch.cuda.Event(), torch.cuda.Event()]
        consumed = [torch.cuda.Event(), torch.cuda.Event()]
        # every step's loss is copied to pinned host memory and read by the host
        # two steps later (two slots), so the read does not idle the GPU
        loss_host = torch.empty(2, dtype=torch.float32, pin_memory=True)
        loss_ready = [torch.cuda.Event(), torch.cuda.Event()]

        # the same camera views as the timed loop above (views differ in their
        # visible and tile-entry counts, so a different sample of views would
        # measure different work)
        timed_views = [view_of(s) for s in range(args.warmup + 1, args.warmup + 1 + args.steps)]

        def upload(i, first):
            b = i % 2
            with torch.cuda.stream(copy_stream):
                if not first:
                    copy_stream.wait_event(consumed[b])
                stages[b].copy_(targets_host[timed_views[i % len(timed_views)] % n_tgt], non_blocking=True)
                copied[b].record(copy_stream)

        def e2e_steps(k):
            nonlocal step
            out = []
            upload(0, True)
            for i in range(k):
                step += 1
                v = timed_views[i % len(timed_views)]
                b = i % 2
                if i + 1 < k:
                    upload(i + 1, i < 1)  # the next step's target, behind this one's compute
                torch.cuda.current_stream(dev).wait_event(copied[b])
                runner.train_step(v, step, target=stages[b])
                consumed[b].record()
                slot = i % 2
                if i >= 2:
                    loss_ready[slot].synchronize()
                    out.append(float(loss_host[slot]))
                loss_host[slot:slot + 1].copy_(runner.loss_value().reshape(1), non_blocking=True)
                loss_ready[slot].record()
            return out

        # untimed warm-up of this loop too: its first pinned-memory copies carry
        # a one-time cost (~30 ms measured on 2 GPUs)
        e2e_steps(args.warmup)
        torch.cuda.synchronize(dev)
        barrier(world)
        torch.cuda.synchronize(dev)
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record()
        losses = e2e_steps(args.steps)
        a1.record()
        torch.cuda.synchronize(dev)
        for i in range(max(args.steps - 2, 0), args.steps):
            losses.append(float(loss_host[i % 2]))
        assert len(losses) == args.steps and all(np.isfinite(losses))
        barrier(world)
        ms_e2e = max_over_ranks(a0.elapsed_time(a1) / args.steps, world)
        e2e = {"value": world * 1000.0 / ms_e2e, "unit": "train steps/s", "ms_per_step": ms_e2e,
               "h2d_bytes_per_step": int(stages[0].numel()), "d2h_bytes_per_step": 4,
               "h2d": "pinned host -> device on a copy stream, one step ahead of the compute"}

    # ---- three densify/prune steps on this scene, two training steps apart (all ranks:
    # the statistics are all-reduced); the first also allocates the density-step workspace
    densify_ms = None
    if not args.no_extras:
        al = runner.allocator
        rounds = []
        gen = torch.Generator(device=dev)
        gen.manual_seed(5)
        try:
            for rnd in range(3):
                for _ in range(2):
                    step += 1
                    runner.train_step(view_of(step), step, target=targets_dev[view_of(step) % n_tgt])
                # statistics with mean 1e-4: about e^-2 = 13.5% of the Gaussians exceed the 2e-4 threshold
                al.grad2d.exponential_(1e4, generator=gen)
                al.count.fill_(1.0)
                barrier(world)
                torch.cuda.synchronize(dev)
                t0 = time.perf_counter()
                n_p, n_s = runner.densify(step + 1)
                torch.cuda.synchronize(dev)
                rounds.append({"ms": (time.perf_counter() - t0) * 1e3, "pruned": n_p, "refined": n_s,
                               "active_after": al.num_active})
            densify_ms = {"rounds": rounds, "ms_after_first": float(np.mean([r["ms"] for r in rounds[1:]])),
                          "note": "wall clock incl. the host count read-back; the first round allocates the "
                                  "density-step workspace"}
        except MemoryError as e:
            densify_ms = {"error": str(e), "rounds": rounds}

    # ---- the large workload's standalone fused Adam: 6M rows x 59 columns, theta/m/v/g
    # ---- the reference trainer's L1 + D-SSIM image loss (forward + gradient) on this image size
    l1_dssim = None
    if not args.no_extras:
        l1_dssim = l1_dssim_timing(runner.last_frame.color, targets_dev[0], dev)
    adam_6m = None
    if world == 1 and not args.no_extras:
        adam_6m = adam_standalone(6_000_000, L, dev)

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = cpu_baseline(args.workload, args.cpu_seconds)

    if rank == 0:
        line = {"metric": metric_name(args.workload), "value": value,
                "unit": "train steps/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic",
                "config": workload_config(args, world),
                "grad_reduce": ("nvlink multicast sum fused into the sharded adam" if runner.sharded else
                                ("nvlink multicast row sum" if runner.fused_reduce is not None else
                                 ("nccl reduce-scatter, adam on 1/N of the rows, all-gather of the rasterizer's "
                                  "columns" if runner.sharded_nccl else
                                  (f"nccl all-reduce in {runner.cfg.allreduce_buckets} row ranges, pipelined with "
                                   "the replicated adam" if world > 1 else "none")))),
                "grad_row_floats": runner.g_stride,
                "before_sum_ms": per_rank,
                "mpix_per_s": value * P / 1e6, "visible_mean": Vm, "entries_mean": Km,
                "adam_gbs": per.get("adam", {}).get("gbs"),
                "kernels_ms": {k: round(v["ms"], 4) for k, v in per.items()},
                "phases_ms": {k: round(v, 4) for k, v in phase.items()},
                "roofline": roof, "clocks": clk, "e2e": e2e, "cpu_baseline": base,
                "densify": densify_ms, "adam_6m": adam_6m, "l1_dssim_loss": l1_dssim,
                "gpu_launches": int(launches)}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
