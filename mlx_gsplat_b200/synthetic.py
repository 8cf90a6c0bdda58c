"""Seeded synthetic scenes, cameras and targets for the benchmark workloads.

The reference trains on COLMAP scenes (``mlx_gsplat/dataset.py``) or, when no
scene is present, on a synthetic 3,000-point cloud (``mlx_gsplat/trainer.py:121-136``).
No dataset is available here, so every workload is drawn from seeded NumPy
generators with the shapes and value distributions of the five workloads:

===========  ==========  =====  =====  ===========  ======  =====================
workload     Gaussians   SH     views  image        focal   camera ring
===========  ==========  =====  =====  ===========  ======  =====================
tiny-3k      3,000       0      8      120x90       100     r=4, h=0.5
mid-200k     200,000     0      32     648x420      500     r=4, h=0.5
outdoor-1m   1,000,000   3      160    1297x840     1150    r=6, h ~ N(0, 0.5)
densify-4m   300k/4M     3      256    1920x1080    1600    r=6, h ~ N(0, 0.5)
large-6m     6,000,000   3      512    3840x2160    3200    r=18, h ~ N(0, 1.5)
===========  ==========  =====  =====  ===========  ======  =====================

Conventions: world up is +z; cameras are OpenCV world-to-camera matrices
(+x right, +y down, +z forward) looking at the origin.  Colours are stored as
SH coefficients (DC first, then the rest), so an RGB value ``c`` is stored as
``(c - 0.5) / SH_C0`` (``mlx_gsplat/trainer.py:105-107``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

SH_C0 = 0.28209479177387814


@dataclass
class Workload:
    name: str
    num_gaussians: int
    sh_degree: int
    num_views: int
    width: int
    height: int
    focal: float
    ring_radius: float
    ring_height: float
    height_jitter: float
    mean_kind: str          # "cube" | "mixture"
    mean_extent: float      # cube half-size, or mixture scale multiplier
    log_scale_mu: float
    log_scale_sigma: float
    opac_mu: float
    opac_sigma: float
    color_kind: str         # "rgb_sigmoid" | "sh_normal"
    target_kind: str        # "render" | "uint8"
    capacity: Optional[int] = None
    extra: Dict[str, float] = field(default_factory=dict)

    @property
    def pixels(self) -> int:
        return self.width * self.height

    @property
    def sh_dim(self) -> int:
        return 3 * (self.sh_degree + 1) ** 2


WORKLOADS: Dict[str, Workload] = {
    "tiny-3k": Workload("tiny-3k", 3000, 0, 8, 120, 90, 100.0, 4.0, 0.5, 0.0,
                        "cube", 1.0, -3.0, 0.3, 0.0, 1.0, "rgb_sigmoid", "render"),
    "mid-200k": Workload("mid-200k", 200_000, 0, 32, 648, 420, 500.0, 4.0, 0.5, 0.0,
                         "cube", 3.0, -4.0, 0.5, 0.0, 1.0, "rgb_sigmoid", "uint8"),
    "outdoor-1m": Workload("outdoor-1m", 1_000_000, 3, 160, 1297, 840, 1150.0, 6.0, 0.0, 0.5,
                           "mixture", 1.0, -4.5, 0.7, -1.0, 1.5, "sh_normal", "uint8"),
    "densify-4m": Workload("densify-4m", 300_000, 3, 256, 1920, 1080, 1600.0, 6.0, 0.0, 0.5,
                           "mixture", 1.0, -4.5, 0.7, -1.0, 1.5, "sh_normal", "uint8",
                           capacity=4_000_000),
    "large-6m": Workload("large-6m", 6_000_000, 3, 512, 3840, 2160, 3200.0, 18.0, 0.0, 1.5,
                         "mixture", 3.0, -4.5, 0.7, -1.0, 1.5, "sh_normal", "uint8"),
}


def _unit_quats(rng: np.random.Generator, n: int) -> np.ndarray:
    q = rng.standard_normal((n, 4)).astype(np.float32)
    return (q / np.linalg.norm(q, axis=1, keepdims=True)).astype(np.float32)


def make_gaussians(wl: Workload, seed: int = 0, n: Optional[int] = None) -> Dict[str, np.ndarray]:
    """Draw one seeded Gaussian set: ``means [n,3], quats [n,4], scales [n,3]``
    (log-scale), ``opacities [n,1]`` (logit), ``sh0 [n,3]``, ``shN [n, 3*((d+1)^2-1)]``."""
    rng = np.random.default_rng(seed)
    n = wl.num_gaussians if n is None else int(n)
    if wl.mean_kind == "cube":
        means = rng.uniform(-wl.mean_extent, wl.mean_extent, (n, 3))
    else:
        n_core = int(round(0.7 * n))
        core = rng.normal(0.0, 2.0, (n_core, 3))
        d = rng.standard_normal((n - n_core, 3))
        shell = 20.0 * d / np.linalg.norm(d, axis=1, keepdims=True)
        means = np.concatenate([core, shell], 0)[rng.permutation(n)] * wl.mean_extent
    means = means.astype(np.float32)
    scales = rng.normal(wl.log_scale_mu, wl.log_scale_sigma, (n, 3)).astype(np.float32)
    quats = _unit_quats(rng, n)
    opac = rng.normal(wl.opac_mu, wl.opac_sigma, (n, 1)).astype(np.float32)
    n_rest = 3 * ((wl.sh_degree + 1) ** 2 - 1)
    if wl.color_kind == "rgb_sigmoid":
        rgb = 1.0 / (1.0 + np.exp(-rng.standard_normal((n, 3))))
        sh0 = ((rgb - 0.5) / SH_C0).astype(np.float32)
        shN = np.zeros((n, n_rest), np.float32)
    else:
        sh = rng.normal(0.0, 0.1, (n, 3 + n_rest)).astype(np.float32)
        sh0, shN = sh[:, :3].copy(), sh[:, 3:].copy()
    return {"means": means, "quats": quats, "scales": scales, "opacities": opac,
            "sh0": sh0, "shN": shN}


def look_at_w2c(cam_pos: np.ndarray) -> np.ndarray:
    """OpenCV world-to-camera matrix for a camera at ``cam_pos`` looking at the
    origin with world +z up."""
    c = np.asarray(cam_pos, np.float64)
    f = -c / np.linalg.norm(c)
    up = np.array([0.0, 0.0, 1.0])
    right = np.cross(f, up)
    if np.linalg.norm(right) < 1e-8:
        right = np.array([1.0, 0.0, 0.0])
    right /= np.linalg.norm(right)
    down = np.cross(f, right)
    R_c2w = np.stack([right, down, f], axis=1)
    w2c = np.eye(4)
    w2c[:3, :3] = R_c2w.T
    w2c[:3, 3] = -R_c2w.T @ c
    return w2c.astype(np.float32)


def make_cameras(wl: Workload, seed: int = 2, num_views: Optional[int] = None):
    """Ring cameras: returns ``(viewmats [V,4,4], K [3,3])`` as float32."""
    rng = np.random.default_rng(seed)
    nv = wl.num_views if num_views is None else int(num_views)
    az = 2.0 * np.pi * np.arange(nv) / nv
    h = wl.ring_height + (rng.normal(0.0, wl.height_jitter, nv) if wl.height_jitter > 0 else np.zeros(nv))
    views = np.stack([look_at_w2c(np.array([wl.ring_radius * np.cos(a), wl.ring_radius * np.sin(a), hh]))
                      for a, hh in zip(az, h)])
    K = np.array([[wl.focal, 0.0, wl.width / 2.0],
                  [0.0, wl.focal, wl.height / 2.0],
                  [0.0, 0.0, 1.0]], np.float32)
    return views.astype(np.float32), K


def scene_scale(viewmats: np.ndarray) -> float:
    """Scene extent from the cameras (mlx_gsplat/dataset.py:404-408): the largest
    distance of a camera centre from the mean centre."""
    v = np.asarray(viewmats, np.float64)
    centres = np.stack([-(m[:3, :3].T @ m[:3, 3]) for m in v])
    return float(np.max(np.linalg.norm(centres - centres.mean(0), axis=1)))


def make_uint8_targets(wl: Workload, num: int, seed: int = 1) -> np.ndarray:
    """Seeded random uint8 RGB images ``[num, H, W, 3]``."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, (num, wl.height, wl.width, 3), dtype=np.uint8)


def colors_for_degree(g: Dict[str, np.ndarray], degree: int) -> np.ndarray:
    """The trainer's SH gather (``mlx_gsplat/trainer.py:239-250``): DC plus the
    first ``3*((d+1)^2-1)`` rest coefficients."""
    k = 3 * ((degree + 1) ** 2 - 1)
    return np.concatenate([g["sh0"], g["shN"][:, :k]], axis=1).astype(np.float32)


def list_workloads() -> List[str]:
    return list(WORKLOADS.keys())
