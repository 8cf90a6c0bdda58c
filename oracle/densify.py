"""Trainer-side policy oracles — TEST INFRASTRUCTURE ONLY.

NumPy float32 restatements of mlx_gsplat/trainer.py:

* ``grad2d_proxy``      — :300-318, ``sqrt(sum(dL/dmean^2) + 1e-8) * |z_cam| / fx``
  scatter-added into ``grad2d`` (and ``count += 1``) at the visible physical slots.
* ``densify_masks``     — :428-477, the grow (clone/split) and prune decisions.
* ``child_params``      — :479-507, child values given the noise draws
  (``noise_means1``, ``noise_means2``, ``noise_quats2``; the reference draws
  them with ``mx.random.normal`` in that order).
* ``quat_renorm``       — :380-387.
* ``densify_window`` / ``opacity_reset_interval`` / ``lr_at`` — :358, :416-425.
"""
from __future__ import annotations

from typing import Dict, Tuple

import numpy as np

f32 = np.float32


def lr_at(lr: float, step: int, max_steps: int) -> float:
    """trainer.py:358 (float64 Python arithmetic)."""
    return lr * (0.01 ** (step / max_steps))


def opacity_reset_interval(max_steps: int) -> int:
    return 1000 if max_steps <= 3000 else 3000


def densify_window(max_steps: int) -> Tuple[int, int]:
    start = 300 if max_steps <= 3000 else 500
    end = 15000 if max_steps >= 30000 else int(max_steps * 0.7)
    return start, end


def is_densify_step(step: int, max_steps: int, refine_every: int = 100) -> bool:
    s, e = densify_window(max_steps)
    return s <= step <= e and step % refine_every == 0


def grad2d_proxy(grad_means_visible: np.ndarray, means_visible: np.ndarray, viewmat: np.ndarray,
                 fx: float) -> np.ndarray:
    """Per visible Gaussian: ``sqrt(sum(g^2) + 1e-8) * |z| / fx`` (float32)."""
    g = np.asarray(grad_means_visible, f32)
    m = np.asarray(means_visible, f32)
    v = np.asarray(viewmat, f32)
    z = ((m[:, 0] * v[2, 0] + m[:, 1] * v[2, 1]) + m[:, 2] * v[2, 2]) + v[2, 3]
    norm = np.sqrt(np.sum(g * g, axis=1) + f32(1e-8))
    return (norm * np.abs(z) / f32(fx)).astype(f32)


def densify_masks(grad2d_active: np.ndarray, count_active: np.ndarray, scales: np.ndarray,
                  opacities: np.ndarray, means: np.ndarray, quats: np.ndarray, scene_scale: float,
                  num_active: int, grad_threshold: float = 0.0002, min_active_for_prune: int = 80000):
    """trainer.py:435-477.  Returns ``(refine_mask, split_mask, prune_mask)``
    where ``refine = duplicate | split`` is what the allocator receives as its
    split mask and ``split`` marks the scale-shrinking subset."""
    avg = (np.asarray(grad2d_active, f32) / np.maximum(np.asarray(count_active, f32), f32(1.0))).astype(f32)
    high = avg > f32(grad_threshold)
    smax = np.exp(np.asarray(scales, f32)).max(axis=1)
    small = smax <= 0.01 * scene_scale
    dup = high & small
    split = high & ~small
    refine = dup | split
    raw_op = (f32(1.0) / (f32(1.0) + np.exp(-np.asarray(opacities, f32)))).reshape(-1)
    too_dim = raw_op < f32(0.005)
    too_large = smax > 0.1 * scene_scale
    nan_mask = (~np.isfinite(scales).all(axis=1) | ~np.isfinite(opacities).reshape(-1)
                | ~np.isfinite(means).all(axis=1))
    qn = np.sqrt(np.sum(np.asarray(quats, f32) * np.asarray(quats, f32), axis=1))
    bad_quat = np.abs(qn - f32(1.0)) > f32(5e-2)
    prune = too_dim | too_large | nan_mask | bad_quat
    if num_active < min_active_for_prune:
        prune = nan_mask | bad_quat
    return refine, split, prune


def child_params(active: Dict[str, np.ndarray], refine_mask: np.ndarray, split_mask: np.ndarray,
                 noise_means1: np.ndarray, noise_means2: np.ndarray, noise_quats2: np.ndarray
                 ) -> Dict[str, np.ndarray]:
    """trainer.py:479-507.  ``active`` holds the gathered active rows per group."""
    ridx = np.where(refine_mask)[0]
    out = {}
    split_in_refine = np.asarray(split_mask)[ridx][:, None]
    for name, vals in active.items():
        p = np.asarray(vals, f32)[ridx]
        if name == "means":
            out["means_child1"] = p + np.asarray(noise_means1, f32) * f32(0.02)
            out["means_child2"] = p + np.asarray(noise_means2, f32) * f32(0.02)
        elif name == "scales":
            cs = p - np.where(split_in_refine, f32(np.log(1.6)), f32(0.0))
            out["scales_child1"] = cs.astype(f32)
            out["scales_child2"] = cs.astype(f32)
        elif name == "opacities":
            out["opacities_child1"] = p * f32(0.95)
            out["opacities_child2"] = p * f32(0.95)
        elif name == "quats":
            c2 = p + np.asarray(noise_quats2, f32) * f32(0.01)
            out["quats_child1"] = p / np.sqrt(np.sum(p * p, axis=1, keepdims=True) + f32(1e-8))
            out["quats_child2"] = c2 / np.sqrt(np.sum(c2 * c2, axis=1, keepdims=True) + f32(1e-8))
        else:
            out[f"{name}_child1"] = p.copy()
            out[f"{name}_child2"] = p.copy()
    return out


def quat_renorm(q: np.ndarray) -> np.ndarray:
    q = np.asarray(q, f32)
    return (q / np.sqrt(np.sum(q * q, axis=1, keepdims=True) + f32(1e-8))).astype(f32)


def scene_scale_from_cameras(viewmats: np.ndarray) -> float:
    """dataset.py:404-408 on world-to-camera matrices (camera centres ``-R^T t``)."""
    c = np.stack([-(v[:3, :3].T @ v[:3, 3]) for v in np.asarray(viewmats, np.float64)])
    return float(np.max(np.linalg.norm(c - c.mean(0), axis=1)))
