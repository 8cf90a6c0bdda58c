"""CPU restatement of the target resize — TEST INFRASTRUCTURE ONLY.

``bilinear_resize`` follows ``bilinear_resize_mlx`` (mlx_gsplat/rendering.py:6-38)
in NumPy float32, one rounded operation at a time in the reference's order;
``target_from_u8`` is the trainer's ``image / 255.0`` (mlx_gsplat/trainer.py:369)
followed by that resize (trainer.py:231-234).
"""
from __future__ import annotations

import numpy as np


def bilinear_resize(img: np.ndarray, H_out: int, W_out: int) -> np.ndarray:
    f32 = np.float32
    img = np.asarray(img, f32)
    H_in, W_in, _ = img.shape
    xs = np.arange(W_out, dtype=f32)
    ys = np.arange(H_out, dtype=f32)
    xs_in = xs * f32((W_in - 1) / max(1, W_out - 1))
    ys_in = ys * f32((H_in - 1) / max(1, H_out - 1))
    x0 = np.floor(xs_in).astype(np.int32)
    x1 = np.minimum(x0 + 1, W_in - 1)
    y0 = np.floor(ys_in).astype(np.int32)
    y1 = np.minimum(y0 + 1, H_in - 1)
    wx = (xs_in - x0.astype(f32)).reshape(1, W_out, 1)
    wy = (ys_in - y0.astype(f32)).reshape(H_out, 1, 1)
    r0, r1 = img[y0], img[y1]
    c00, c10, c01, c11 = r0[:, x0], r0[:, x1], r1[:, x0], r1[:, x1]
    one = f32(1.0)
    top = (one - wx) * c00 + wx * c10
    bottom = (one - wx) * c01 + wx * c11
    return ((one - wy) * top + wy * bottom).astype(f32)


def target_from_u8(img_u8: np.ndarray, H_out: int, W_out: int) -> np.ndarray:
    return bilinear_resize(np.asarray(img_u8).astype(np.float32) / np.float32(255.0), H_out, W_out)
