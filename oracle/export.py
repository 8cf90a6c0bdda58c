"""CPU restatement of the reference trainer's PLY export — TEST INFRASTRUCTURE
ONLY (the checker for ``RunnerMLX.export_to_ply``).

``mlx_gsplat/trainer.py:570-631``: the active parameters, quaternions divided
by (norm + 1e-8), log-scales clipped to [-10, -2] and opacity logits to
[-5, 2], concatenated as means | zero normals | sh0 | shN | opacity | scales |
quats and written as a binary little-endian PLY with the reference's header.
"""
from __future__ import annotations

from typing import Dict

import numpy as np


def ply_bytes(active: Dict[str, np.ndarray]) -> bytes:
    means = np.asarray(active["means"], np.float32)
    scales = np.asarray(active["scales"], np.float32)
    quats = np.asarray(active["quats"], np.float32)
    opacities = np.asarray(active["opacities"], np.float32)
    sh0 = np.asarray(active["sh0"], np.float32)
    shN = np.asarray(active["shN"], np.float32)
    n = means.shape[0]
    quats = quats / (np.linalg.norm(quats, axis=-1, keepdims=True) + 1e-8)
    scales = np.clip(scales, -10.0, -2.0)
    opacities = np.clip(opacities, -5.0, 2.0)
    arr = np.concatenate([means, np.zeros((n, 3), np.float32), sh0, shN, opacities, scales, quats], axis=-1)
    head = [b"ply\n", b"format binary_little_endian 1.0\n", f"element vertex {n}\n".encode()]
    head += [f"property float {p}\n".encode() for p in ("x", "y", "z", "nx", "ny", "nz")]
    head += [f"property float f_dc_{j}\n".encode() for j in range(sh0.shape[1])]
    head += [f"property float f_rest_{j}\n".encode() for j in range(shN.shape[1])]
    head += [b"property float opacity\n"]
    head += [f"property float scale_{i}\n".encode() for i in range(scales.shape[1])]
    head += [f"property float rot_{i}\n".encode() for i in range(quats.shape[1])]
    head += [b"end_header\n"]
    return b"".join(head) + arr.astype(np.float32).tobytes()
