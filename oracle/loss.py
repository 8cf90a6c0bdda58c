"""CPU restatement of the reference trainer's image loss — TEST INFRASTRUCTURE ONLY
(the checker for the GPU loss kernels; nothing on the product path imports it).

* ``ssim``: ``mlx_gsplat/trainer.py:164-190`` — per channel, the 11x11 window
  of ones / 121 applied with zero padding 5 (a grouped convolution) to C, T,
  C*C, T*T and C*T; sigma terms as differences with the squared means;
  C1 = 0.01^2, C2 = 0.03^2; the mean of the SSIM map over pixels and channels.
* ``l1_dssim_loss``: ``trainer.py:276-279`` — 0.8 * mean|C - T| +
  0.2 * 0.5 * (1 - SSIM(C, T)), and its gradient with respect to C (torch
  autograd).

Images are HWC.  Pinned against fixtures produced by the reference's own
``_ssim`` (``tests/golden/gen_golden.py``).
"""
from __future__ import annotations

from typing import Tuple

import numpy as np
import torch
import torch.nn.functional as F

WINDOW = 11
C1 = 0.01 ** 2
C2 = 0.03 ** 2


def _box(x: torch.Tensor) -> torch.Tensor:
    """[1, 3, H, W] -> the same, each channel convolved with ones(11, 11) / 121."""
    w = torch.ones((3, 1, WINDOW, WINDOW), dtype=x.dtype) / (WINDOW * WINDOW)
    return F.conv2d(x, w, padding=WINDOW // 2, groups=3)


def ssim(c: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
    x1 = c.permute(2, 0, 1)[None]
    x2 = t.permute(2, 0, 1)[None]
    mu1, mu2 = _box(x1), _box(x2)
    mu1_sq, mu2_sq, mu1_mu2 = mu1 * mu1, mu2 * mu2, mu1 * mu2
    s1 = _box(x1 * x1) - mu1_sq
    s2 = _box(x2 * x2) - mu2_sq
    s12 = _box(x1 * x2) - mu1_mu2
    m = ((2 * mu1_mu2 + C1) * (2 * s12 + C2)) / ((mu1_sq + mu2_sq + C1) * (s1 + s2 + C2))
    return torch.mean(m)


def l1_dssim_loss(c: np.ndarray, t: np.ndarray, w_l1: float = 0.8, w_dssim: float = 0.2,
                  dtype=torch.float64) -> Tuple[float, float, np.ndarray]:
    """Returns (loss, ssim, dloss/dC) for HWC images ``c`` (rendered) and ``t``."""
    ct = torch.tensor(np.asarray(c), dtype=dtype, requires_grad=True)
    tt = torch.tensor(np.asarray(t), dtype=dtype)
    s = ssim(ct, tt)
    loss = w_l1 * torch.mean(torch.abs(ct - tt)) + w_dssim * 0.5 * (1.0 - s)
    (g,) = torch.autograd.grad(loss, ct)
    return float(loss), float(s.detach()), g.numpy()
