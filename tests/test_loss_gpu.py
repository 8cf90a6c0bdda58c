"""The L1 + D-SSIM image loss kernels (``gs_l1_dssim_loss``) against the
reference-generated fixtures and the oracle (float64 torch-CPU restatement of
``mlx_gsplat/trainer.py:164-190, 276-279``).  Loss 1e-5 relative, gradient
``assert_grad_close`` (1e-3 relative)."""
import os

import numpy as np
import pytest
import torch

from gsutil import assert_grad_close
from mlx_gsplat_b200 import _lib
from oracle import loss as oloss

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _gpu_loss(c, t):
    lib = _lib.lib()
    H, W, _ = c.shape
    C = torch.from_numpy(np.ascontiguousarray(c)).to(DEV)
    T = torch.from_numpy(np.ascontiguousarray(t)).to(DEV)
    out = torch.zeros(2, dtype=torch.float32, device=DEV)
    dC = torch.empty_like(C)
    sb = torch.empty(lib.gs_l1_dssim_scratch_bytes(W, H), dtype=torch.uint8, device=DEV)
    _lib.check(lib.gs_l1_dssim_loss(C.data_ptr(), T.data_ptr(), int(T.dtype == torch.uint8), W, H, 0.8, 0.2,
                                    out.data_ptr(), out[1:].data_ptr(), dC.data_ptr(), sb.data_ptr(), sb.numel(),
                                    _lib.stream_ptr()))
    torch.cuda.synchronize()
    return float(out[0]), float(out[1]), dC.cpu().numpy()


def test_matches_reference_fixtures(golden_dir):
    d = np.load(os.path.join(golden_dir, "ssim.npz"))
    for i in range(3):
        loss, ssim, g = _gpu_loss(d[f"c_{i}"], d[f"t_{i}"])
        np.testing.assert_allclose(ssim, float(d[f"ssim_{i}"]), rtol=1e-5)
        np.testing.assert_allclose(loss, float(d[f"loss_{i}"]), rtol=1e-5)
        assert_grad_close(g, d[f"grad_{i}"], what=f"case {i}")


@pytest.mark.parametrize("h,w,u8", [(45, 77, True), (90, 120, False), (840, 1297, True)])
def test_matches_oracle(h, w, u8):
    rng = np.random.default_rng(h * w)
    c = rng.uniform(0, 1, (h, w, 3)).astype(np.float32)
    if u8:
        t = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
        tf = t.astype(np.float32) / np.float32(255.0)
    else:
        t = np.clip(c + rng.normal(0, 0.1, c.shape), 0, 1).astype(np.float32)
        tf = t
    loss, ssim, g = _gpu_loss(c, t)
    ref_loss, ref_ssim, ref_g = oloss.l1_dssim_loss(c, tf)
    np.testing.assert_allclose(ssim, ref_ssim, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(loss, ref_loss, rtol=1e-5)
    assert_grad_close(g, ref_g, what=f"{h}x{w}")


def test_rejects_bad_arguments():
    lib = _lib.lib()
    assert lib.gs_l1_dssim_loss(None, None, 0, 8, 8, 0.8, 0.2, None, None, None, None, 0, None) == _lib.GS_ERR_INVALID
