"""The allocation-free cull entry point (gs_cull_noalloc) against the regular
one (gs_cull with a caller scratch buffer), called through the C ABI.

gs_cull_noalloc exists for callers that cannot allocate device memory (a host
binding the C ABI from a runtime without a device allocator, or a process whose
device memory belongs to another framework's pool): its scratch is a fixed
array inside the library.  The cull is an index computation, so the two entry
points must agree exactly.  Two calls in a row check that the shared array
carries nothing over from one call to the next.  This file is collected last
so that a failure here never hides another test's result.
"""
import numpy as np
import pytest
import torch

from mlx_gsplat_b200 import _lib, synthetic
from mlx_gsplat_b200.rendering import camera_struct, gaussians_struct

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _both(lib, g, n, cam):
    st = _lib.stream_ptr()
    ids_a = torch.full((n,), -7, dtype=torch.int32, device=DEV)
    cnt_a = torch.zeros(1, dtype=torch.int32, device=DEV)
    sb = torch.empty(lib.gs_cull_scratch_bytes(n), dtype=torch.uint8, device=DEV)
    _lib.check(lib.gs_cull(g, n, cam, 0.01, 1e10, -5.3, ids_a.data_ptr(), cnt_a.data_ptr(), sb.data_ptr(),
                           sb.numel(), st), "gs_cull")
    ids_b = torch.full((n,), -9, dtype=torch.int32, device=DEV)
    cnt_b = torch.zeros(1, dtype=torch.int32, device=DEV)
    _lib.check(lib.gs_cull_noalloc(g, n, cam, 0.01, 1e10, -5.3, ids_b.data_ptr(), cnt_b.data_ptr(), st),
               "gs_cull_noalloc")
    torch.cuda.synchronize()
    V = int(cnt_a.item())
    assert int(cnt_b.item()) == V
    return ids_a[:V].cpu().numpy(), ids_b[:V].cpu().numpy()


def test_cull_noalloc_matches_cull_on_consecutive_calls():
    lib = _lib.lib()
    wl = synthetic.WORKLOADS["outdoor-1m"]
    views, K = synthetic.make_cameras(wl, seed=2, num_views=4)
    for n, view in ((1_000_000, 0), (300_001, 1)):  # second call smaller: stale scratch would show
        gsd = synthetic.make_gaussians(wl, seed=n, n=n)
        means = torch.from_numpy(gsd["means"]).to(DEV)
        opac = torch.from_numpy(gsd["opacities"]).to(DEV)
        g = gaussians_struct(means, opacities=opac)
        cam = camera_struct(views[view], K, wl.width, wl.height, wl.width, wl.height)
        a, b = _both(lib, g, n, cam)
        assert a.size > 0
        np.testing.assert_array_equal(a, b)


def test_cull_noalloc_rejects_sizes_beyond_its_limit():
    lib = _lib.lib()
    means = torch.zeros((4, 3), dtype=torch.float32, device=DEV)
    g = gaussians_struct(means)
    cam = camera_struct(np.eye(4), np.eye(3), 8, 8, 8, 8)
    out = torch.empty(4, dtype=torch.int32, device=DEV)
    cnt = torch.empty(1, dtype=torch.int32, device=DEV)
    st = lib.gs_cull_noalloc(g, (1 << 23) + 1, cam, 0.01, 1e10, -5.3, out.data_ptr(), cnt.data_ptr(),
                             _lib.stream_ptr())
    assert st == _lib.GS_ERR_CAPACITY
    assert b"limit" in lib.gs_last_error()
