"""Cull, scan and radix sort on the GPU: bit-exact against the oracle / NumPy."""
import os

import numpy as np
import pytest
import torch

from mlx_gsplat_b200 import _lib, frustum_culling_mlx, synthetic
from mlx_gsplat_b200.rendering import camera_struct, cull_ids, gaussians_struct
from oracle import rendering as orend

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_cull_matches_reference_golden(golden_dir):
    d = np.load(os.path.join(golden_dir, "cull.npz"))
    W, H = int(d["width"]), int(d["height"])
    means = torch.from_numpy(d["means"]).to(DEV)
    opac = torch.from_numpy(d["opacities"]).to(DEV)
    for i in range(d["views"].shape[0]):
        ids = frustum_culling_mlx(means, None, None, d["views"][i], d["K"], W, H, opacities=opac)
        np.testing.assert_array_equal(ids.cpu().numpy(), d[f"ids_{i}"])
    away = frustum_culling_mlx(means, None, None, d["away_view"], d["K"], W, H, opacities=opac)
    assert away.numel() == 0
    quirk = frustum_culling_mlx(means, None, None, d["away_view"], d["K"], W, H, opacities=opac, empty_quirk=True)
    np.testing.assert_array_equal(quirk.cpu().numpy(), d["ids_away"])


@pytest.mark.parametrize("wl_name,n", [("mid-200k", 200_000), ("outdoor-1m", 1_000_000), ("tiny-3k", 1),
                                       ("tiny-3k", 2049), ("large-6m", 6_000_000)])
def test_cull_bit_exact_vs_oracle_full_size(wl_name, n):
    wl = synthetic.WORKLOADS[wl_name]
    g = synthetic.make_gaussians(wl, seed=0, n=n)
    views, K = synthetic.make_cameras(wl, seed=2, num_views=4)
    means = torch.from_numpy(g["means"]).to(DEV)
    opac = torch.from_numpy(g["opacities"]).to(DEV)
    for vm in views[:2]:
        ids = frustum_culling_mlx(means, None, None, vm, K, wl.width, wl.height, opacities=opac)
        ref = orend.cull(g["means"], g["opacities"], vm, K, wl.width, wl.height)
        np.testing.assert_array_equal(ids.cpu().numpy(), ref)


def test_cull_through_indirection_table_and_strided_rows():
    wl = synthetic.WORKLOADS["mid-200k"]
    g = synthetic.make_gaussians(wl, seed=3, n=50_000)
    views, K = synthetic.make_cameras(wl, seed=2, num_views=2)
    rng = np.random.default_rng(0)
    maxg = 80_000
    table = rng.permutation(maxg)[:50_000].astype(np.int32)
    slab = np.zeros((maxg, 8), np.float32)
    slab[table, 1:4] = g["means"]
    slab[table, 5] = g["opacities"][:, 0]
    S = torch.from_numpy(slab).to(DEV)
    gs = gaussians_struct(S[:, 1:4], opacities=S[:, 5:6], table=torch.from_numpy(table).to(DEV))
    cam = camera_struct(views[0], K, wl.width, wl.height, wl.width, wl.height)
    ids, _, V = cull_ids(gs, 50_000, cam, torch.device(DEV))
    ref = orend.cull(g["means"], g["opacities"], views[0], K, wl.width, wl.height)
    np.testing.assert_array_equal(ids[:V].cpu().numpy(), ref)


@pytest.mark.parametrize("n", [1, 7, 2048, 2049, 4096, 4097, 8193, 100_003, 3_000_000])
def test_scan_exact(n):
    """Exclusive scan with the total at out[n]: the one-CTA path (up to 4,096
    values) and the three-kernel path."""
    lib = _lib.lib()
    rng = np.random.default_rng(n)
    x = rng.integers(0, 50, n).astype(np.int32)
    X = torch.from_numpy(x).to(DEV)
    out = torch.empty(n + 1, dtype=torch.int32, device=DEV)
    sb = torch.empty(lib.gs_scan_scratch_bytes(n), dtype=torch.uint8, device=DEV)
    _lib.check(lib.gs_exclusive_scan_u32(X.data_ptr(), out.data_ptr(), n, sb.data_ptr(), sb.numel(),
                                         _lib.stream_ptr()))
    ref = np.concatenate([[0], np.cumsum(x)]).astype(np.int64)
    np.testing.assert_array_equal(out.cpu().numpy().astype(np.int64), ref)


@pytest.mark.parametrize("n,lo,hi,kmax", [(1, 0, 32, 2 ** 32), (2048, 0, 32, 2 ** 32), (5000, 0, 13, 4293),
                                          (1_000_000, 0, 32, 2 ** 32), (777_777, 0, 15, 32400),
                                          (3_000_000, 0, 16, 100), (123_456, 4, 20, 2 ** 24)])
def test_radix_sort_stable_exact(n, lo, hi, kmax):
    lib = _lib.lib()
    rng = np.random.default_rng(n + lo)
    keys = rng.integers(0, kmax, n, dtype=np.uint64).astype(np.uint32)
    vals = np.arange(n, dtype=np.uint32)
    K = torch.from_numpy(keys.view(np.int32)).to(DEV)
    Vv = torch.from_numpy(vals.view(np.int32)).to(DEV)
    ko = torch.empty_like(K)
    vo = torch.empty_like(Vv)
    sb = torch.empty(lib.gs_radix_sort_scratch_bytes(n), dtype=torch.uint8, device=DEV)
    _lib.check(lib.gs_radix_sort_pairs(K.data_ptr(), Vv.data_ptr(), ko.data_ptr(), vo.data_ptr(), n, lo, hi,
                                       sb.data_ptr(), sb.numel(), _lib.stream_ptr()))
    sortkey = (keys >> np.uint32(lo)) & np.uint32((1 << (hi - lo)) - 1 if hi - lo < 32 else 0xFFFFFFFF)
    order = np.argsort(sortkey, kind="stable")
    np.testing.assert_array_equal(vo.cpu().numpy().view(np.uint32), vals[order])
    np.testing.assert_array_equal(ko.cpu().numpy().view(np.uint32), keys[order])
    # no values: vals_out is the sorting permutation itself
    if hi > lo:
        vo.fill_(-1)
        _lib.check(lib.gs_radix_sort_pairs(K.data_ptr(), None, ko.data_ptr(), vo.data_ptr(), n, lo, hi,
                                           sb.data_ptr(), sb.numel(), _lib.stream_ptr()))
        np.testing.assert_array_equal(vo.cpu().numpy(), order.astype(np.int32))
