"""Fused Adam on the GPU against the oracle (and the reference's own MSL kernel text)."""
import os

import numpy as np
import pytest
import torch

from gsutil import assert_adam_close, assert_adam_update_close
from mlx_gsplat_b200 import FusedMLXAdam, ext
from mlx_gsplat_b200.allocator import SlabLayout
from oracle import adam as oadam
from oracle import densify as odens

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(seed, maxg, n, dim, nan=True):
    rng = np.random.default_rng(seed)
    theta = rng.normal(0, 1, (maxg, dim)).astype(np.float32)
    m = rng.normal(0, 0.1, (maxg, dim)).astype(np.float32)
    v = np.abs(rng.normal(0, 0.01, (maxg, dim))).astype(np.float32)
    g = rng.normal(0, 0.1, (n, dim)).astype(np.float32)
    if nan:
        g[0, 0] = np.nan
        g[min(1, n - 1), dim - 1] = np.inf
        g[min(2, n - 1), 0] = 1e30
    idx = rng.permutation(maxg)[:n].astype(np.int32)
    return theta, g, m, v, idx


@pytest.mark.parametrize("dim,lo,hi,wd", [(3, -1e10, 1e10, 0.0), (3, -10.0, -2.0, 0.0), (1, -5.0, 2.0, 0.0),
                                          (4, -1e10, 1e10, 0.01), (45, -1e10, 1e10, 0.0)])
def test_launch_fused_adam_step_bit_exact(dim, lo, hi, wd):
    theta, g, m, v, idx = _case(1, 3000, 2500, dim)
    T = [torch.from_numpy(x.copy()).to(DEV) for x in (theta, g, m, v, idx)]
    a = [x.copy() for x in (theta, g, m, v, idx)]
    b = [x.copy() for x in (theta, g, m, v, idx)]
    for step in (1, 2, 3, 10):
        ext.launch_fused_adam_step(T[0].data_ptr(), T[1].data_ptr(), T[2].data_ptr(), T[3].data_ptr(),
                                   T[4].data_ptr(), theta.shape[0], idx.shape[0], dim, 1e-3, 0.9, 0.999, 1e-15, wd,
                                   step, lo, hi)
        oadam.fused_adam_a1(*a, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-15, weight_decay=wd, step=step,
                            a_min=lo, a_max=hi)
        if oadam.ref_available():
            oadam.ref_fused_adam_a1(*b, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-15, weight_decay=wd, step=step,
                                    a_min=lo, a_max=hi)
    torch.cuda.synchronize()
    for i, name in enumerate(("theta", "g", "m", "v")):
        got = T[i].cpu().numpy()
        np.testing.assert_array_equal(got, a[i], err_msg=name)
        if oadam.ref_available():
            np.testing.assert_array_equal(got, b[i], err_msg=name + " vs reference kernel")


def test_pure_adam_matches_reference_golden(golden_dir):
    d = np.load(os.path.join(golden_dir, "adam_pure.npz"))
    names = ["means", "scales", "quats", "opacities", "sh0", "shN"]
    p = {k: torch.from_numpy(d["p0_" + k]).to(DEV) for k in names}
    m = {k: torch.zeros_like(p[k]) for k in names}
    v = {k: torch.zeros_like(p[k]) for k in names}
    opt = FusedMLXAdam(lr=1e-3, betas=(0.9, 0.999), eps=1e-15)
    for t in range(1, 4):
        g = {k: torch.from_numpy(d[f"g{t}_" + k]).to(DEV) for k in names}
        p, m, v = opt.step(p, g, m, v, use_metal_fusion=False)
        for k in names:
            assert_adam_close(p[k].cpu().numpy(), d[f"p{t}_" + k], what=f"p{t} {k}")
            assert_adam_close(m[k].cpu().numpy(), d[f"m{t}_" + k], what=f"m{t} {k}")
            assert_adam_close(v[k].cpu().numpy(), d[f"v{t}_" + k], what=f"v{t} {k}")


def test_optimizer_fused_path_over_slab_views_matches_oracle():
    """The reference call form (one launch per group, pools as strided slab views)."""
    from mlx_gsplat_b200 import PointerStableChunkedAllocator
    rng = np.random.default_rng(4)
    al = PointerStableChunkedAllocator(500, sh_degree=1, device=DEV)
    dims = al.layout.dims
    init = {k: rng.normal(0, 1, (300, dd)).astype(np.float32) for k, dd in dims.items()}
    al.set_initial_gaussians(init)
    grads = {k: torch.from_numpy(rng.normal(0, 0.1, (300, dd)).astype(np.float32)).to(DEV) for k, dd in dims.items()}
    pools0 = {k: al.physical_pools[k].cpu().numpy().copy() for k in dims}
    opt = FusedMLXAdam(lr=1e-3, eps=1e-15)
    ap = al.get_active_parameters()
    am, av = al.get_active_adam_states()
    opt.step(ap, grads, am, av, use_metal_fusion=True, physical_pools=al.physical_pools,
             adam_m_pools=al.adam_m_pools, adam_v_pools=al.adam_v_pools, indirection_table=al.indirection_table,
             cached_pointers=al.cached_pointers, cached_indices_addr=al.cached_indices_addr)
    torch.cuda.synchronize()
    table = al.indirection_table.cpu().numpy()
    for k, dd in dims.items():
        th = np.ascontiguousarray(pools0[k])
        mm = np.zeros_like(th)
        vv = np.zeros_like(th)
        lo, hi = oadam.group_clamp(k)
        oadam.fused_adam_a1(th, grads[k].cpu().numpy(), mm, vv, table, lr=1e-3, beta1=0.9, beta2=0.999,
                            eps=1e-15, weight_decay=0.0, step=1, a_min=lo, a_max=hi)
        np.testing.assert_array_equal(al.physical_pools[k].cpu().numpy(), th, err_msg=k)
        np.testing.assert_array_equal(al.adam_m_pools[k].cpu().numpy(), mm, err_msg=k)


@pytest.mark.parametrize("exact", [True, False], ids=["exact", "approx-step"])
@pytest.mark.parametrize("sh_degree", [0, 1, 3])
def test_slab_adam_matches_per_group_oracle_and_renorm(sh_degree, exact):
    L = SlabLayout(sh_degree)
    rng = np.random.default_rng(7 + sh_degree)
    maxg, n = 4000, 3500
    theta = rng.normal(0, 1, (maxg, L.stride)).astype(np.float32)
    m = rng.normal(0, 0.1, (maxg, L.stride)).astype(np.float32)
    v = np.abs(rng.normal(0, 0.01, (maxg, L.stride))).astype(np.float32)
    g = rng.normal(0, 0.1, (n, L.stride)).astype(np.float32)
    g[5, 2] = np.nan
    idx = rng.permutation(maxg)[:n].astype(np.int32)
    T = [torch.from_numpy(x.copy()).to(DEV) for x in (theta, g, m, v, idx)]
    theta0 = theta.copy()
    lo, hi = L.col_bounds()
    opt = FusedMLXAdam(lr=2e-3, eps=1e-15)
    for step in (1, 2):
        opt.step_slab(T[0], T[1], T[2], T[3], T[4], n, L.ncols, lo.tolist(), hi.tolist(), quat_col=L.quat_col,
                      exact=exact)
        for name, off in L.offsets.items():
            dd = L.dims[name]
            th = np.ascontiguousarray(theta[:, off:off + dd])
            mm = np.ascontiguousarray(m[:, off:off + dd])
            vv = np.ascontiguousarray(v[:, off:off + dd])
            gg = np.ascontiguousarray(g[:, off:off + dd])
            a, b = (-10.0, -2.0) if name == "scales" else ((-5.0, 2.0) if name == "opacities" else (-1e10, 1e10))
            oadam.fused_adam_a1(th, gg, mm, vv, idx, lr=2e-3, beta1=0.9, beta2=0.999, eps=1e-15, weight_decay=0.0,
                                step=step, a_min=a, a_max=b)
            if name == "quats":
                th[idx] = odens.quat_renorm(th[idx])
            theta[:, off:off + dd] = th
            m[:, off:off + dd] = mm
            v[:, off:off + dd] = vv
    torch.cuda.synchronize()
    got = T[0].cpu().numpy()
    q = L.offsets["quats"]
    rest = [c for c in range(L.ncols) if not q <= c < q + 4]
    if exact:
        np.testing.assert_array_equal(got[:, rest], theta[:, rest])
        assert_adam_close(got[:, q:q + 4], theta[:, q:q + 4], what="renormalised quats")
    else:
        assert_adam_update_close(got[:, rest], theta[:, rest], theta0[:, rest], what="approximate step")
        assert_adam_update_close(got[:, q:q + 4], theta[:, q:q + 4], theta0[:, q:q + 4], what="renormalised quats")
    # the moments are rounded exactly either way
    np.testing.assert_array_equal(T[2].cpu().numpy()[:, :L.ncols], m[:, :L.ncols])
    np.testing.assert_array_equal(T[3].cpu().numpy()[:, :L.ncols], v[:, :L.ncols])
    # padding columns untouched
    np.testing.assert_array_equal(got[:, L.ncols:], theta[:, L.ncols:])


def test_grad_scale_and_rejects_bad_args():
    from mlx_gsplat_b200 import _lib
    lib = _lib.lib()
    theta, g, m, v, idx = _case(2, 64, 40, 4, nan=False)
    T = [torch.from_numpy(x.copy()).to(DEV) for x in (theta, g, m, v, idx)]
    st = lib.gs_fused_adam_group(T[0].data_ptr(), T[1].data_ptr(), T[2].data_ptr(), T[3].data_ptr(),
                                 T[4].data_ptr(), 40, 4, 4, 4, 1e-3, 0.9, 0.999, 1e-8, 0.0, 1, -1e10, 1e10, 1.0,
                                 0.5, 0, _lib.stream_ptr())
    assert st == 0
    a = [x.copy() for x in (theta, g * np.float32(0.5), m, v, idx)]
    oadam.fused_adam_a1(*a, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, step=1, a_min=-1e10,
                        a_max=1e10)
    np.testing.assert_array_equal(T[0].cpu().numpy(), a[0])
    assert lib.gs_fused_adam_group(T[0].data_ptr(), T[1].data_ptr(), T[2].data_ptr(), T[3].data_ptr(),
                                   T[4].data_ptr(), 40, 4, 4, 4, 1e-3, 0.9, 0.999, 1e-8, 0.0, 0, -1e10, 1e10, 1.0,
                                   1.0, 0, _lib.stream_ptr()) == _lib.GS_ERR_INVALID
