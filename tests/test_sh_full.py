"""The full spherical-harmonics colour mode (``sh_mode="full"``, degrees 2 and
3; the reference evaluates degree <= 1 only, mlx_gsplat/rendering.py:229-244).

CPU: the oracle's basis is the real SH basis (orthonormal on the sphere, by
quadrature) and the full mode equals the reference mode at degree <= 1.
GPU: images within 1e-4 and gradients within 1e-3 relative of the dense oracle
in the full mode (``tests/gsutil.py``), through the autograd entry point and
through the trainer's pooled rows."""
import numpy as np
import pytest
import torch

from gsutil import assert_grad_close, assert_image_close
from oracle import rendering as orend

DEV = "cuda"
NAMES = ("means", "quats", "scales", "opacities", "colors")


def _sphere_quadrature(n_theta=24, n_phi=48):
    """Gauss-Legendre in cos(theta) x uniform phi: exact for the products of
    two degree <= 3 polynomials on the unit sphere."""
    u, wu = np.polynomial.legendre.leggauss(n_theta)
    phi = np.arange(n_phi) * (2 * np.pi / n_phi)
    U, P = np.meshgrid(u, phi, indexing="ij")
    s = np.sqrt(1 - U ** 2)
    x, y, z = s * np.cos(P), s * np.sin(P), U
    w = np.repeat(wu[:, None], n_phi, 1) * (2 * np.pi / n_phi)
    return x.ravel(), y.ravel(), z.ravel(), w.ravel()


def test_oracle_basis_is_orthonormal():
    x, y, z, w = _sphere_quadrature()
    basis = [np.full_like(x, orend.SH_C0), orend.SH_C1 * y, orend.SH_C1 * z, orend.SH_C1 * x]
    basis += orend._sh_hi_basis(x, y, z, 3)
    B = np.stack(basis)  # 16 functions
    G = (B * w) @ B.T
    np.testing.assert_allclose(G, np.eye(16), atol=1e-12)


@pytest.mark.parametrize("ncols", [3, 12])
def test_oracle_full_equals_reference_up_to_degree_1(ncols):
    rng = np.random.default_rng(0)
    n = 200
    means = torch.from_numpy(rng.uniform(-1, 1, (n, 3)))
    quats = torch.from_numpy(rng.normal(0, 1, (n, 4)))
    scales = torch.from_numpy(rng.normal(-3, 0.3, (n, 3)))
    opac = torch.from_numpy(rng.normal(0, 1, (n, 1)))
    cols = torch.from_numpy(rng.normal(0, 0.5, (n, ncols)))
    vm = torch.eye(4, dtype=torch.float64)
    vm[2, 3] = 4.0
    K = torch.tensor([[100.0, 0, 60], [0, 100.0, 45], [0, 0, 1]], dtype=torch.float64)
    a = orend.project(means, quats, scales, opac, cols, vm, K, 120, 90, 120, 90, sh_mode="reference")
    b = orend.project(means, quats, scales, opac, cols, vm, K, 120, 90, 120, 90, sh_mode="full")
    assert torch.equal(a["rgb"], b["rgb"])


def test_oracle_degree_from_columns():
    assert [orend.sh_full_degree(c) for c in (3, 12, 27, 48, 60)] == [0, 1, 2, 3, 3]


# ----------------------------------------------------------------------------- GPU
def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def _tiny_scene(ncols, seed=0):
    from mlx_gsplat_b200 import synthetic
    wl = synthetic.WORKLOADS["tiny-3k"]
    g = synthetic.make_gaussians(wl, seed=seed, n=3000)
    rng = np.random.default_rng(seed + 10)
    rest = rng.normal(0, 0.3, (3000, ncols - 3)).astype(np.float32)
    cols = np.concatenate([g["sh0"], rest], 1).astype(np.float32)
    return wl, g, cols


@pytest.mark.gpu
@pytest.mark.parametrize("ncols", [27, 48], ids=["degree2", "degree3"])
def test_full_sh_forward_backward_vs_oracle(ncols):
    from mlx_gsplat_b200 import frustum_culling_mlx, rasterize_gaussians_mlx, synthetic
    wl, g, cols = _tiny_scene(ncols)
    views, K = synthetic.make_cameras(wl, seed=2)
    rng = np.random.default_rng(1)
    P = wl.pixels
    for vi in (0, 5):
        vm = views[vi]
        params = {k: _t(g[k]) for k in ("means", "quats", "scales", "opacities")}
        ids = frustum_culling_mlx(params["means"], None, None, vm, K, wl.width, wl.height,
                                  opacities=params["opacities"])
        idn = ids.cpu().numpy().astype(np.int64)
        for k in params:
            params[k].requires_grad_(True)
        params["colors"] = _t(cols[idn]).requires_grad_(True)
        C, A = rasterize_gaussians_mlx(params["means"], params["quats"], params["scales"], params["opacities"],
                                       params["colors"], vm, K, wl.width, wl.height, ids, render_width=wl.width,
                                       render_height=wl.height, sh_mode="full")
        wC = rng.uniform(-1, 1, (wl.height, wl.width, 3)).astype(np.float32) / P
        wA = rng.uniform(-1, 1, (wl.height, wl.width, 1)).astype(np.float32) / P
        (torch.sum(C * _t(wC)) + torch.sum(A * _t(wA))).backward()
        Cr, Ar, gr = orend.rasterize_dense_vjp(g["means"][idn], g["quats"][idn], g["scales"][idn],
                                               g["opacities"][idn], cols[idn], vm, K, wl.width, wl.height,
                                               wl.width, wl.height, dL_dC=wC, dL_dA=wA, sh_mode="full")
        assert_image_close(C.detach().cpu().numpy(), Cr, what=f"view {vi} colors")
        assert_image_close(A.detach().cpu().numpy(), Ar, what=f"view {vi} alphas")
        for k in NAMES:
            got = params[k].grad.cpu().numpy()
            if k != "colors":
                got = got[idn]
            assert_grad_close(got, gr[k], what=f"view {vi} grad {k}")
        # the higher degrees change the image (the mode is not a no-op)
        Cref, _ = rasterize_gaussians_mlx(params["means"], params["quats"], params["scales"], params["opacities"],
                                          params["colors"], vm, K, wl.width, wl.height, ids,
                                          render_width=wl.width, render_height=wl.height)
        assert float((Cref - C).abs().max()) > 1e-2


@pytest.mark.gpu
def test_full_sh_degree1_identical_to_reference_mode():
    from mlx_gsplat_b200 import frustum_culling_mlx, rasterize_gaussians_mlx, synthetic
    wl, g, cols = _tiny_scene(12)
    views, K = synthetic.make_cameras(wl, seed=2)
    vm = views[2]
    T = {k: _t(g[k]) for k in ("means", "quats", "scales", "opacities")}
    ids = frustum_culling_mlx(T["means"], None, None, vm, K, wl.width, wl.height, opacities=T["opacities"])
    c = _t(cols)
    out = [rasterize_gaussians_mlx(T["means"], T["quats"], T["scales"], T["opacities"], c, vm, K, wl.width,
                                   wl.height, ids, render_width=wl.width, render_height=wl.height, sh_mode=m)
           for m in ("reference", "full")]
    assert torch.equal(out[0][0], out[1][0]) and torch.equal(out[0][1], out[1][1])


@pytest.mark.gpu
def test_trainer_full_sh_gradient_rows_vs_oracle(monkeypatch):
    """The trainer's pooled-row path (vector row loads and stores, indirection
    table) in the full mode at SH degree 3 (step 3 of a degree-per-step
    schedule): gradient rows against the dense oracle, on the outdoor scene's
    distributions at 8,000 Gaussians and 216x140 (so the dense oracle stays
    fast)."""
    import dataclasses

    from mlx_gsplat_b200 import synthetic
    from mlx_gsplat_b200.trainer import runner_for_workload, sh_cols_for
    wl = dataclasses.replace(synthetic.WORKLOADS["outdoor-1m"], name="outdoor-small", num_gaussians=8000,
                             width=216, height=140, focal=1150.0 / 6)
    monkeypatch.setitem(synthetic.WORKLOADS, wl.name, wl)
    r = runner_for_workload(wl.name, max_steps=50, num_views=4, lr=1e-3, eps=1e-15, sh_eval="full")
    r.row_mode = "dense"
    al, L = r.allocator, r.layout
    step = 3
    assert sh_cols_for(step, r.cfg) == 48
    theta0 = al.theta.cpu().numpy().copy()
    table = al.indirection_table.cpu().numpy()
    frame = r.train_step(1, step)
    torch.cuda.synchronize()
    N = al.num_active
    grad = r.grad[:N].cpu().numpy()
    act = {k: theta0[table][:, o:o + L.dims[k]] for k, o in L.offsets.items()}
    ids = frame.ids[:frame.V].cpu().numpy().astype(np.int64)
    colors = np.concatenate([act["sh0"], act["shN"]], 1)
    C = frame.color.cpu().numpy()
    tf = r.targets[1].cpu().numpy().astype(np.float32) / np.float32(255.0)
    dC = np.sign(C.astype(np.float64) - tf) / (3.0 * r.cfg.render_width * r.cfg.render_height)
    _, _, gr = orend.rasterize_dense_vjp(act["means"][ids], act["quats"][ids], act["scales"][ids],
                                         act["opacities"][ids], colors[ids], r.viewmats[1], r.K, r.cfg.width,
                                         r.cfg.height, r.cfg.render_width, r.cfg.render_height, dL_dC=dC,
                                         pixel_ids=None, sh_mode="full")
    reg = r.cfg.param_reg
    for k in ("means", "quats", "scales", "opacities"):
        ref = np.full((N, L.dims[k]), reg, np.float64)
        ref[ids] += gr[k]
        o = L.offsets[k]
        assert_grad_close(grad[:, o:o + L.dims[k]], ref, what="grad " + k)
    refc = np.zeros((N, L.color_cols), np.float64)
    refc[ids] = reg + gr["colors"]
    assert_grad_close(grad[:, L.color_col:L.color_col + L.color_cols], refc, what="grad colors")
