"""Pin the CPU oracle against the golden fixtures written by running the
reference's own Python (``tests/golden/gen_golden.py``) and against the
reference's own Metal Adam source compiled for the CPU (``oracle/build_ref.py``)."""
import os

import numpy as np
import pytest
import torch

from oracle import adam as oadam
from oracle import allocator as oalloc
from oracle import rendering as orend


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_cull_matches_reference(golden_dir):
    d = _load(golden_dir, "cull.npz")
    W, H = int(d["width"]), int(d["height"])
    for i in range(d["views"].shape[0]):
        ids = orend.cull(d["means"], d["opacities"], d["views"][i], d["K"], W, H)
        np.testing.assert_array_equal(ids, d[f"ids_{i}"])
        # partially visible: each view keeps some and drops some
        assert 0 < ids.size < d["means"].shape[0]


def test_cull_empty_quirk(golden_dir):
    d = _load(golden_dir, "cull.npz")
    W, H = int(d["width"]), int(d["height"])
    q = orend.cull(d["means"], d["opacities"], d["away_view"], d["K"], W, H, empty_quirk=True)
    np.testing.assert_array_equal(q, d["ids_away"])
    assert orend.cull(d["means"], d["opacities"], d["away_view"], d["K"], W, H).size == 0


@pytest.mark.parametrize("case", ["sh0", "sh1", "sh3", "scaled"])
def test_dense_raster_matches_reference(golden_dir, case):
    d = _load(golden_dir, "raster.npz")
    p = lambda k: d[f"{case}_{k}"]  # noqa: E731
    W, H, RW, RH = [int(x) for x in p("dims")]
    ids = p("ids").astype(np.int64)
    args = (p("means")[ids], p("quats")[ids], p("scales")[ids], p("opacities")[ids], p("colors"),
            p("viewmat"), p("K"), W, H, RW, RH)
    C, A = orend.rasterize_dense(*args, dtype=torch.float32)
    np.testing.assert_allclose(C, p("out_colors"), atol=2e-6)
    np.testing.assert_allclose(A, p("out_alphas"), atol=2e-6)
    C64, _ = orend.rasterize_dense(*args, dtype=torch.float64)
    np.testing.assert_allclose(C64, p("out_colors"), atol=2e-5)

    # gradients of  mean|C - target| + mean(A * wA)  through the VJP path
    P = RW * RH
    diff = C.astype(np.float64) - p("target")
    dC = np.sign(diff) / (3.0 * P)
    dA = p("wA") / P
    _, _, g = orend.rasterize_dense_vjp(*args, dL_dC=dC, dL_dA=dA, dtype=torch.float64)
    for k in ("means", "quats", "scales", "opacities", "colors"):
        ref = p("grad_" + k)
        got = g[k] if k == "colors" else np.zeros_like(ref)
        if k != "colors":
            got[ids] = g[k]
        err = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
        assert err < 1e-4, (k, err)


def test_dense_raster_with_alpha_mask_matches_reference(golden_dir):
    """rendering.py:289-290: the reference multiplies the clipped alphas by
    mask[j], j the depth-sorted position (the mask is not permuted by the
    sort).  The golden ran the reference's own rasterizer with a mask."""
    d = _load(golden_dir, "raster_mask.npz")
    W, H, RW, RH = [int(x) for x in d["dims"]]
    ids = d["ids"].astype(np.int64)
    args = (d["means"][ids], d["quats"][ids], d["scales"][ids], d["opacities"][ids], d["colors"],
            d["viewmat"], d["K"], W, H, RW, RH)
    C, A = orend.rasterize_dense(*args, dtype=torch.float32, mask=d["mask"])
    np.testing.assert_allclose(C, d["out_colors"], atol=2e-6)
    np.testing.assert_allclose(A, d["out_alphas"], atol=2e-6)
    # the mask must go by depth rank: applied by visible position instead, the image differs
    pg_order = orend.project(*[torch.as_tensor(np.asarray(a)) for a in args[:5]], torch.as_tensor(d["viewmat"]),
                             torch.as_tensor(d["K"]), W, H, RW, RH)["order"].numpy()
    C_wrong, _ = orend.rasterize_dense(*args, dtype=torch.float32, mask=d["mask"][pg_order])
    assert np.abs(C_wrong - d["out_colors"]).max() > 1e-3
    P = RW * RH
    dC = np.sign(C.astype(np.float64) - d["target"]) / (3.0 * P)
    _, _, g = orend.rasterize_dense_vjp(*args, dL_dC=dC, dL_dA=d["wA"] / P, dtype=torch.float64, mask=d["mask"])
    for k in ("means", "quats", "scales", "opacities", "colors"):
        ref = d["grad_" + k]
        got = g[k] if k == "colors" else np.zeros_like(ref)
        if k != "colors":
            got[ids] = g[k]
        err = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
        assert err < 1e-4, (k, err)


def test_adam_pure_matches_reference(golden_dir):
    d = _load(golden_dir, "adam_pure.npz")
    names = ["means", "scales", "quats", "opacities", "sh0", "shN"]
    p = {k: d["p0_" + k] for k in names}
    m = {k: np.zeros_like(p[k]) for k in names}
    v = {k: np.zeros_like(p[k]) for k in names}
    for t in range(1, 4):
        g = {k: d[f"g{t}_" + k] for k in names}
        p, m, v = oadam.pure_adam_a2(p, g, m, v, t, lr=1e-3, eps=1e-15)
        for k in names:
            np.testing.assert_allclose(p[k], d[f"p{t}_" + k], rtol=1e-6, atol=1e-7)
            np.testing.assert_allclose(m[k], d[f"m{t}_" + k], rtol=1e-6, atol=1e-9)
            np.testing.assert_allclose(v[k], d[f"v{t}_" + k], rtol=1e-6, atol=1e-12)


def _adam_inputs(seed, maxg=64, n=40, dim=3):
    rng = np.random.default_rng(seed)
    theta = rng.normal(0, 1, (maxg, dim)).astype(np.float32)
    m = rng.normal(0, 0.1, (maxg, dim)).astype(np.float32)
    v = np.abs(rng.normal(0, 0.01, (maxg, dim))).astype(np.float32)
    g = rng.normal(0, 0.1, (n, dim)).astype(np.float32)
    g[0, 0] = np.nan
    g[1, dim - 1] = np.inf
    idx = rng.permutation(maxg)[:n].astype(np.int32)
    return theta, g, m, v, idx


@pytest.mark.skipif(not oadam.ref_available(), reason="reference MSL checker not built")
@pytest.mark.parametrize("dim,lo,hi,wd", [(3, -1e10, 1e10, 0.0), (3, -10.0, -2.0, 0.0), (1, -5.0, 2.0, 0.01),
                                          (45, -1e10, 1e10, 0.0)])
def test_adam_a1_restatement_matches_reference_kernel(dim, lo, hi, wd):
    a = _adam_inputs(3, dim=dim)
    b = tuple(x.copy() for x in a)
    for step in (1, 2, 7):
        oadam.fused_adam_a1(*a, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-15, weight_decay=wd, step=step,
                            a_min=lo, a_max=hi)
        oadam.ref_fused_adam_a1(*b, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-15, weight_decay=wd, step=step,
                                a_min=lo, a_max=hi)
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x, y)


def test_allocator_matches_reference(golden_dir):
    d = _load(golden_dir, "allocator.npz")
    dims = {"means": 3, "scales": 3, "quats": 4, "opacities": 1, "sh0": 3, "shN": 9}
    o = oalloc.PoolOracle(96, sh_degree=1)
    o.set_initial_gaussians({k: d["init_" + k] for k in dims})
    np.testing.assert_array_equal(o.table, d["table0"])
    np.testing.assert_array_equal(o.free_list_array(), d["free0"])
    for r in range(3):
        sp = {k + s: d[f"r{r}_sp_{k}{s}"] for k in dims for s in ("_child1", "_child2")}
        n_p, n_s = o.split_and_prune(d[f"r{r}_prune"], d[f"r{r}_split"], sp)
        np.testing.assert_array_equal([n_p, n_s], d[f"r{r}_counts"])
        np.testing.assert_array_equal(o.table, d[f"r{r}_table"])
        np.testing.assert_array_equal(o.free_list_array(), d[f"r{r}_free"])
        for k in dims:
            np.testing.assert_array_equal(o.pools[k], d[f"r{r}_pool_{k}"])
            np.testing.assert_array_equal(o.m[k], d[f"r{r}_m_{k}"])
    n = o.num_active
    sp = {k + s: np.zeros((n, dd), np.float32) for k, dd in dims.items() for s in ("_child1", "_child2")}
    with pytest.raises(MemoryError):
        o.split_and_prune(np.zeros(n, bool), np.ones(n, bool), sp)
    assert bool(d["oom_raised"])


def test_l1_dssim_loss_matches_reference(golden_dir):
    from oracle import loss as oloss
    d = _load(golden_dir, "ssim.npz")
    for i in range(3):
        c, t = d[f"c_{i}"], d[f"t_{i}"]
        loss, s, g = oloss.l1_dssim_loss(c, t)
        np.testing.assert_allclose(s, float(d[f"ssim_{i}"]), rtol=2e-6, atol=1e-7)
        np.testing.assert_allclose(loss, float(d[f"loss_{i}"]), rtol=2e-6, atol=1e-7)
        ref = d[f"grad_{i}"].astype(np.float64)
        assert np.abs(g - ref).max() <= 1e-4 * np.abs(ref).max(), i
