"""The fused training step (cull -> raster fwd + L1 -> raster bwd -> slab Adam)
against the oracle pipeline, and a short training run."""
import numpy as np
import pytest
import torch

from gsutil import assert_adam_update_close, assert_grad_close
from mlx_gsplat_b200 import synthetic
from mlx_gsplat_b200.trainer import runner_for_workload, sh_cols_for
from oracle import adam as oadam
from oracle import densify as odens
from oracle import rendering as orend

pytestmark = pytest.mark.gpu


def _small_outdoor(monkeypatch):
    """The outdoor scene's distributions (SH degree 3 stored) at 8,000
    Gaussians and 216x140, small enough for the dense oracle."""
    import dataclasses
    wl = dataclasses.replace(synthetic.WORKLOADS["outdoor-1m"], name="outdoor-small", num_gaussians=8000,
                             width=216, height=140, focal=1150.0 / 6)
    monkeypatch.setitem(synthetic.WORKLOADS, wl.name, wl)
    return wl.name


@pytest.mark.parametrize("wl_name,n,loss,step", [("tiny-3k", 3000, "l1", 1), ("mid-200k", 20_000, "l1", 1),
                                                 ("tiny-3k", 3000, "l1+dssim", 1),
                                                 ("mid-200k", 20_000, "l1+dssim", 1),
                                                 ("outdoor-small", None, "l1", 1),
                                                 ("outdoor-small", None, "l1", 3)])
def test_train_step_matches_oracle(monkeypatch, wl_name, n, loss, step):
    """One step's gradient rows and Adam update against the oracle.  The
    outdoor-small cases store SH degree 3 (48 colour floats) and run with
    narrow gradient rows (23 gradient columns + the view count; Adam rebuilds
    the regulariser-only colour columns) at SH degree 1 (step 1, 12 colour
    columns read) and degree 3 (step 3: 48 colour columns get the regulariser)."""
    if wl_name == "outdoor-small":
        _small_outdoor(monkeypatch)
    r = runner_for_workload(wl_name, max_steps=50, n=n, num_views=4, lr=1e-3, eps=1e-15, loss=loss)
    r.row_mode = "dense"  # write every gradient row so the test can inspect them
    al, L = r.allocator, r.layout
    if wl_name == "outdoor-small":
        assert r.g_cols == 23 and r.g_stride == 24
    theta0 = al.theta.cpu().numpy().copy()
    table = al.indirection_table.cpu().numpy()
    frame = r.train_step(0, step)
    torch.cuda.synchronize()
    N = al.num_active
    grad = r.full_gradient_rows(step, N).cpu().numpy()
    # --- oracle gradients: dense VJP over the visible rows, cotangent from the GPU image
    act = {k: theta0[table][:, o:o + L.dims[k]] for k, o in L.offsets.items()}
    ids = frame.ids[:frame.V].cpu().numpy().astype(np.int64)
    ref_ids = orend.cull(act["means"], act["opacities"], r.viewmats[0], r.K, r.cfg.width, r.cfg.height)
    np.testing.assert_array_equal(ids, ref_ids)
    ncols = sh_cols_for(step, r.cfg)
    colors = np.concatenate([act["sh0"], act["shN"]], 1)[:, :ncols]
    C = frame.color.cpu().numpy()
    target = r.targets[0].cpu().numpy()
    tf = target.astype(np.float32) / np.float32(255.0) if target.dtype == np.uint8 else target
    P = r.cfg.render_width * r.cfg.render_height
    if loss == "l1":
        dC = np.sign(C.astype(np.float64) - tf) / (3.0 * P)
    else:
        from oracle import loss as oloss
        ref_loss, _, dC = oloss.l1_dssim_loss(C, tf)
        assert abs(float(r.loss_value()) - ref_loss) <= 1e-5 * abs(ref_loss)
    _, _, gr = orend.rasterize_dense_vjp(act["means"][ids], act["quats"][ids], act["scales"][ids],
                                         act["opacities"][ids], colors[ids], r.viewmats[0], r.K, r.cfg.width,
                                         r.cfg.height, r.cfg.render_width, r.cfg.render_height, dL_dC=dC)
    reg = r.cfg.param_reg
    for k in ("means", "quats", "scales", "opacities"):
        ref = np.full((N, L.dims[k]), reg, np.float64)
        ref[ids] += gr[k]
        o = L.offsets[k]
        assert_grad_close(grad[:, o:o + L.dims[k]], ref, what="grad " + k)
    refc = np.zeros((N, L.color_cols), np.float64)
    refc[ids, :ncols] = reg
    refc[ids, :ncols] += gr["colors"]
    assert_grad_close(grad[:, L.color_col:L.color_col + L.color_cols], refc, what="grad colors")
    # --- oracle Adam on the GPU's gradients (fused semantics + quaternion renorm)
    after = al.theta.cpu().numpy()
    lr = 1e-3 * (0.01 ** (step / r.cfg.max_steps))
    for k, o in L.offsets.items():
        dd = L.dims[k]
        th = np.ascontiguousarray(theta0[:, o:o + dd])
        mm = np.zeros_like(th)
        vv = np.zeros_like(th)
        lo, hi = oadam.group_clamp(k)
        oadam.fused_adam_a1(th, np.ascontiguousarray(grad[:, o:o + dd]), mm, vv, table, lr=np.float32(lr),
                            beta1=0.9, beta2=0.999, eps=1e-15, weight_decay=0.0, step=1, a_min=lo, a_max=hi)
        if k == "quats":
            th[table] = odens.quat_renorm(th[table])
        assert_adam_update_close(after[:, o:o + dd], th, theta0[:, o:o + dd], what="adam " + k)


def test_unseen_rows_from_visibility_bits_match_dense_rows():
    """One GPU: Adam takes the gradient of Gaussians a view does not see from the
    cull's visibility bits instead of pre-filled rows.  Kernel level, bit-exact:
    the same visible rows, garbage in the unseen rows of the sparse run."""
    from mlx_gsplat_b200.allocator import SlabLayout
    from mlx_gsplat_b200.optimizer import FusedMLXAdam
    L = SlabLayout(3)
    rng = np.random.default_rng(3)
    n, maxg = 50_000, 60_000
    theta = rng.normal(0, 1, (maxg, L.stride)).astype(np.float32)
    table = rng.permutation(maxg)[:n].astype(np.int32)
    seen = rng.uniform(0, 1, n) < 0.4
    words = np.zeros((n + 31) // 32, np.uint32)
    for r in np.nonzero(seen)[0]:
        words[r >> 5] |= np.uint32(1) << np.uint32(r & 31)
    pattern = np.zeros(L.stride, np.float32)
    pattern[:11] = 1e-5
    g_dense = rng.normal(0, 0.1, (maxg, L.stride)).astype(np.float32)
    g_dense[:n][~seen] = pattern
    g_sparse = g_dense.copy()
    g_sparse[:n][~seen] = 123.0  # never read
    lo, hi = L.col_bounds()
    out = []
    for g, vis in ((g_dense, None), (g_sparse, words)):
        T = [torch.from_numpy(x.copy()).cuda() for x in (theta, g)]
        m = torch.zeros_like(T[0])
        v = torch.zeros_like(T[0])
        tab = torch.from_numpy(table).cuda()
        W = None if vis is None else torch.from_numpy(vis.view(np.int32)).cuda()
        opt = FusedMLXAdam(lr=1e-3, eps=1e-15)
        for _ in range(2):
            opt.step_slab(T[0], T[1], m, v, tab, n, L.ncols, lo.tolist(), hi.tolist(), quat_col=0,
                          visible_words=None if W is None else W.data_ptr(),
                          unseen_grad=None if W is None else pattern[:L.ncols].tolist())
        torch.cuda.synchronize()
        out.append([x.cpu().numpy() for x in (T[0], m, v)])
    for a, b in zip(*out):
        np.testing.assert_array_equal(a, b)


def test_adam_split_by_visibility_equals_one_launch():
    """Adam over the unseen rows (what the trainer runs on a side stream right
    after the cull) then over the seen rows, with one step count, gives the
    one-launch update bit for bit (narrow gradient rows included)."""
    from mlx_gsplat_b200 import _lib
    from mlx_gsplat_b200.allocator import SlabLayout
    from mlx_gsplat_b200.optimizer import FusedMLXAdam
    L = SlabLayout(3)
    rng = np.random.default_rng(4)
    n, maxg = 40_000, 50_000
    theta = rng.normal(0, 1, (maxg, L.stride)).astype(np.float32)
    table = rng.permutation(maxg)[:n].astype(np.int32)
    seen = rng.uniform(0, 1, n) < 0.5
    words = np.zeros((n + 31) // 32, np.uint32)
    for r in np.nonzero(seen)[0]:
        words[r >> 5] |= np.uint32(1) << np.uint32(r & 31)
    g = rng.normal(0, 0.1, (maxg, 24)).astype(np.float32)
    g[:, 23] = 1.0
    unseen = np.zeros(L.ncols, np.float32)
    unseen[:11] = 1e-5
    coef = [1e-5 if c >= 23 else 0.0 for c in range(L.ncols)]
    lo, hi = L.col_bounds()
    out = []
    for split in (False, True):
        th = torch.from_numpy(theta.copy()).cuda()
        gg = torch.from_numpy(g).cuda()
        m = torch.zeros_like(th)
        v = torch.zeros_like(th)
        tab = torch.from_numpy(table).cuda()
        W = torch.from_numpy(words.view(np.int32)).cuda()
        opt = FusedMLXAdam(lr=1e-3, eps=1e-15)
        kw = dict(quat_col=0, visible_words=W.data_ptr(), unseen_grad=unseen.tolist(), g_cols=23, count_col=23,
                  count_coef=coef)
        for _ in range(2):
            if split:
                opt.step_slab(th, gg, m, v, tab, n, L.ncols, lo.tolist(), hi.tolist(),
                              row_select=_lib.GS_ROWS_UNSEEN, **kw)
                opt.step_slab(th, gg, m, v, tab, n, L.ncols, lo.tolist(), hi.tolist(),
                              row_select=_lib.GS_ROWS_SEEN, advance=False, **kw)
            else:
                opt.step_slab(th, gg, m, v, tab, n, L.ncols, lo.tolist(), hi.tolist(), **kw)
        torch.cuda.synchronize()
        out.append([x.cpu().numpy() for x in (th, m, v)])
    for a, b in zip(*out):
        np.testing.assert_array_equal(a, b)
    assert not np.array_equal(out[0][0], theta)


def test_gradient_row_modes_agree():
    """End to end through the trainer, the three ways of forming the gradient
    rows of unseen Gaussians: "sparse" (one GPU: regulariser rows selected by
    the visibility bits), "dense" (every row filled first) and "summed" (the
    multi-GPU form: rows without the geometry regulariser in a zeroed slab, the
    sum over GPUs — here one — and ``world * reg`` added by Adam).  The
    rasterizer's gradient reductions are float atomics, so two runs differ in
    the last bits; Adam turns that into parameter differences of a few ulp
    (tolerance 1e-5 relative)."""
    runs = []
    for mode in ("sparse", "dense", "summed"):
        r = runner_for_workload("mid-200k", max_steps=50, n=30_000, num_views=4, lr=1e-3, eps=1e-15)
        r.row_mode = mode
        for step in range(1, 4):
            r.train_step(step - 1, step)
        torch.cuda.synchronize()
        runs.append([t.cpu().numpy() for t in (r.allocator.theta, r.allocator.adam_m, r.allocator.adam_v)])
    for other in runs[1:]:
        np.testing.assert_allclose(runs[0][0], other[0], rtol=1e-5, atol=1e-6)


def test_training_reduces_loss():
    r = runner_for_workload("tiny-3k", max_steps=60, lr=1e-2, eps=1e-15)
    losses = []
    for step in range(1, 61):
        r.train_step((step - 1) % 8, step)
        if step % 8 == 1:
            losses.append(float(r.loss_value()))
    assert losses[-1] < 0.8 * losses[0], losses


@pytest.mark.parametrize("wl_name,n", [("tiny-3k", 3000), ("outdoor-small", None)])
def test_grad2d_statistic_matches_oracle(monkeypatch, wl_name, n):
    """The densification statistic of mlx_gsplat/trainer.py:300-318 over two
    steps: ``grad2d[slot] += sqrt(sum (dL/dmean + 1e-5)^2 + 1e-8) * |z| / fx``
    and ``count[slot] += 1`` at the physical slots of the visible Gaussians,
    accumulated by the projection backward.  Checked two ways each step:
    within 1e-5 relative of the oracle's ``grad2d_proxy`` evaluated on the
    GPU's own mean gradients (the formula itself), and within the gradient
    tolerance of the dense oracle's mean gradients (end to end); the counts
    exactly."""
    if wl_name == "outdoor-small":
        _small_outdoor(monkeypatch)
    r = runner_for_workload(wl_name, max_steps=50, n=n, num_views=4, lr=1e-3, eps=1e-15)
    r.row_mode = "dense"  # rows hold dL/dmean + 1e-5 for every Gaussian
    al, L = r.allocator, r.layout
    M = al.max_gaussians
    g2_exact = np.zeros(M, np.float64)
    g2_e2e = np.zeros(M, np.float64)
    cnt = np.zeros(M, np.float32)
    om = L.offsets["means"]
    for step, view in ((1, 0), (2, 1)):
        theta0 = al.theta.cpu().numpy().copy()
        table = al.indirection_table.cpu().numpy()
        frame = r.train_step(view, step)
        torch.cuda.synchronize()
        ids = frame.ids[:frame.V].cpu().numpy().astype(np.int64)
        assert ids.size > 0
        vm = r.viewmats[view]
        fx = float(r.K[0, 0])
        means = theta0[table][:, om:om + 3]
        grad = r.full_gradient_rows(step).cpu().numpy()
        gm_gpu = grad[ids, om:om + 3]
        slots = table[ids]
        g2_exact[slots] += odens.grad2d_proxy(gm_gpu, means[ids], vm, fx)
        # end to end: the dense oracle's own mean gradients (+ the 1e-5 regulariser)
        act = {k: theta0[table][:, o:o + L.dims[k]] for k, o in L.offsets.items()}
        colors = np.concatenate([act["sh0"], act["shN"]], 1)[:, :sh_cols_for(step, r.cfg)]
        C = frame.color.cpu().numpy()
        tgt = r.targets[view].cpu().numpy()
        tf = tgt.astype(np.float32) / np.float32(255.0) if tgt.dtype == np.uint8 else tgt
        dC = np.sign(C.astype(np.float64) - tf) / (3.0 * r.cfg.render_width * r.cfg.render_height)
        _, _, gr = orend.rasterize_dense_vjp(act["means"][ids], act["quats"][ids], act["scales"][ids],
                                             act["opacities"][ids], colors[ids], vm, r.K, r.cfg.width,
                                             r.cfg.height, r.cfg.render_width, r.cfg.render_height, dL_dC=dC)
        g2_e2e[slots] += odens.grad2d_proxy((gr["means"] + r.cfg.param_reg).astype(np.float32), means[ids], vm, fx)
        cnt[slots] += 1.0
        got = al.grad2d.cpu().numpy().astype(np.float64)
        np.testing.assert_array_equal(al.count.cpu().numpy(), cnt, err_msg=f"step {step} count")
        np.testing.assert_allclose(got, g2_exact, rtol=1e-5, atol=0, err_msg=f"step {step} grad2d (formula)")
        assert_grad_close(got, g2_e2e, what=f"step {step} grad2d (end to end)")
    assert cnt.max() == 2  # some Gaussians were seen by both views: the statistic accumulated
