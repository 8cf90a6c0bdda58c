"""Tile rasterizer (forward + backward) against the dense oracle and the
reference-generated golden vectors.  Tolerances: ``tests/gsutil.py``
(images 1e-4 absolute, gradients 1e-3 relative)."""
import os

import numpy as np
import pytest
import torch

from gsutil import assert_grad_close, assert_image_close
from mlx_gsplat_b200 import _lib, frustum_culling_mlx, rasterize_gaussians_mlx, synthetic
from mlx_gsplat_b200.rendering import (DEFAULT_SETTINGS, camera_struct, gaussians_struct, grads_struct,
                                       render_backward, render_forward)
from oracle import rendering as orend

pytestmark = pytest.mark.gpu
DEV = "cuda"
NAMES = ("means", "quats", "scales", "opacities", "colors")


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def _scene(wl_name, n, seed=0, sh_dim=None):
    wl = synthetic.WORKLOADS[wl_name]
    g = synthetic.make_gaussians(wl, seed=seed, n=n)
    cols = np.concatenate([g["sh0"], g["shN"]], 1)
    if sh_dim is not None:
        cols = cols[:, :sh_dim]
    return wl, g, cols.astype(np.float32)


@pytest.mark.parametrize("case", ["sh0", "sh1", "sh3", "scaled"])
def test_matches_reference_golden(golden_dir, case):
    d = np.load(os.path.join(golden_dir, "raster.npz"))
    p = lambda k: d[f"{case}_{k}"]  # noqa: E731
    W, H, RW, RH = [int(x) for x in p("dims")]
    params = {k: _t(p(k)).requires_grad_(True) for k in NAMES}
    ids = _t(p("ids"))
    C, A = rasterize_gaussians_mlx(params["means"], params["quats"], params["scales"], params["opacities"],
                                   params["colors"], p("viewmat"), p("K"), W, H, ids, render_width=RW,
                                   render_height=RH)
    assert_image_close(C.detach().cpu().numpy(), p("out_colors"), what="colors")
    assert_image_close(A.detach().cpu().numpy(), p("out_alphas"), what="alphas")
    loss = torch.mean(torch.abs(C - _t(p("target")))) + torch.mean(A * _t(p("wA")))
    loss.backward()
    assert abs(float(loss) - float(p("loss"))) < 1e-5
    for k in NAMES:
        assert_grad_close(params[k].grad.cpu().numpy(), p("grad_" + k), what=f"{case} grad {k}")


def test_alpha_mask_matches_reference_golden(golden_dir):
    """The reference's alpha mask (rendering.py:289-290): mask[j] multiplies the
    clipped alpha of the j-th visible Gaussian in depth order.  Golden from
    the reference's own rasterizer, with the same loss as the other cases."""
    d = np.load(os.path.join(golden_dir, "raster_mask.npz"))
    W, H, RW, RH = [int(x) for x in d["dims"]]
    params = {k: _t(d[k]).requires_grad_(True) for k in NAMES}
    C, A = rasterize_gaussians_mlx(params["means"], params["quats"], params["scales"], params["opacities"],
                                   params["colors"], d["viewmat"], d["K"], W, H, _t(d["ids"]), render_width=RW,
                                   render_height=RH, mask=_t(d["mask"]))
    assert_image_close(C.detach().cpu().numpy(), d["out_colors"], what="masked colors")
    assert_image_close(A.detach().cpu().numpy(), d["out_alphas"], what="masked alphas")
    loss = torch.mean(torch.abs(C - _t(d["target"]))) + torch.mean(A * _t(d["wA"]))
    loss.backward()
    assert abs(float(loss) - float(d["loss"])) < 1e-5
    for k in NAMES:
        assert_grad_close(params[k].grad.cpu().numpy(), d["grad_" + k], what=f"masked grad {k}")


def test_alpha_mask_full_image_vs_oracle():
    """A mask over the 3,000-Gaussian scene (values in [0, 1], some exactly 0
    and 1), whole image and every gradient against the dense oracle; and the
    mask's bounds are checked.  The mask goes by depth rank, and among 3,000
    Gaussians some depths are closer than float32 resolution: the oracle
    (float64) is told the depth order the float32 kernels rank by
    (``depth_order_f32``) to assign the mask values, and composites in its own."""
    wl, g, cols = _scene("tiny-3k", 3000, seed=3, sh_dim=12)
    views, K = synthetic.make_cameras(wl, seed=2)
    vm = views[5]
    params = {"means": _t(g["means"]), "quats": _t(g["quats"]), "scales": _t(g["scales"]),
              "opacities": _t(g["opacities"])}
    ids = frustum_culling_mlx(params["means"], None, None, vm, K, wl.width, wl.height,
                              opacities=params["opacities"])
    idn = ids.cpu().numpy()
    V = idn.size
    rng = np.random.default_rng(8)
    mask = rng.uniform(0, 1, V).astype(np.float32)
    mask[rng.permutation(V)[:V // 4]] = 0.0
    cols_vis = cols[idn.astype(np.int64)]
    for k in params:
        params[k].requires_grad_(True)
    params["colors"] = _t(cols_vis).requires_grad_(True)
    C, A = rasterize_gaussians_mlx(params["means"], params["quats"], params["scales"], params["opacities"],
                                   params["colors"], vm, K, wl.width, wl.height, ids, render_width=wl.width,
                                   render_height=wl.height, mask=_t(mask))
    wC = rng.uniform(-1, 1, (wl.height, wl.width, 3)).astype(np.float32) / wl.pixels
    torch.sum(C * _t(wC)).backward()
    ids64 = idn.astype(np.int64)
    Cr, Ar, gr = orend.rasterize_dense_vjp(g["means"][ids64], g["quats"][ids64], g["scales"][ids64],
                                           g["opacities"][ids64], cols_vis, vm, K, wl.width, wl.height, wl.width,
                                           wl.height, dL_dC=wC, chunk=256, mask=mask,
                                           mask_order=orend.depth_order_f32(g["means"][ids64], vm))
    assert_image_close(C.detach().cpu().numpy(), Cr, what="masked colors")
    assert_image_close(A.detach().cpu().numpy(), Ar, what="masked alphas")
    for k in ("means", "quats", "scales", "opacities"):
        ref = np.zeros_like(g[k], dtype=np.float64)
        ref[ids64] = gr[k]
        assert_grad_close(params[k].grad.cpu().numpy(), ref, what="masked grad " + k)
    assert_grad_close(params["colors"].grad.cpu().numpy(), gr["colors"], what="masked grad colors")
    for bad in (np.full(V, 1.5, np.float32), -np.ones(V, np.float32), np.ones(V + 1, np.float32)):
        with pytest.raises(ValueError):
            rasterize_gaussians_mlx(params["means"], params["quats"], params["scales"], params["opacities"],
                                    params["colors"], vm, K, wl.width, wl.height, ids, render_width=wl.width,
                                    render_height=wl.height, mask=_t(bad))


def _oracle_grads(g, cols_vis, ids, vm, K, W, H, dC, dA=None, pixel_ids=None, chunk=None):
    ids64 = ids.astype(np.int64)
    chunk = chunk or (256 if pixel_ids is None else 16)
    C, A, gr = orend.rasterize_dense_vjp(g["means"][ids64], g["quats"][ids64], g["scales"][ids64],
                                         g["opacities"][ids64], cols_vis, vm, K, W, H, W, H, dL_dC=dC, dL_dA=dA,
                                         pixel_ids=pixel_ids, chunk=chunk)
    full = {}
    for k in ("means", "quats", "scales", "opacities"):
        z = np.zeros_like(g[k], dtype=np.float64)
        z[ids64] = gr[k]
        full[k] = z
    full["colors"] = gr["colors"]
    return C, A, full


@pytest.mark.parametrize("sh_dim,saturate", [(3, False), (12, False), (12, True)],
                         ids=["sh0", "sh1", "sh1-saturated"])
def test_tiny_full_image_forward_backward_vs_oracle(sh_dim, saturate):
    """Whole image and every gradient against the dense oracle.  The saturated
    case raises every opacity logit by 8 (alpha clipped at 0.99), so that many
    pixels reach T < 1e-6 and stop compositing early; the dense oracle never
    stops, and the difference stays below the remaining transmittance."""
    wl, g, cols = _scene("tiny-3k", 3000, seed=0, sh_dim=sh_dim)
    if saturate:
        g = dict(g)
        g["opacities"] = (g["opacities"] + 8.0).astype(np.float32)
    views, K = synthetic.make_cameras(wl, seed=2)
    rng = np.random.default_rng(1)
    P = wl.pixels
    for vi in (0, 3):
        vm = views[vi]
        params = {"means": _t(g["means"]), "quats": _t(g["quats"]), "scales": _t(g["scales"]),
                  "opacities": _t(g["opacities"])}
        ids = frustum_culling_mlx(params["means"], None, None, vm, K, wl.width, wl.height,
                                  opacities=params["opacities"])
        idn = ids.cpu().numpy()
        cols_vis = cols[idn.astype(np.int64)]
        for k in params:
            params[k].requires_grad_(True)
        params["colors"] = _t(cols_vis).requires_grad_(True)
        C, A = rasterize_gaussians_mlx(params["means"], params["quats"], params["scales"], params["opacities"],
                                       params["colors"], vm, K, wl.width, wl.height, ids, render_width=wl.width,
                                       render_height=wl.height)
        wC = rng.uniform(-1, 1, (wl.height, wl.width, 3)).astype(np.float32) / P
        wA = rng.uniform(-1, 1, (wl.height, wl.width, 1)).astype(np.float32) / P
        (torch.sum(C * _t(wC)) + torch.sum(A * _t(wA))).backward()
        Cr, Ar, gr = _oracle_grads(g, cols_vis, idn, vm, K, wl.width, wl.height, wC, wA)
        if saturate:
            assert (1.0 - A.detach().cpu().numpy() < 1e-6).mean() > 0.05, "too few saturated pixels"
        assert_image_close(C.detach().cpu().numpy(), Cr, what=f"view {vi} colors")
        assert_image_close(A.detach().cpu().numpy(), Ar, what=f"view {vi} alphas")
        for k in NAMES:
            assert_grad_close(params[k].grad.cpu().numpy(), gr[k], what=f"view {vi} grad {k}")


def _subset(wl, n_pix, seed):
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(wl.pixels, n_pix, replace=False))


@pytest.mark.parametrize("wl_name,n,n_pix,view_ids,chunk", [("mid-200k", 200_000, 512, (1,), 16),
                                                            ("outdoor-1m", 1_000_000, 512, (1, 5), 16),
                                                            ("large-6m", 6_000_000, 32, (3,), 4)])
def test_full_size_pixel_subset_vs_oracle(wl_name, n, n_pix, view_ids, chunk):
    """Full-size scenes: the oracle evaluates only a pixel subset (dense over every
    visible Gaussian); the cotangent is non-zero only there.  The large scene
    (6,000,000 Gaussians at 3840x2160, about 2.8 M visible) runs 32 pixels;
    the outdoor scene two views of 512 pixels each."""
    sh_dim = 12 if synthetic.WORKLOADS[wl_name].sh_degree > 0 else 3
    wl, g, cols = _scene(wl_name, n, seed=0, sh_dim=sh_dim)
    views, K = synthetic.make_cameras(wl, seed=2, num_views=8)
    for vi in view_ids:
        vm = views[vi]
        params = {"means": _t(g["means"]), "quats": _t(g["quats"]), "scales": _t(g["scales"]),
                  "opacities": _t(g["opacities"])}
        ids = frustum_culling_mlx(params["means"], None, None, vm, K, wl.width, wl.height,
                                  opacities=params["opacities"])
        idn = ids.cpu().numpy()
        cols_vis = cols[idn.astype(np.int64)]
        for k in params:
            params[k].requires_grad_(True)
        params["colors"] = _t(cols_vis).requires_grad_(True)
        C, A = rasterize_gaussians_mlx(params["means"], params["quats"], params["scales"], params["opacities"],
                                       params["colors"], vm, K, wl.width, wl.height, ids, render_width=wl.width,
                                       render_height=wl.height)
        pix = _subset(wl, n_pix, seed=5 + vi)
        rng = np.random.default_rng(2 + vi)
        wsub = rng.uniform(-1, 1, (n_pix, 3)).astype(np.float32)
        wC = np.zeros((wl.pixels, 3), np.float32)
        wC[pix] = wsub
        (torch.sum(C * _t(wC.reshape(wl.height, wl.width, 3)))).backward()
        Cr, Ar, gr = _oracle_grads(g, cols_vis, idn, vm, K, wl.width, wl.height, wsub, None, pixel_ids=pix,
                                   chunk=chunk)
        Cg = C.detach().cpu().numpy().reshape(-1, 3)[pix]
        Ag = A.detach().cpu().numpy().reshape(-1, 1)[pix]
        assert_image_close(Cg, Cr, what=f"view {vi} colors at subset")
        assert_image_close(Ag, Ar, what=f"view {vi} alphas at subset")
        for k in NAMES:
            assert_grad_close(params[k].grad.cpu().numpy(), gr[k], what=f"{wl_name} view {vi} grad {k}")
        del params, C, A, gr


def test_fused_l1_loss_matches_autograd_path():
    wl, g, cols = _scene("mid-200k", 50_000, seed=1)
    views, K = synthetic.make_cameras(wl, seed=2, num_views=4)
    vm = views[2]
    target = synthetic.make_uint8_targets(wl, 1, seed=1)[0]
    gs = {k: _t(g[k]) for k in ("means", "quats", "scales", "opacities")}
    colors = _t(cols)
    ids = frustum_culling_mlx(gs["means"], None, None, vm, K, wl.width, wl.height, opacities=gs["opacities"])
    V = int(ids.numel())
    cam = camera_struct(vm, K, wl.width, wl.height, wl.width, wl.height)
    st = gaussians_struct(gs["means"], gs["quats"], gs["scales"], gs["opacities"], colors)
    T8 = _t(target)
    f = render_forward(st, ids, V, cam, DEFAULT_SETTINGS, torch.device(DEV), loss_mode=_lib.GS_LOSS_L1_U8,
                       target=T8)
    loss = float(f.loss_partials.sum()) / (3 * wl.pixels)
    Cn = f.color.cpu().numpy().astype(np.float64)
    ref_loss = np.mean(np.abs(Cn - target.astype(np.float32) / np.float32(255.0)))
    assert abs(loss - ref_loss) < 1e-6
    grads = {k: torch.zeros_like(v) for k, v in gs.items()}
    gcol = torch.zeros_like(colors)
    out = grads_struct(grads["means"], grads["quats"], grads["scales"], grads["opacities"], gcol, colors_write=3)
    render_backward(f, st, out, torch.device(DEV))
    # same thing through autograd with an explicit cotangent sign(C - t) / (3P)
    p2 = {k: v.clone().requires_grad_(True) for k, v in gs.items()}
    c2 = colors.clone().requires_grad_(True)
    C, A = rasterize_gaussians_mlx(p2["means"], p2["quats"], p2["scales"], p2["opacities"], c2, vm, K, wl.width,
                                   wl.height, ids, render_width=wl.width, render_height=wl.height)
    tf = T8.float() / 255.0
    torch.mean(torch.abs(C - tf)).backward()
    for k in gs:
        assert_grad_close(grads[k].cpu().numpy(), p2[k].grad.cpu().numpy(), rtol=1e-5, what=k)
    assert_grad_close(gcol.cpu().numpy(), c2.grad.cpu().numpy(), rtol=1e-5, what="colors")


def test_empty_and_degenerate_inputs():
    wl, g, cols = _scene("tiny-3k", 200, seed=4)
    views, K = synthetic.make_cameras(wl, seed=2)
    m = _t(g["means"])
    C, A = rasterize_gaussians_mlx(m, _t(g["quats"]), _t(g["scales"]), _t(g["opacities"]), _t(cols), views[0], K,
                                   wl.width, wl.height, torch.zeros(0, dtype=torch.int32, device=DEV),
                                   render_width=wl.width, render_height=wl.height)
    assert float(C.abs().sum()) == 0.0 and float(A.abs().sum()) == 0.0
    # one huge Gaussian just in front of the camera covering every tile, plus zero quats
    g2 = {k: v[:20].copy() for k, v in g.items()}
    cam_c = -(views[0][:3, :3].T @ views[0][:3, 3])
    fwd = -cam_c / np.linalg.norm(cam_c)
    g2["means"][0] = (cam_c + 0.05 * fwd).astype(np.float32)
    g2["scales"][0] = -2.0
    g2["quats"][1] = 0.0
    c2 = cols[:20]
    ids = np.arange(20, dtype=np.int32)
    params = {k: _t(g2[k]).requires_grad_(True) for k in ("means", "quats", "scales", "opacities")}
    params["colors"] = _t(c2).requires_grad_(True)
    C, A = rasterize_gaussians_mlx(params["means"], params["quats"], params["scales"], params["opacities"],
                                   params["colors"], views[0], K, wl.width, wl.height, _t(ids),
                                   render_width=wl.width, render_height=wl.height)
    rng = np.random.default_rng(0)
    wC = rng.uniform(-1, 1, C.shape).astype(np.float32) / wl.pixels
    torch.sum(C * _t(wC)).backward()
    Cr, Ar, gr = _oracle_grads(g2, c2, ids, views[0], K, wl.width, wl.height, wC.reshape(-1, 3))
    assert_image_close(C.detach().cpu().numpy(), Cr)
    assert_image_close(A.detach().cpu().numpy(), Ar)
    for k in NAMES:
        assert_grad_close(params[k].grad.cpu().numpy(), gr[k], what="degenerate grad " + k)


def test_binning_scratch_matches_warp_binning():
    """Binning with the scratch (recorded tile masks, CTA-wide counting and
    emission of splats whose box exceeds 256 tiles) gives exactly the entries
    of the all-warp binning, including for boxes of hundreds of tiles."""
    lib = _lib.lib()
    st = _lib.stream_ptr()
    wl, g, cols = _scene("mid-200k", 20_000, seed=3)
    g = dict(g)
    rng = np.random.default_rng(5)
    big = rng.random(g["scales"].shape[0]) < 0.03
    g["scales"] = np.where(big[:, None], g["scales"] + 2.5, g["scales"]).astype(np.float32)
    views, K = synthetic.make_cameras(wl, seed=2)
    vm = views[0]
    T = {k: _t(g[k]) for k in ("means", "quats", "scales", "opacities")}
    colors = _t(cols)
    ids = frustum_culling_mlx(T["means"], None, None, vm, K, wl.width, wl.height, opacities=T["opacities"])
    V = int(ids.numel())
    gst = gaussians_struct(T["means"], T["quats"], T["scales"], T["opacities"], colors)
    cam = camera_struct(vm, K, wl.width, wl.height, wl.width, wl.height)
    rs = DEFAULT_SETTINGS.cstruct()
    ntx, nty = (wl.width + 15) // 16, (wl.height + 15) // 16
    i32 = lambda n: torch.empty(max(n, 1), dtype=torch.int32, device=DEV)
    out = {}
    for mode in ("warp", "scratch"):
        splats = torch.empty((V, 12), dtype=torch.float32, device=DEV)
        dkeys, counts = i32(V), i32(V)
        bs = torch.empty(lib.gs_bin_scratch_bytes(V), dtype=torch.uint8, device=DEV) if mode == "scratch" else None
        _lib.check(lib.gs_project_forward(gst, ids.data_ptr(), V, cam, rs, splats.data_ptr(), dkeys.data_ptr(),
                                          counts.data_ptr(), _lib.ptr(bs), st))
        ks, order = i32(V), i32(V)
        sb = torch.empty(lib.gs_radix_sort_scratch_bytes(V), dtype=torch.uint8, device=DEV)
        _lib.check(lib.gs_radix_sort_pairs(dkeys.data_ptr(), None, ks.data_ptr(), order.data_ptr(), V, 0, 32,
                                           sb.data_ptr(), sb.numel(), st))
        offs = i32(V + 1)
        ob = torch.empty(lib.gs_bin_offsets_scratch_bytes(V), dtype=torch.uint8, device=DEV)
        _lib.check(lib.gs_bin_offsets(order.data_ptr(), counts.data_ptr(), V, offs.data_ptr(), ob.data_ptr(),
                                      ob.numel(), st))
        Kn = int(offs[V].item())
        keys, vals = i32(Kn), i32(Kn)
        flag = torch.zeros(1, dtype=torch.int32, device=DEV)
        _lib.check(lib.gs_bin_emit(splats.data_ptr(), order.data_ptr(), offs.data_ptr(), counts.data_ptr(), V, cam,
                                   rs, keys.data_ptr(), vals.data_ptr(), Kn, flag.data_ptr(), _lib.ptr(bs), st))
        out[mode] = (counts[:V].cpu().numpy(), keys[:Kn].cpu().numpy(), vals[:Kn].cpu().numpy(), int(flag.item()))
        if bs is not None:
            n_big = int(bs[256 * ((bs.data_ptr() + 255) // 256) - bs.data_ptr():][:4].view(torch.int32).item())
            assert n_big > 0, "the scene should have boxes of more than 256 tiles"
    for a, b, what in zip(out["warp"], out["scratch"], ("counts", "keys", "vals", "overflow")):
        np.testing.assert_array_equal(a, b, err_msg=what)
    assert out["warp"][3] == 0
    assert (out["warp"][1] < ntx * nty).all(), "no sentinel entries"
