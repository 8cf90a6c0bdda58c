"""Generate the golden fixtures under ``tests/golden/`` by running the
reference's own, unmodified Python (``mlx_gsplat/rendering.py``,
``optimizer.py``, ``allocator.py``, and the ``_ssim`` method of
``trainer.py``) on seeded inputs.

MLX is not installable here, so ``tests/golden/mlx_shim`` stands in for
``mlx.core`` over torch-CPU (see its docstring).  The fixtures are small
``.npz`` files committed next to this script; they pin the CPU oracle
(``tests/test_oracle_golden.py``).  Run from the repository root:

    python tests/golden/gen_golden.py REFERENCE_ROOT

The reference checkout is needed only to regenerate; the tests read the
committed fixtures.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(HERE, "mlx_shim"))
sys.path.insert(0, ROOT)

import mlx.core as mx  # noqa: E402  (the shim)
from mlx_gsplat_b200 import synthetic  # noqa: E402


def load_ref(ref_root: str, name: str):
    path = os.path.join(ref_root, "mlx_gsplat", name + ".py")
    spec = importlib.util.spec_from_file_location("ref_" + name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def small_scene(n, seed, wl_name="tiny-3k", sh_dim=3):
    wl = synthetic.WORKLOADS[wl_name]
    g = synthetic.make_gaussians(wl, seed=seed, n=n)
    rng = np.random.default_rng(seed + 100)
    colors = g["sh0"]
    if sh_dim > 3:
        colors = np.concatenate([g["sh0"], rng.normal(0, 0.5, (n, sh_dim - 3)).astype(np.float32)], 1)
    return g, colors.astype(np.float32)


def gen_cull(R, out):
    wl = synthetic.WORKLOADS["tiny-3k"]
    g = synthetic.make_gaussians(wl, seed=0, n=3000)
    # widen the spread so that all cull edges are exercised
    g["means"] = (g["means"] * np.float32(3.0)).astype(np.float32)
    views, K = synthetic.make_cameras(wl, seed=2, num_views=8)
    res = {"means": g["means"], "opacities": g["opacities"], "views": views, "K": K,
           "width": np.int32(wl.width), "height": np.int32(wl.height)}
    for i, vm in enumerate(views):
        ids = R.frustum_culling_mlx(mx.array(g["means"]), mx.array(g["quats"]), mx.array(g["scales"]),
                                    mx.array(vm), mx.array(K), wl.width, wl.height,
                                    opacities=mx.array(g["opacities"]))
        res[f"ids_{i}"] = np.array(ids).astype(np.int32)
    # nothing visible: camera looking away -> the reference returns N entries of -1
    away = views[0].copy()
    away[:3, :3] = -away[:3, :3]
    away[:3, 3] = -away[:3, 3]
    ids = R.frustum_culling_mlx(mx.array(g["means"]), mx.array(g["quats"]), mx.array(g["scales"]),
                                mx.array(away), mx.array(K), wl.width, wl.height,
                                opacities=mx.array(g["opacities"]))
    res["away_view"] = away
    res["ids_away"] = np.array(ids).astype(np.int32)
    np.savez_compressed(os.path.join(out, "cull.npz"), **res)


def gen_raster(R, out):
    cases = [
        # name, n, sh_dim, W, H, RW, RH, seed
        ("sh0", 160, 3, 48, 36, 48, 36, 10),
        ("sh1", 160, 12, 48, 36, 48, 36, 11),
        ("sh3", 120, 48, 40, 30, 40, 30, 12),
        ("scaled", 140, 12, 64, 48, 32, 24, 13),
    ]
    res = {}
    wl = synthetic.WORKLOADS["tiny-3k"]
    for name, n, shd, W, H, RW, RH, seed in cases:
        g, colors = small_scene(n, seed, sh_dim=shd)
        views, _ = synthetic.make_cameras(wl, seed=2, num_views=3)
        vm = views[seed % 3]
        K = np.array([[W * 0.9, 0, W / 2.0], [0, W * 0.9, H / 2.0], [0, 0, 1]], np.float32)
        ids = R.frustum_culling_mlx(mx.array(g["means"]), mx.array(g["quats"]), mx.array(g["scales"]),
                                    mx.array(vm), mx.array(K), W, H, opacities=mx.array(g["opacities"]))
        ids = mx.array(np.array(ids), dtype=mx.int32)
        rng = np.random.default_rng(seed + 7)
        target = rng.uniform(0, 1, (RH, RW, 3)).astype(np.float32)
        wA = rng.uniform(-1, 1, (RH, RW, 1)).astype(np.float32)
        tgt = mx.array(target)
        wa = mx.array(wA)

        # colours one row per visible Gaussian (the trainer's calling form)
        col_vis = colors[np.array(ids).astype(np.int64)]

        def loss_fn(p):
            c, a = R.rasterize_gaussians_mlx(p["means"], p["quats"], p["scales"], p["opacities"], p["colors"],
                                             mx.array(vm), mx.array(K), W, H, ids,
                                             render_width=RW, render_height=RH, pixel_chunk_size=512)
            return mx.mean(mx.abs(c - tgt)) + mx.mean(a * wa)

        params = {"means": mx.array(g["means"]), "quats": mx.array(g["quats"]),
                  "scales": mx.array(g["scales"]), "opacities": mx.array(g["opacities"]),
                  "colors": mx.array(col_vis)}
        c, a = R.rasterize_gaussians_mlx(params["means"], params["quats"], params["scales"],
                                         params["opacities"], params["colors"], mx.array(vm), mx.array(K),
                                         W, H, ids, render_width=RW, render_height=RH)
        loss, grads = mx.value_and_grad(loss_fn)(params)
        pre = f"{name}_"
        res.update({pre + "means": g["means"], pre + "quats": g["quats"], pre + "scales": g["scales"],
                    pre + "opacities": g["opacities"], pre + "colors": col_vis, pre + "viewmat": vm,
                    pre + "K": K, pre + "dims": np.array([W, H, RW, RH], np.int32),
                    pre + "ids": np.array(ids).astype(np.int32), pre + "target": target, pre + "wA": wA,
                    pre + "out_colors": np.array(c), pre + "out_alphas": np.array(a),
                    pre + "loss": np.array(loss)})
        for k, v in grads.items():
            res[pre + "grad_" + k] = np.array(v)
    np.savez_compressed(os.path.join(out, "raster.npz"), **res)


def gen_raster_mask(R, out):
    """The rasterizer's alpha mask (rendering.py:289-290), one case with
    colours of SH degree 1: mask values uniform in [0, 1] with a fifth of them
    exactly 0 and a fifth exactly 1; ``raster_mask.npz``."""
    W, H, RW, RH, seed = 48, 36, 48, 36, 21
    wl = synthetic.WORKLOADS["tiny-3k"]
    g, colors = small_scene(160, seed, sh_dim=12)
    views, _ = synthetic.make_cameras(wl, seed=2, num_views=3)
    vm = views[seed % 3]
    K = np.array([[W * 0.9, 0, W / 2.0], [0, W * 0.9, H / 2.0], [0, 0, 1]], np.float32)
    ids = R.frustum_culling_mlx(mx.array(g["means"]), mx.array(g["quats"]), mx.array(g["scales"]),
                                mx.array(vm), mx.array(K), W, H, opacities=mx.array(g["opacities"]))
    ids = mx.array(np.array(ids), dtype=mx.int32)
    V = int(np.array(ids).shape[0])
    rng = np.random.default_rng(seed + 7)
    mask = rng.uniform(0, 1, V).astype(np.float32)
    pick = rng.permutation(V)
    mask[pick[:V // 5]] = 0.0
    mask[pick[V // 5:2 * (V // 5)]] = 1.0
    target = rng.uniform(0, 1, (RH, RW, 3)).astype(np.float32)
    wA = rng.uniform(-1, 1, (RH, RW, 1)).astype(np.float32)
    tgt, wa, mk = mx.array(target), mx.array(wA), mx.array(mask)
    col_vis = colors[np.array(ids).astype(np.int64)]

    def loss_fn(p):
        c, a = R.rasterize_gaussians_mlx(p["means"], p["quats"], p["scales"], p["opacities"], p["colors"],
                                         mx.array(vm), mx.array(K), W, H, ids, render_width=RW, render_height=RH,
                                         pixel_chunk_size=512, mask=mk)
        return mx.mean(mx.abs(c - tgt)) + mx.mean(a * wa)

    params = {"means": mx.array(g["means"]), "quats": mx.array(g["quats"]), "scales": mx.array(g["scales"]),
              "opacities": mx.array(g["opacities"]), "colors": mx.array(col_vis)}
    c, a = R.rasterize_gaussians_mlx(params["means"], params["quats"], params["scales"], params["opacities"],
                                     params["colors"], mx.array(vm), mx.array(K), W, H, ids, render_width=RW,
                                     render_height=RH, mask=mk)
    loss, grads = mx.value_and_grad(loss_fn)(params)
    res = {"means": g["means"], "quats": g["quats"], "scales": g["scales"], "opacities": g["opacities"],
           "colors": col_vis, "viewmat": vm, "K": K, "dims": np.array([W, H, RW, RH], np.int32),
           "ids": np.array(ids).astype(np.int32), "mask": mask, "target": target, "wA": wA,
           "out_colors": np.array(c), "out_alphas": np.array(a), "loss": np.array(loss)}
    for k, v in grads.items():
        res["grad_" + k] = np.array(v)
    np.savez_compressed(os.path.join(out, "raster_mask.npz"), **res)


def gen_adam(O, out):
    rng = np.random.default_rng(5)
    dims = {"means": 3, "scales": 3, "quats": 4, "opacities": 1, "sh0": 3, "shN": 9}
    n = 50
    p = {k: rng.normal(0, 1, (n, d)).astype(np.float32) for k, d in dims.items()}
    m = {k: np.zeros((n, d), np.float32) for k, d in dims.items()}
    v = {k: np.zeros((n, d), np.float32) for k, d in dims.items()}
    opt = O.FusedMLXAdam(lr=1e-3, betas=(0.9, 0.999), eps=1e-15)
    res = {}
    for k in dims:
        res["p0_" + k] = p[k]
    for t in range(1, 4):
        gr = {k: rng.normal(0, 0.1, (n, d)).astype(np.float32) for k, d in dims.items()}
        for k in dims:
            res[f"g{t}_" + k] = gr[k]
        up, um, uv = opt.step({k: mx.array(x) for k, x in p.items()}, {k: mx.array(x) for k, x in gr.items()},
                              {k: mx.array(x) for k, x in m.items()}, {k: mx.array(x) for k, x in v.items()},
                              use_metal_fusion=False)
        p = {k: np.array(x) for k, x in up.items()}
        m = {k: np.array(x) for k, x in um.items()}
        v = {k: np.array(x) for k, x in uv.items()}
        for k in dims:
            res[f"p{t}_" + k] = p[k]
            res[f"m{t}_" + k] = m[k]
            res[f"v{t}_" + k] = v[k]
    np.savez_compressed(os.path.join(out, "adam_pure.npz"), **res)


def gen_alloc(A, out):
    rng = np.random.default_rng(9)
    maxg, sh = 96, 1
    alloc = A.PointerStableChunkedAllocator(max_gaussians=maxg, sh_degree=sh)
    n0 = 60
    dims = {"means": 3, "scales": 3, "quats": 4, "opacities": 1, "sh0": 3, "shN": 9}
    init = {k: rng.normal(0, 1, (n0, d)).astype(np.float32) for k, d in dims.items()}
    alloc.set_initial_gaussians({k: mx.array(x) for k, x in init.items()})
    res = {"init_" + k: x for k, x in init.items()}
    res["table0"] = alloc.indirection_table.copy()
    res["free0"] = np.array(alloc.free_slots, np.int32)
    for r in range(3):
        n = alloc.num_active
        prune = rng.uniform(0, 1, n) < 0.15
        split = rng.uniform(0, 1, n) < 0.25
        ns = int(split.sum())
        sp = {}
        for k, d in dims.items():
            sp[k + "_child1"] = rng.normal(0, 1, (ns, d)).astype(np.float32)
            sp[k + "_child2"] = rng.normal(0, 1, (ns, d)).astype(np.float32)
        for k, x in sp.items():
            res[f"r{r}_sp_{k}"] = x
        res[f"r{r}_prune"] = prune
        res[f"r{r}_split"] = split
        n_p, n_s = alloc.split_and_prune(prune, split, {k: mx.array(x) for k, x in sp.items()})
        res[f"r{r}_counts"] = np.array([n_p, n_s], np.int32)
        res[f"r{r}_table"] = alloc.indirection_table.astype(np.int32).copy()
        res[f"r{r}_free"] = np.array(alloc.free_slots, np.int32)
        for k in dims:
            res[f"r{r}_pool_{k}"] = np.array(alloc.physical_pools[k])
            res[f"r{r}_m_{k}"] = np.array(alloc.adam_m_pools[k])
    # capacity error: ask for more splits than free slots
    n = alloc.num_active
    split = np.ones(n, bool)
    prune = np.zeros(n, bool)
    ns = n
    sp = {k + s: np.zeros((ns, d), np.float32) for k, d in dims.items() for s in ("_child1", "_child2")}
    try:
        alloc.split_and_prune(prune, split, {k: mx.array(x) for k, x in sp.items()})
        res["oom_raised"] = np.array(False)
    except MemoryError:
        res["oom_raised"] = np.array(True)
    np.savez_compressed(os.path.join(out, "allocator.npz"), **res)


def load_ref_ssim(ref_root: str):
    """The reference trainer's ``_ssim`` method (``mlx_gsplat/trainer.py``),
    taken from the file's own text and executed as a plain function over the
    shim: the trainer module itself needs its whole runtime to import."""
    import textwrap
    src = open(os.path.join(ref_root, "mlx_gsplat", "trainer.py")).read()
    start = src.index("    def _ssim(")
    end = src.index("\n    def ", start + 1)
    ns = {"mx": mx}
    exec(textwrap.dedent(src[start:end]), ns)
    return ns["_ssim"]


def gen_ssim(ref_root, out):
    """Loss and gradient of the reference trainer's image loss with a target,
    0.8 * mean|C - T| + 0.2 * 0.5 * (1 - SSIM(C, T)) (trainer.py:276-279), for
    rendered images C against targets T, through the shim's value_and_grad."""
    ssim = load_ref_ssim(ref_root)
    res = {}
    for i, (h, w) in enumerate([(37, 53), (90, 120), (16, 16)]):
        rng = np.random.default_rng(40 + i)
        c = rng.uniform(0, 1, (h, w, 3)).astype(np.float32)
        t = np.clip(c + rng.normal(0, 0.15, (h, w, 3)), 0, 1).astype(np.float32)
        if i == 2:
            t = rng.uniform(0, 1, (h, w, 3)).astype(np.float32)  # unrelated images
        tt = mx.array(t)

        def loss_fn(params):
            pred = params["c"]
            l1 = mx.mean(mx.abs(pred - tt))
            d_ssim = 0.5 * (1.0 - ssim(None, pred, tt))
            return 0.8 * l1 + 0.2 * d_ssim

        loss, grads = mx.value_and_grad(loss_fn)({"c": mx.array(c)})
        res[f"c_{i}"] = c
        res[f"t_{i}"] = t
        res[f"ssim_{i}"] = np.asarray(ssim(None, mx.array(c), tt).detach().numpy(), np.float32)
        res[f"loss_{i}"] = np.asarray(loss.detach().numpy(), np.float32)
        res[f"grad_{i}"] = grads["c"].detach().numpy().astype(np.float32)
    np.savez_compressed(os.path.join(out, "ssim.npz"), **res)


def gen_resize(R, out):
    """The reference's own ``bilinear_resize_mlx`` on seeded images (the
    trainer's ``image / 255.0`` first): downscale, upscale, identity, odd
    ratios and single-row/column outputs."""
    rng = np.random.default_rng(7)
    res = {}
    cases = [(37, 23, 16, 11), (37, 23, 64, 40), (37, 23, 37, 23), (50, 31, 7, 5), (20, 9, 1, 1), (33, 17, 33, 1)]
    for i, (wi, hi, wo, ho) in enumerate(cases):
        img = rng.integers(0, 256, (hi, wi, 3), dtype=np.uint8)
        pix = mx.array(img.astype(np.float32)) / 255.0
        res[f"img_{i}"] = img
        res[f"size_{i}"] = np.array([ho, wo], np.int32)
        res[f"out_{i}"] = np.asarray(R.bilinear_resize_mlx(pix, ho, wo)).astype(np.float32)
    np.savez_compressed(os.path.join(out, "resize.npz"), **res)


COLMAP_SCENE = os.path.join(HERE, "colmap_scene")


def write_colmap_scene(path):
    """A small seeded COLMAP scene: two cameras (PINHOLE, SIMPLE_RADIAL), ten
    images on a ring (ids and file order shuffled, so that name sorting
    matters), 300 points with tracks, 40x30 PNGs in images/ and 20x15 PNGs in
    images_2/."""
    from PIL import Image

    from mlx_gsplat_b200 import dataset as D
    rng = np.random.default_rng(11)
    os.makedirs(os.path.join(path, "sparse", "0"), exist_ok=True)
    cams = [D.Camera(1, "PINHOLE", 40, 30, [37.0, 36.0, 20.0, 15.0]),
            D.Camera(2, "SIMPLE_RADIAL", 40, 30, [35.5, 19.5, 14.5, 0.01])]
    D.write_cameras_binary(cams, os.path.join(path, "sparse", "0", "cameras.bin"))
    images = []
    order = rng.permutation(10)
    for j in order:
        ang = 2 * np.pi * j / 10
        cpos = np.array([4 * np.cos(ang), 0.5 + 0.2 * rng.normal(), 4 * np.sin(ang)])
        fwd = -cpos / np.linalg.norm(cpos)
        right = np.cross(fwd, [0.0, -1.0, 0.0])
        right /= np.linalg.norm(right)
        down = np.cross(fwd, right)
        Rw2c = np.stack([right, down, fwd])
        t = -Rw2c @ cpos
        # quaternion (w, x, y, z) of Rw2c, scaled by a non-unit factor (the reader normalises)
        w = np.sqrt(max(1e-12, 1 + np.trace(Rw2c))) / 2
        q = np.array([w, (Rw2c[2, 1] - Rw2c[1, 2]) / (4 * w), (Rw2c[0, 2] - Rw2c[2, 0]) / (4 * w),
                      (Rw2c[1, 0] - Rw2c[0, 1]) / (4 * w)]) * 1.3
        pts = np.stack([rng.uniform(0, 40, 5), rng.uniform(0, 30, 5), rng.integers(-1, 300, 5)], 1)
        images.append((int(100 + 7 * j), q, t, 1 + int(j % 2), f"img_{j:03d}.png", pts))
    D.write_images_binary(images, os.path.join(path, "sparse", "0", "images.bin"))
    xyz = rng.normal(0, 1, (300, 3))
    rgb = rng.integers(0, 256, (300, 3))
    err = rng.uniform(0, 2, 300)
    tracks = [np.stack([rng.integers(100, 170, k), rng.integers(0, 5, k)], 1) for k in rng.integers(0, 6, 300)]
    D.write_points3D_binary(xyz, rgb, err, tracks, os.path.join(path, "sparse", "0", "points3D.bin"))
    for sub, (w, h) in (("images", (40, 30)), ("images_2", (20, 15))):
        os.makedirs(os.path.join(path, sub), exist_ok=True)
        for j in range(10):
            yy, xx = np.mgrid[0:h, 0:w]
            base = np.stack([xx * 255 // w, yy * 255 // h, (xx + yy + 25 * j) % 256], -1)
            img = (base + rng.integers(0, 16, (h, w, 3))).clip(0, 255).astype(np.uint8)
            Image.fromarray(img).save(os.path.join(path, sub, f"img_{j:03d}.png"))


def _imageio_stand_in():
    """``imageio.v2`` (absent here) for the reference's dataset module: reads
    and writes through Pillow, which is what imageio uses for PNG/JPEG."""
    import types

    from PIL import Image
    v2 = types.ModuleType("imageio.v2")
    v2.imread = lambda p: np.asarray(Image.open(p))
    v2.imwrite = lambda p, a: Image.fromarray(np.asarray(a)).save(p)
    top = types.ModuleType("imageio")
    top.v2 = v2
    sys.modules["imageio"] = top
    sys.modules["imageio.v2"] = v2


def gen_colmap(ref_root, out):
    """The reference's own ``Parser`` and ``Dataset`` (dataset.py:258-479) on the
    fixture scene, normalised and not, at factor 1 and 2."""
    write_colmap_scene(COLMAP_SCENE)
    _imageio_stand_in()
    Dm = load_ref(ref_root, "dataset")
    res = {}
    for normalize in (False, True):
        for factor in (1, 2):
            key = f"n{int(normalize)}_f{factor}"
            p = Dm.Parser(COLMAP_SCENE, factor=factor, normalize=normalize)
            res[key + "_names"] = np.array(p.image_names)
            res[key + "_paths"] = np.array([os.path.relpath(x, COLMAP_SCENE) for x in p.image_paths])
            res[key + "_c2w"] = p.camtoworlds
            res[key + "_camera_ids"] = np.array(p.camera_ids)
            for cid, K in p.Ks_dict.items():
                res[f"{key}_K{cid}"] = K
                res[f"{key}_imsize{cid}"] = np.array(p.imsize_dict[cid])
                res[f"{key}_params{cid}"] = p.params_dict[cid]
            res[key + "_points"] = p.points
            res[key + "_points_rgb"] = p.points_rgb
            res[key + "_points_err"] = p.points_err
            res[key + "_transform"] = p.transform
            res[key + "_scene_scale"] = np.float64(p.scene_scale)
            for split in ("train", "test"):
                d = Dm.Dataset(p, split=split, preload_images=True)
                res[f"{key}_{split}_indices"] = d.indices
                item = d[1]
                res[f"{key}_{split}_item1_K"] = np.asarray(item["K"])
                res[f"{key}_{split}_item1_c2w"] = np.asarray(item["camtoworld"])
                res[f"{key}_{split}_item1_image"] = np.asarray(item["image"])
    np.savez_compressed(os.path.join(out, "colmap.npz"), **res)


def main():
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/gen_golden.py REFERENCE_ROOT [fixture ...]")
    ref_root = sys.argv[1]
    only = set(sys.argv[2:])  # e.g. raster_mask: regenerate only those fixtures
    torch.manual_seed(0)
    torch.set_num_threads(1)  # a fixed summation order for the reference's matmuls
    R = load_ref(ref_root, "rendering")
    O = load_ref(ref_root, "optimizer")
    cwd = os.getcwd()
    tmp_dir = tempfile.TemporaryDirectory(prefix="gen_golden_")
    os.chdir(tmp_dir.name)  # the allocator writes a log next to its own file; keep any stray output out of the repo
    try:
        A = load_ref(ref_root, "allocator")
        gens = {"cull": lambda: gen_cull(R, HERE), "raster": lambda: gen_raster(R, HERE),
                "raster_mask": lambda: gen_raster_mask(R, HERE), "adam_pure": lambda: gen_adam(O, HERE),
                "allocator": lambda: gen_alloc(A, HERE), "ssim": lambda: gen_ssim(ref_root, HERE),
                "resize": lambda: gen_resize(R, HERE), "colmap": lambda: gen_colmap(ref_root, HERE)}
        for name, gen in gens.items():
            if not only or name in only:
                gen()
    finally:
        os.chdir(cwd)
        tmp_dir.cleanup()
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
