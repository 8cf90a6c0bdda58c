"""The COLMAP scene loader and the target resize against the reference's own
code: ``tests/golden/colmap.npz`` holds the reference ``Parser``/``Dataset``
results (mlx_gsplat/dataset.py:258-479) on the committed fixture scene
``tests/golden/colmap_scene``, and ``resize.npz`` the reference
``bilinear_resize_mlx`` (mlx_gsplat/rendering.py:6-38) on seeded images
(both made by ``tests/golden/gen_golden.py``).  Index and image results are
compared exactly; the float64 pose arithmetic is the reference's, so poses,
intrinsics and points are compared exactly too."""
import os

import numpy as np
import pytest
import torch

from mlx_gsplat_b200 import dataset as D
from oracle import image as oimage

HERE = os.path.dirname(os.path.abspath(__file__))
SCENE = os.path.join(HERE, "golden", "colmap_scene")


@pytest.fixture(scope="module")
def colmap_golden():
    return np.load(os.path.join(HERE, "golden", "colmap.npz"))


@pytest.mark.parametrize("normalize", [False, True])
@pytest.mark.parametrize("factor", [1, 2])
def test_parser_matches_reference(colmap_golden, normalize, factor):
    g = colmap_golden
    key = f"n{int(normalize)}_f{factor}"
    p = D.Parser(SCENE, factor=factor, normalize=normalize)
    assert p.image_names == list(g[key + "_names"])
    assert [os.path.relpath(x, SCENE) for x in p.image_paths] == list(g[key + "_paths"])
    np.testing.assert_array_equal(p.camtoworlds, g[key + "_c2w"])
    assert p.camera_ids == list(g[key + "_camera_ids"])
    for cid in p.Ks_dict:
        np.testing.assert_array_equal(p.Ks_dict[cid], g[f"{key}_K{cid}"])
        assert tuple(p.imsize_dict[cid]) == tuple(g[f"{key}_imsize{cid}"])
        np.testing.assert_array_equal(p.params_dict[cid], g[f"{key}_params{cid}"])
    np.testing.assert_array_equal(p.points, g[key + "_points"])
    np.testing.assert_array_equal(p.points_rgb, g[key + "_points_rgb"])
    np.testing.assert_array_equal(p.points_err, g[key + "_points_err"])
    np.testing.assert_array_equal(p.transform, g[key + "_transform"])
    assert p.scene_scale == float(g[key + "_scene_scale"])
    for split in ("train", "test"):
        d = D.Dataset(p, split=split, preload_images=True)
        np.testing.assert_array_equal(d.indices, g[f"{key}_{split}_indices"])
        item = d[1]
        np.testing.assert_array_equal(item["K"].numpy(), g[f"{key}_{split}_item1_K"])
        np.testing.assert_array_equal(item["camtoworld"].numpy(), g[f"{key}_{split}_item1_c2w"])
        np.testing.assert_array_equal(item["image"].numpy(), g[f"{key}_{split}_item1_image"])


def test_binary_readers_round_trip(tmp_path):
    """Every COLMAP camera model: written, read back, and the pinhole part taken
    from COLMAP's parameter order (one focal length for the SIMPLE_* and
    RADIAL* models)."""
    cams = []
    for mid, (name, npar, single) in D.CAMERA_MODELS.items():
        cams.append(D.Camera(mid + 1, name, 100 + mid, 50 + mid, [10.0 + k for k in range(npar)]))
    D.write_cameras_binary(cams, str(tmp_path / "cameras.bin"))
    back = D.read_cameras_binary(str(tmp_path / "cameras.bin"))
    assert list(back) == [c.camera_id for c in cams]
    for c in cams:
        b = back[c.camera_id]
        assert (b.camera_type, b.width, b.height, b.params) == (c.camera_type, c.width, c.height, c.params)
        single = D.CAMERA_MODELS[D.CAMERA_MODEL_IDS[c.camera_type]][2]
        want = (10.0, 10.0, 11.0, 12.0) if single else (10.0, 11.0, 12.0, 13.0)
        assert (b.fx, b.fy, b.cx, b.cy) == want
    xyz = np.arange(12, dtype=np.float64).reshape(4, 3) / 7
    rgb = np.array([[1, 2, 3], [4, 5, 6], [7, 8, 9], [250, 251, 252]])
    err = np.array([0.5, 0.25, 2.0, 0.0])
    tracks = [np.zeros((0, 2)), np.array([[1, 2]]), np.array([[3, 4], [5, 6], [7, 8]]), np.zeros((0, 2))]
    D.write_points3D_binary(xyz, rgb, err, tracks, str(tmp_path / "points3D.bin"))
    p, c, e = D.read_points3D_binary(str(tmp_path / "points3D.bin"))
    np.testing.assert_array_equal(p, xyz.astype(np.float32))
    np.testing.assert_array_equal(c, rgb.astype(np.uint8))
    np.testing.assert_array_equal(e, err.astype(np.float32))


def test_missing_sparse_dir_raises(tmp_path):
    with pytest.raises(FileNotFoundError):
        D.Parser(str(tmp_path))


def test_jpg_sources_are_downscaled_to_png(tmp_path):
    """factor > 1 with JPEG sources: the images are downscaled (bicubic, rounded
    size) into images_<factor>_png and read from there (dataset.py:224-243, 335-340)."""
    import shutil

    from PIL import Image
    scene = tmp_path / "scene"
    shutil.copytree(os.path.join(SCENE, "sparse"), scene / "sparse")
    (scene / "images").mkdir()
    for f in sorted(os.listdir(os.path.join(SCENE, "images"))):
        im = Image.open(os.path.join(SCENE, "images", f))
        im.save(scene / "images" / f, format="JPEG")  # JPEG bytes under the COLMAP names
    # COLMAP's names end in .png here; a .jpg first file triggers the resize, so rename
    for f in sorted(os.listdir(scene / "images")):
        os.rename(scene / "images" / f, scene / "images" / (os.path.splitext(f)[0] + ".jpg"))
    import struct
    src = open(os.path.join(SCENE, "sparse", "0", "images.bin"), "rb").read()
    (scene / "sparse" / "0" / "images.bin").write_bytes(src.replace(b".png\x00", b".jpg\x00"))
    assert struct.unpack("<Q", src[:8])[0] == 10
    p = D.Parser(str(scene), factor=2)
    assert all(x.endswith(".png") and "images_2_png" in x for x in p.image_paths)
    assert D.imread_rgb(p.image_paths[0]).shape == (15, 20, 3)
    assert tuple(p.imsize_dict[1]) == (20, 15)


def test_resize_oracle_matches_reference():
    d = np.load(os.path.join(HERE, "golden", "resize.npz"))
    i = 0
    while f"img_{i}" in d:
        ho, wo = d[f"size_{i}"]
        got = oimage.target_from_u8(d[f"img_{i}"], int(ho), int(wo))
        np.testing.assert_array_equal(got, d[f"out_{i}"], err_msg=f"case {i}")
        i += 1
    assert i >= 6


# ----------------------------------------------------------------------------- GPU
@pytest.mark.gpu
def test_resize_kernel_matches_reference_bit_exact():
    from mlx_gsplat_b200 import bilinear_resize_mlx
    d = np.load(os.path.join(HERE, "golden", "resize.npz"))
    i = 0
    while f"img_{i}" in d:
        ho, wo = (int(x) for x in d[f"size_{i}"])
        img = torch.from_numpy(d[f"img_{i}"]).cuda()
        got = bilinear_resize_mlx(img, ho, wo).cpu().numpy()
        np.testing.assert_array_equal(got, d[f"out_{i}"], err_msg=f"uint8 case {i}")
        # the float input divided on the host (a true division, as the reference's)
        imgf = torch.from_numpy(d[f"img_{i}"].astype(np.float32) / np.float32(255.0)).cuda()
        gotf = bilinear_resize_mlx(imgf, ho, wo).cpu().numpy()
        np.testing.assert_array_equal(gotf, d[f"out_{i}"], err_msg=f"float case {i}")
        i += 1


@pytest.mark.gpu
def test_resize_kernel_large_image_vs_oracle():
    """A full-size target (1297x840 -> 648x420 and -> 1297x840) against the
    NumPy restatement, bit for bit."""
    from mlx_gsplat_b200 import bilinear_resize_mlx
    rng = np.random.default_rng(3)
    img = rng.integers(0, 256, (840, 1297, 3), dtype=np.uint8)
    t = torch.from_numpy(img).cuda()
    for ho, wo in ((420, 648), (840, 1297), (1080, 1920)):
        got = bilinear_resize_mlx(t, ho, wo).cpu().numpy()
        np.testing.assert_array_equal(got, oimage.target_from_u8(img, ho, wo), err_msg=f"{wo}x{ho}")


@pytest.mark.gpu
def test_dataset_device_images_match_host_cache():
    p = D.Parser(SCENE, factor=1, normalize=True)
    d = D.Dataset(p, split="train")
    for i in range(len(d)):
        up = d.device_image(i, "cuda").cpu()
        assert torch.equal(up, d.image_u8(i))
    assert d.to_device("cuda") == sum(int(t.numel()) for t in d.preloaded_images.values())
    for i in range(len(d)):
        assert torch.equal(d.device_image(i, "cuda").cpu(), d.image_u8(i))


@pytest.mark.gpu
@pytest.mark.parametrize("render_size", [(40, 30), (24, 18)], ids=["native", "resized"])
def test_trainer_on_colmap_scene(render_size):
    """``RunnerMLX(cfg)`` on the fixture scene, as the reference trainer starts
    on real data: normalised scene, Gaussians from the SfM points, one camera
    per training image (world-to-camera = inverse of the parser's pose), and
    each step's target the uint8 image, resized on the GPU to the render size
    (bit for bit the reference's ``bilinear_resize_mlx(image / 255.0)``)."""
    from mlx_gsplat_b200.trainer import MLXConfig, RunnerMLX
    from oracle import rendering as orend
    RW, RH = render_size
    cfg = MLXConfig(max_gaussians=2000, max_steps=6, data_dir=SCENE, data_factor=1, render_width=RW,
                    render_height=RH, sh_degree=3, densify=False, opacity_reset=False, lr=1e-3)
    r = RunnerMLX(cfg)
    p = D.Parser(SCENE, factor=1, normalize=True)
    assert r.allocator.num_active == len(p.points) == 300
    assert len(r.cams) == len(r.train_dataset) == 8
    np.testing.assert_allclose(r.viewmats[2], np.linalg.inv(p.camtoworlds[r.train_dataset.indices[2]]),
                               rtol=0, atol=1e-6)
    assert r.scene_scale == float(p.scene_scale)
    for item in (0, 5):
        tgt = r.dataset_target(item).cpu().numpy()
        img = r.train_dataset.image_u8(item).numpy()
        want = img if (RW, RH) == (40, 30) else oimage.target_from_u8(img, RH, RW)
        np.testing.assert_array_equal(tgt, want)
    # the cull of one view against the oracle on the same (uploaded) Gaussians
    al, L = r.allocator, r.layout
    th = al.theta.cpu().numpy()[al.indirection_table.cpu().numpy()]
    frame = r.train_step(3, 1)
    ref = orend.cull(th[:, L.offsets["means"]:L.offsets["means"] + 3], th[:, L.offsets["opacities"]],
                     r.viewmats[3], r.K[3] if r.K.ndim == 3 else r.K, 40, 30)
    np.testing.assert_array_equal(frame.ids[:frame.V].cpu().numpy(), ref)
    assert frame.V > 0
    r.train()
    assert np.isfinite(float(r.loss_value()))


@pytest.mark.gpu
def test_trainer_reference_synthetic_mode():
    """Without a COLMAP scene the reference trainer runs its synthetic mode:
    3,000 random Gaussians, an identity camera, no target (loss mean(render))."""
    from mlx_gsplat_b200.trainer import MLXConfig, RunnerMLX
    cfg = MLXConfig(max_gaussians=10_000, max_steps=5, use_real_data=False, densify=False, lr=1e-3)
    r = RunnerMLX(cfg)
    assert r.allocator.num_active == 3000 and r.train_dataset is None and r.targets is None
    r.train(log_every=0)
    f = r.last_frame
    assert (f.cam.render_width, f.cam.render_height) == (200, 150) and f.V > 0
    assert abs(float(r.loss_value()) - float(f.color.mean())) < 1e-6


@pytest.mark.gpu
def test_command_line_trains_and_exports(tmp_path, monkeypatch):
    """``python -m mlx_gsplat_b200.train`` on the fixture scene: trains with the
    reference's loss and writes ``<scene>_mlx_custom_3dgs.ply`` at the end."""
    from mlx_gsplat_b200 import train
    monkeypatch.chdir(tmp_path)
    r = train.main(["--data_dir", SCENE, "--max_steps", "5", "--data_factor", "1", "--render_width", "24",
                    "--render_height", "18", "--max_gaussians", "2000"])
    out = tmp_path / "colmap_scene_mlx_custom_3dgs.ply"
    assert out.exists() and out.stat().st_size > 300 * 14 * 4
    assert r.cfg.loss == "l1+dssim" and np.isfinite(float(r.loss_value()))
