"""COLMAP scenes for the trainer: binary model readers, world normalisation,
the train/test image split and the uint8 image cache, with the names and
results of the reference's ``mlx_gsplat/dataset.py``.

* ``read_cameras_binary`` / ``read_images_binary`` / ``read_points3D_binary``
  (dataset.py:101-214) read COLMAP's binary model files; the matching
  ``write_*_binary`` functions write them (for synthetic scenes and tests).
* ``similarity_from_cameras``, ``align_principle_axes``, ``transform_points``,
  ``transform_cameras`` (dataset.py:15-92): the normalisation the parser
  applies with ``normalize=True``.
* ``Parser`` (dataset.py:258-408) and ``Dataset`` (dataset.py:411-479) keep the
  reference's attributes and item dictionary.  Images are decoded with Pillow
  (the reference uses imageio, which decodes PNG/JPEG through Pillow too) and
  cached as uint8 — in pinned host memory, and optionally in HBM
  (``Dataset.to_device``), so that a training step uploads (or reads) 3 bytes
  per pixel instead of 12.

Differences from the reference, each deliberate:
* camera models: the number of parameters and the focal/centre positions
  follow COLMAP's own model table for every model id; the reference assumes 4
  parameters for ids above 5 and reads ``RADIAL`` (f, cx, cy, k1, k2) as if
  it had two focal lengths.  Ids 0-2 and 4-5 read identically.
* ``Dataset`` random patches use a seeded generator (``seed``) instead of the
  global NumPy state.
"""
from __future__ import annotations

import os
import struct
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

# ============================================================================ normalisation
# (dataset.py:15-92; same arithmetic, so normalised scenes match the reference's)


def similarity_from_cameras(c2w: np.ndarray, strict_scaling: bool = False, center_method: str = "focus") -> np.ndarray:
    """4x4 similarity that rotates the cameras' mean up vector (-y of each
    camera) onto -y, centres the scene at the median of the points nearest to
    the origin along each camera's viewing ray ("focus") or at the median
    camera position ("poses"), and scales the median (or, strict, maximum)
    camera distance to 1."""
    t = c2w[:, :3, 3]
    R = c2w[:, :3, :3]
    ups = np.sum(R * np.array([0, -1.0, 0]), axis=-1)
    world_up = np.mean(ups, axis=0)
    world_up /= np.linalg.norm(world_up)
    up_cam = np.array([0.0, -1.0, 0.0])
    c = (up_cam * world_up).sum()
    v = np.cross(world_up, up_cam)
    vx = np.array([[0.0, -v[2], v[1]], [v[2], 0.0, -v[0]], [-v[1], v[0], 0.0]])
    if c > -1:
        R_align = np.eye(3) + vx + (vx @ vx) * 1 / (1 + c)  # Rodrigues form of the rotation taking up to -y
    else:
        R_align = np.array([[-1.0, 0.0, 0.0], [0.0, 1.0, 0.0], [0.0, 0.0, 1.0]])
    R = R_align @ R
    fwds = np.sum(R * np.array([0, 0.0, 1.0]), axis=-1)
    t = (R_align @ t[..., None])[..., 0]
    if center_method == "focus":
        nearest = t + (fwds * -t).sum(-1)[:, None] * fwds
        translate = -np.median(nearest, axis=0)
    elif center_method == "poses":
        translate = -np.median(t, axis=0)
    else:
        raise ValueError(f"Unknown center_method {center_method}")
    transform = np.eye(4)
    transform[:3, 3] = translate
    transform[:3, :3] = R_align
    scale_fn = np.max if strict_scaling else np.median
    scale = 1.0 / scale_fn(np.linalg.norm(t + translate, axis=-1))
    transform[:3, :] *= scale
    return transform


def align_principle_axes(point_cloud: np.ndarray) -> np.ndarray:
    """4x4 rigid transform that moves the median point to the origin and the
    principal axes of the points (largest variance first) onto x, y, z."""
    centroid = np.median(point_cloud, axis=0)
    cov = np.cov(point_cloud - centroid, rowvar=False)
    evals, evecs = np.linalg.eigh(cov)
    evecs = evecs[:, evals.argsort()[::-1]]
    if np.linalg.det(evecs) < 0:
        evecs[:, 0] *= -1
    rot = evecs.T
    transform = np.eye(4)
    transform[:3, :3] = rot
    transform[:3, 3] = -rot @ centroid
    return transform


def transform_points(matrix: np.ndarray, points: np.ndarray) -> np.ndarray:
    assert matrix.shape == (4, 4)
    assert len(points.shape) == 2 and points.shape[1] == 3
    return points @ matrix[:3, :3].T + matrix[:3, 3]


def transform_cameras(matrix: np.ndarray, camtoworlds: np.ndarray) -> np.ndarray:
    """Applies ``matrix`` to camera-to-world poses and removes its scale from
    the rotation part."""
    assert matrix.shape == (4, 4)
    assert len(camtoworlds.shape) == 3 and camtoworlds.shape[1:] == (4, 4)
    camtoworlds = np.einsum("nij, ki -> nkj", camtoworlds, matrix)
    scaling = np.linalg.norm(camtoworlds[:, 0, :3], axis=1)
    camtoworlds[:, :3, :3] = camtoworlds[:, :3, :3] / scaling[:, None, None]
    return camtoworlds


# ============================================================================ COLMAP binary model
# COLMAP camera models: id -> (name, number of parameters, single focal length)
CAMERA_MODELS: Dict[int, Tuple[str, int, bool]] = {
    0: ("SIMPLE_PINHOLE", 3, True),
    1: ("PINHOLE", 4, False),
    2: ("SIMPLE_RADIAL", 4, True),
    3: ("RADIAL", 5, True),
    4: ("OPENCV", 8, False),
    5: ("OPENCV_FISHEYE", 8, False),
    6: ("FULL_OPENCV", 12, False),
    7: ("FOV", 5, False),
    8: ("SIMPLE_RADIAL_FISHEYE", 4, True),
    9: ("RADIAL_FISHEYE", 5, True),
    10: ("THIN_PRISM_FISHEYE", 12, False),
}
CAMERA_MODEL_IDS = {name: mid for mid, (name, _, _) in CAMERA_MODELS.items()}


class Camera:
    """One COLMAP camera: ``camera_id, camera_type, width, height, params`` and
    the pinhole part ``fx, fy, cx, cy`` (distortion parameters are kept in
    ``params`` and not applied, as in the reference)."""

    def __init__(self, camera_id: int, camera_type: str, width: int, height: int, params):
        self.camera_id = camera_id
        self.camera_type = camera_type
        self.width = width
        self.height = height
        self.params = tuple(float(p) for p in params)
        single = CAMERA_MODELS[CAMERA_MODEL_IDS[camera_type]][2]
        p = self.params
        if single:
            self.fx = self.fy = p[0]
            self.cx, self.cy = p[1], p[2]
        else:
            self.fx, self.fy, self.cx, self.cy = p[0], p[1], p[2], p[3]


def qvec_to_rotmat(qvec: np.ndarray) -> np.ndarray:
    """Rotation matrix of a unit quaternion (w, x, y, z)."""
    w, x, y, z = qvec
    return np.array([
        [1 - 2 * y ** 2 - 2 * z ** 2, 2 * x * y - 2 * z * w, 2 * x * z + 2 * y * w],
        [2 * x * y + 2 * z * w, 1 - 2 * x ** 2 - 2 * z ** 2, 2 * y * z - 2 * x * w],
        [2 * x * z - 2 * y * w, 2 * y * z + 2 * x * w, 1 - 2 * x ** 2 - 2 * y ** 2],
    ])


class ColmapImage:
    """One registered image: ``image_id, qvec`` (normalised), ``tvec,
    camera_id, name`` and ``R()`` (world-to-camera rotation)."""

    def __init__(self, image_id: int, qvec: np.ndarray, tvec: np.ndarray, camera_id: int, name: str):
        self.image_id = image_id
        self.qvec = qvec
        self.tvec = tvec
        self.camera_id = camera_id
        self.name = name
        self._R = qvec_to_rotmat(qvec)

    def R(self) -> np.ndarray:
        return self._R


class _Reader:
    def __init__(self, path: str):
        with open(path, "rb") as f:
            self.buf = f.read()
        self.pos = 0

    def take(self, fmt: str):
        s = struct.Struct("<" + fmt)
        out = s.unpack_from(self.buf, self.pos)
        self.pos += s.size
        return out

    def cstring(self) -> str:
        end = self.buf.index(b"\x00", self.pos)
        name = self.buf[self.pos:end].decode("utf-8")
        self.pos = end + 1
        return name


def read_cameras_binary(path: str) -> Dict[int, Camera]:
    """``cameras.bin``: uint64 count; per camera int32 id, int32 model id,
    uint64 width, uint64 height, float64 params[model's count]."""
    r = _Reader(path)
    (n,) = r.take("Q")
    cams = {}
    for _ in range(n):
        cid, mid, w, h = r.take("iiQQ")
        if mid not in CAMERA_MODELS:
            raise ValueError(f"{path}: unknown COLMAP camera model id {mid}")
        name, npar, _ = CAMERA_MODELS[mid]
        params = r.take("d" * npar)
        cams[cid] = Camera(cid, name, w, h, params)
    return cams


def read_images_binary(path: str) -> Dict[int, ColmapImage]:
    """``images.bin``: uint64 count; per image int32 id, float64 qvec[4]
    (w, x, y, z), float64 tvec[3], int32 camera id, NUL-terminated name,
    uint64 number of 2-D points, then that many (float64 x, float64 y,
    int64 point id) records (skipped).  Insertion order = file order."""
    r = _Reader(path)
    (n,) = r.take("Q")
    images = {}
    for _ in range(n):
        iid, qw, qx, qy, qz, tx, ty, tz, cid = r.take("idddddddi")
        name = r.cstring()
        (npts,) = r.take("Q")
        r.pos += 24 * npts
        q = np.array([qw, qx, qy, qz])
        images[iid] = ColmapImage(iid, q / np.linalg.norm(q), np.array([tx, ty, tz]), cid, name)
    return images


def read_points3D_binary(path: str) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """``points3D.bin``: uint64 count; per point uint64 id, float64 xyz[3],
    uint8 rgb[3], float64 error, uint64 track length, then that many
    (int32 image id, int32 point2D index) pairs (skipped).  Returns
    ``(xyz float32 [n,3], rgb uint8 [n,3], error float32 [n])``."""
    r = _Reader(path)
    (n,) = r.take("Q")
    xyz = np.empty((n, 3), np.float64)
    rgb = np.empty((n, 3), np.uint8)
    err = np.empty(n, np.float64)
    rec = struct.Struct("<QdddBBBdQ")
    buf, pos = r.buf, r.pos
    for i in range(n):
        _, x, y, z, cr, cg, cb, e, tl = rec.unpack_from(buf, pos)
        xyz[i] = (x, y, z)
        rgb[i] = (cr, cg, cb)
        err[i] = e
        pos += rec.size + 8 * tl
    return xyz.astype(np.float32), rgb, err.astype(np.float32)


def write_cameras_binary(cameras: List[Camera], path: str) -> None:
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(cameras)))
        for c in cameras:
            mid = CAMERA_MODEL_IDS[c.camera_type]
            if len(c.params) != CAMERA_MODELS[mid][1]:
                raise ValueError(f"{c.camera_type} takes {CAMERA_MODELS[mid][1]} parameters")
            f.write(struct.pack("<iiQQ", c.camera_id, mid, c.width, c.height))
            f.write(struct.pack("<" + "d" * len(c.params), *c.params))


def write_images_binary(images: List[Tuple[int, np.ndarray, np.ndarray, int, str, np.ndarray]], path: str) -> None:
    """``images``: (image id, qvec, tvec, camera id, name, points2D [k, 3] as
    (x, y, point id)) per image."""
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(images)))
        for iid, q, t, cid, name, pts in images:
            f.write(struct.pack("<idddddddi", iid, *[float(v) for v in q], *[float(v) for v in t], cid))
            f.write(name.encode("utf-8") + b"\x00")
            pts = np.asarray(pts, np.float64).reshape(-1, 3)
            f.write(struct.pack("<Q", len(pts)))
            for x, y, pid in pts:
                f.write(struct.pack("<ddq", x, y, int(pid)))


def write_points3D_binary(xyz: np.ndarray, rgb: np.ndarray, err: np.ndarray, tracks: List[np.ndarray],
                          path: str) -> None:
    """``tracks[i]``: [k, 2] (image id, point2D index) pairs of point i."""
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(xyz)))
        for i in range(len(xyz)):
            tr = np.asarray(tracks[i], np.int64).reshape(-1, 2)
            f.write(struct.pack("<QdddBBBdQ", i + 1, *[float(v) for v in xyz[i]], *[int(v) for v in rgb[i]],
                                float(err[i]), len(tr)))
            for a, b in tr:
                f.write(struct.pack("<ii", int(a), int(b)))


# ============================================================================ images
def _rel_paths(d: str) -> List[str]:
    out = []
    for dp, _, fn in os.walk(d):
        for f in fn:
            out.append(os.path.relpath(os.path.join(dp, f), d))
    return out


def imread_rgb(path: str) -> np.ndarray:
    """HWC uint8 RGB (the first three channels of the decoded image)."""
    from PIL import Image
    with Image.open(path) as im:
        a = np.array(im)
    if a.ndim == 2:
        a = np.repeat(a[..., None], 3, 2)
    return np.ascontiguousarray(a[..., :3]).astype(np.uint8, copy=False)


def _resize_image_folder(image_dir: str, resized_dir: str, factor: int) -> str:
    """Downscales every image by ``factor`` (bicubic, rounded size) into PNGs
    (dataset.py:224-243); existing outputs are kept."""
    from PIL import Image
    os.makedirs(resized_dir, exist_ok=True)
    for rel in _rel_paths(image_dir):
        out = os.path.join(resized_dir, os.path.splitext(rel)[0] + ".png")
        if os.path.isfile(out):
            continue
        img = imread_rgb(os.path.join(image_dir, rel))
        size = (int(round(img.shape[1] / factor)), int(round(img.shape[0] / factor)))
        os.makedirs(os.path.dirname(out) or ".", exist_ok=True)
        Image.fromarray(img).resize(size, Image.BICUBIC).save(out)
    return resized_dir


# ============================================================================ parser / dataset
class Parser:
    """COLMAP scene (dataset.py:258-408): ``image_names`` (sorted),
    ``image_paths``, ``camtoworlds [n,4,4]``, ``camera_ids``, ``Ks_dict``,
    ``params_dict``, ``imsize_dict``, ``mask_dict``, ``points``,
    ``points_err``, ``points_rgb``, ``transform`` and ``scene_scale`` (largest
    camera distance from the cameras' mean position)."""

    def __init__(self, data_dir: str, factor: int = 1, normalize: bool = False, test_every: int = 8,
                 test_after: int = -1):
        self.data_dir = data_dir
        self.factor = factor
        self.normalize = normalize
        self.test_every = test_every
        self.test_after = test_after
        colmap_dir = os.path.join(data_dir, "sparse/0/")
        if not os.path.exists(colmap_dir):
            colmap_dir = os.path.join(data_dir, "sparse")
        if not os.path.exists(colmap_dir):
            raise FileNotFoundError(f"COLMAP sparse directory {colmap_dir} does not exist.")
        cams = read_cameras_binary(os.path.join(colmap_dir, "cameras.bin"))
        imgs = read_images_binary(os.path.join(colmap_dir, "images.bin"))
        points, points_rgb, points_err = read_points3D_binary(os.path.join(colmap_dir, "points3D.bin"))
        if len(imgs) == 0:
            raise ValueError("No images found in COLMAP sparse reconstruct.")

        bottom = np.array([0, 0, 0, 1]).reshape(1, 4)
        w2c, camera_ids = [], []
        self.Ks_dict, self.params_dict, self.imsize_dict, self.mask_dict = {}, {}, {}, {}
        for k in imgs:
            im = imgs[k]
            w2c.append(np.concatenate([np.concatenate([im.R(), im.tvec.reshape(3, 1)], 1), bottom], 0))
            camera_ids.append(im.camera_id)
            cam = cams[im.camera_id]
            K = np.array([[cam.fx, 0, cam.cx], [0, cam.fy, cam.cy], [0, 0, 1]])
            K[:2, :] /= factor
            self.Ks_dict[im.camera_id] = K
            self.params_dict[im.camera_id] = np.array(cam.params, dtype=np.float32)
            self.imsize_dict[im.camera_id] = (cam.width // factor, cam.height // factor)
            self.mask_dict[im.camera_id] = None
        camtoworlds = np.linalg.inv(np.stack(w2c, 0))
        names = [imgs[k].name for k in imgs]
        inds = np.argsort(names)
        image_names = [names[i] for i in inds]
        camtoworlds = camtoworlds[inds]
        camera_ids = [camera_ids[i] for i in inds]

        self.extconf = {"spiral_radius_scale": 1.0, "no_factor_suffix": False}
        suffix = f"_{factor}" if factor > 1 and not self.extconf["no_factor_suffix"] else ""
        colmap_image_dir = os.path.join(data_dir, "images")
        image_dir = os.path.join(data_dir, "images" + suffix)
        if not os.path.exists(colmap_image_dir):
            raise ValueError(f"Image folder {colmap_image_dir} does not exist.")
        colmap_files = sorted(_rel_paths(colmap_image_dir))
        image_files = list(colmap_files)
        if factor > 1 and os.path.splitext(image_files[0])[1].lower() == ".jpg":
            image_dir = _resize_image_folder(colmap_image_dir, image_dir + "_png", factor=factor)
            image_files = sorted(_rel_paths(image_dir))
        colmap_to_image = dict(zip(colmap_files, image_files))
        image_paths = [os.path.join(image_dir, colmap_to_image[f]) for f in image_names]

        if normalize:
            T1 = similarity_from_cameras(camtoworlds)
            camtoworlds = transform_cameras(T1, camtoworlds)
            points = transform_points(T1, points)
            T2 = align_principle_axes(points)
            camtoworlds = transform_cameras(T2, camtoworlds)
            points = transform_points(T2, points)
            transform = T2 @ T1
        else:
            transform = np.eye(4)

        self.image_names = image_names
        self.image_paths = image_paths
        self.camtoworlds = camtoworlds
        self.camera_ids = camera_ids
        self.points = points
        self.points_err = points_err
        self.points_rgb = points_rgb
        self.point_indices = {}
        self.transform = transform

        # intrinsics follow the size of the images actually on disk
        actual_h, actual_w = imread_rgb(self.image_paths[0]).shape[:2]
        colmap_w, colmap_h = self.imsize_dict[self.camera_ids[0]]
        s_h, s_w = actual_h / colmap_h, actual_w / colmap_w
        for cid, K in self.Ks_dict.items():
            K[0, :] *= s_w
            K[1, :] *= s_h
            w, h = self.imsize_dict[cid]
            self.imsize_dict[cid] = (int(w * s_w), int(h * s_h))

        locs = camtoworlds[:, :3, 3]
        self.scene_scale = np.max(np.linalg.norm(locs - np.mean(locs, axis=0), axis=1))


class Dataset:
    """Train or test split of a ``Parser`` (dataset.py:411-479): every
    ``test_every``-th image is a test image (or, with ``test_after``, the
    images after that index).  Items are ``{"K", "camtoworld", "image",
    "image_id"}`` with ``image`` float32 HWC in [0, 255] (torch, host), as
    the reference returns.  Preloaded images are kept as uint8 in pinned
    host memory; ``to_device`` keeps a copy of them in HBM and
    ``device_image`` returns the uint8 image of an item on the device (from
    the HBM copy, or uploaded from pinned memory on the current stream)."""

    def __init__(self, parser: Parser, split: str = "train", patch_size: Optional[int] = None,
                 preload_images: bool = True, seed: int = 0):
        self.parser = parser
        self.split = split
        self.patch_size = patch_size
        self.preload_images = preload_images
        self.rng = np.random.default_rng(seed)
        idx = np.arange(len(parser.image_names))
        if parser.test_every != -1:
            self.indices = idx[idx % parser.test_every != 0] if split == "train" else idx[idx % parser.test_every == 0]
        elif parser.test_after != -1:
            self.indices = idx[idx <= parser.test_after] if split == "train" else idx[idx > parser.test_after]
        else:
            self.indices = idx
        self.preloaded_images: Dict[int, torch.Tensor] = {}
        self._device_images: Dict[int, torch.Tensor] = {}
        self._stage: Dict[Tuple[torch.device, Tuple[int, ...]], torch.Tensor] = {}
        if preload_images:
            pin = torch.cuda.is_available()
            for i in self.indices:
                t = torch.from_numpy(imread_rgb(parser.image_paths[i]))
                self.preloaded_images[int(i)] = t.pin_memory() if pin else t

    def __len__(self) -> int:
        return len(self.indices)

    def image_u8(self, item: int) -> torch.Tensor:
        """Host uint8 HWC image of an item (pinned when preloaded)."""
        index = int(self.indices[item])
        if self.preload_images:
            return self.preloaded_images[index]
        return torch.from_numpy(imread_rgb(self.parser.image_paths[index]))

    def __getitem__(self, item: int) -> Dict[str, object]:
        index = int(self.indices[item])
        image = self.image_u8(item).to(torch.float32)
        K = self.parser.Ks_dict[self.parser.camera_ids[index]].copy()
        c2w = self.parser.camtoworlds[index]
        if self.patch_size is not None:
            h, w = image.shape[:2]
            x = int(self.rng.integers(0, max(w - self.patch_size, 1)))
            y = int(self.rng.integers(0, max(h - self.patch_size, 1)))
            image = image[y:y + self.patch_size, x:x + self.patch_size]
            K[0, 2] -= x
            K[1, 2] -= y
        return {"K": torch.from_numpy(K.astype(np.float32)), "camtoworld": torch.from_numpy(c2w.astype(np.float32)),
                "image": image, "image_id": item}

    def to_device(self, device) -> int:
        """Copies every preloaded image to ``device`` (uint8, 3 bytes per
        pixel); returns the bytes held."""
        if not self.preload_images:
            raise ValueError("to_device needs preload_images=True")
        total = 0
        for i, t in self.preloaded_images.items():
            self._device_images[i] = t.to(device, non_blocking=True)
            total += t.numel()
        return total

    def device_image(self, item: int, device) -> torch.Tensor:
        """uint8 HWC image of an item on ``device``: the HBM copy when
        ``to_device`` was called, otherwise an asynchronous upload from the
        pinned cache into a staging buffer on the current stream (the next
        upload of the same shape reuses the buffer after the work already
        queued on that stream)."""
        index = int(self.indices[item])
        if index in self._device_images:
            return self._device_images[index]
        src = self.image_u8(item)
        key = (torch.device(device), tuple(src.shape))
        st = self._stage.get(key)
        if st is None:
            st = self._stage[key] = torch.empty(src.shape, dtype=torch.uint8, device=device)
        st.copy_(src, non_blocking=True)
        return st
