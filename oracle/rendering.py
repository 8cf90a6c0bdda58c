"""CPU restatement of the reference rasterizer path — TEST INFRASTRUCTURE ONLY.

Follows ``mlx_gsplat/rendering.py`` line by line:

* ``cull``             — ``frustum_culling_mlx`` (rendering.py:41-94), NumPy float32
  with a fixed operation order (no fused multiply-add), so that the index
  decision is reproducible bit for bit.
* ``project``          — rendering.py:153-244 (camera transform, covariance,
  EWA projection, depth argsort, conic, sigmoid opacity, SH<=1 colour).
  ``sh_mode="full"`` extends the colour to real spherical harmonics of
  degree 2 and 3 (``sh_color_full``); the reference has no such mode, so this
  part is the library's own definition restated, checked against the
  reference mode at degree <= 1 and by autograd.
* ``rasterize_dense``  — rendering.py:246-308, the dense per-pixel compositing
  over *every* visible Gaussian in depth order (exclusive cumprod
  transmittance, weights, colour and alpha sums).  Differentiable through
  torch-CPU autograd; MLX's tie rules for ``clip``/``maximum`` gradients are
  kept by writing them as ``where`` with strict comparisons (MLX:
  ``maximum(a,b)`` sends the gradient to ``a`` only where ``a > b``).
* ``rasterize_dense_vjp`` — the same function's vector-Jacobian product,
  evaluated one pixel chunk at a time so that memory stays bounded (the
  per-Gaussian quantities are leaves for each chunk; their accumulated
  cotangents are pushed through ``project`` once at the end).  Pixel subsets
  are supported: the image is evaluated only at the listed pixels and the
  cotangent is taken as zero elsewhere.

Known differences from MLX itself: argsort tie order (stable here), the
last-ulp behaviour of transcendental functions and of matmul summation order.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import numpy as np
import torch

SH_C0 = 0.28209479177387814
SH_C1 = 0.4886025119029199


def _sh_hi_basis(x, y, z, deg):
    """Real SH basis of degrees 2 (and 3) at unit direction components
    (x, y, z), normalisation constants computed from their closed forms."""
    pi = np.pi
    k0, k1, k2 = 0.5 * np.sqrt(15 / pi), 0.25 * np.sqrt(5 / pi), 0.25 * np.sqrt(15 / pi)
    xx, yy, zz = x * x, y * y, z * z
    out = [k0 * x * y, -k0 * y * z, k1 * (2 * zz - xx - yy), -k0 * x * z, k2 * (xx - yy)]
    if deg >= 3:
        k3, k4 = 0.25 * np.sqrt(35 / (2 * pi)), 0.5 * np.sqrt(105 / pi)
        k5, k6, k7 = 0.25 * np.sqrt(21 / (2 * pi)), 0.25 * np.sqrt(7 / pi), 0.25 * np.sqrt(105 / pi)
        out += [-k3 * y * (3 * xx - yy), k4 * x * y * z, -k5 * y * (4 * zz - xx - yy),
                k6 * z * (2 * zz - 3 * xx - 3 * yy), -k5 * x * (4 * zz - xx - yy), k7 * z * (xx - yy),
                -k3 * x * (xx - 3 * yy)]
    return out


def sh_full_degree(ncols: int) -> int:
    """Degree held by ``ncols`` colour floats in the full mode (3 (d+1)^2, d <= 3)."""
    return 3 if ncols >= 48 else 2 if ncols >= 27 else 1 if ncols >= 12 else 0


def sh_color_full(cs, dirs):
    """RGB before the +0.5 / clip of the full SH mode: channel ch's
    coefficients are ``cs[:, 3 + k*ch : 3 + k*(ch+1)]`` with k = (d+1)^2 - 1;
    the first three multiply (y, z, x) with the reference's degree-1 constant
    and sign (rendering.py:232-242), then the degree-2 and -3 basis."""
    d = sh_full_degree(cs.shape[1])
    rgb = cs[:, :3] * SH_C0
    if d == 0:
        return rgb
    k = (d + 1) ** 2 - 1
    x, y, z = dirs[:, 0], dirs[:, 1], dirs[:, 2]
    hi = _sh_hi_basis(x, y, z, d) if d >= 2 else []
    chans = []
    for ch in range(3):
        c0 = 3 + k * ch
        # the degree-1 term exactly as rendering.py:237-241 forms it
        acc = SH_C1 * (cs[:, c0] * y + cs[:, c0 + 1] * z + cs[:, c0 + 2] * x)
        for j, b in enumerate(hi):
            acc = acc + cs[:, c0 + 3 + j] * b
        chans.append(acc)
    return rgb + torch.stack(chans, 1)


# ----------------------------------------------------------------------------- cull
def cull(means: np.ndarray, opacities: Optional[np.ndarray], viewmat: np.ndarray, K: np.ndarray,
         width: int, height: int, near_plane: float = 0.01, far_plane: float = 1e10,
         opacity_threshold: float = -5.3, empty_quirk: bool = False) -> np.ndarray:
    """``frustum_culling_mlx`` (rendering.py:41-94).  Returns ascending int32 ids.

    The camera-space point is ``[x,y,z,1] @ viewmat.T`` summed left to right
    (``((x*v[i,0] + y*v[i,1]) + z*v[i,2]) + v[i,3]``) in float32 with every
    product and sum rounded separately.  ``empty_quirk=True`` reproduces the
    reference's ``sorted_indices[-0:]`` behaviour when nothing is visible
    (it returns all N entries, every one ``-1``); the default returns an empty
    array.
    """
    f32 = np.float32
    m = np.asarray(means, f32)
    v = np.asarray(viewmat, f32)
    x, y, z = m[:, 0], m[:, 1], m[:, 2]

    def row(i):
        return ((x * v[i, 0] + y * v[i, 1]) + z * v[i, 2]) + v[i, 3]

    cx_, cy_, cz_ = row(0), row(1), row(2)
    Kf = np.asarray(K, f32)
    fx, fy, cx, cy = Kf[0, 0], Kf[1, 1], Kf[0, 2], Kf[1, 2]
    near = f32(near_plane)
    far = f32(far_plane)
    dsafe = np.where(cz_ > near, cz_, near).astype(f32)
    x2d = (cx_ * fx) / dsafe + cx
    y2d = (cy_ * fy) / dsafe + cy
    tol = f32(50.0)
    valid = ((cz_ > near) & (cz_ < far) & (x2d + tol >= 0) & (x2d - tol < f32(width))
             & (y2d + tol >= 0) & (y2d - tol < f32(height)))
    if opacities is not None:
        valid &= np.asarray(opacities, f32).reshape(-1) >= f32(opacity_threshold)
    ids = np.nonzero(valid)[0].astype(np.int32)
    if ids.size == 0 and empty_quirk:
        return np.full(m.shape[0], -1, np.int32)
    return ids


def depth_order_f32(means: np.ndarray, viewmat: np.ndarray) -> np.ndarray:
    """The depth order a float32 renderer gets: camera z as in ``cull``
    (float32, left to right, every product and sum rounded), stable argsort
    (ties by input position).  Rasterizers that rank depths in float64 can
    order nearly equal depths differently."""
    f32 = np.float32
    m = np.asarray(means, f32)
    v = np.asarray(viewmat, f32)
    z = ((m[:, 0] * v[2, 0] + m[:, 1] * v[2, 1]) + m[:, 2] * v[2, 2]) + v[2, 3]
    return np.argsort(z, kind="stable")


# ----------------------------------------------------------------------------- projection
def _gt(x, c):
    """MLX ``maximum(x, c)`` with its gradient rule (to ``x`` only where ``x > c``)."""
    return torch.where(x > c, x, torch.full_like(x, c))


def _clip(x, lo, hi):
    """MLX ``clip`` = ``minimum(maximum(x, lo), hi)`` with strict-comparison gradients."""
    y = torch.where(x > lo, x, torch.full_like(x, lo))
    return torch.where(y < hi, y, torch.full_like(y, hi))


def project(means, quats, scales, opacities, colors, viewmat, K, width, height,
            render_width, render_height, sh_mode: str = "reference") -> Dict[str, torch.Tensor]:
    """rendering.py:153-244 on already-gathered active rows (all torch, one dtype).

    Returns per-Gaussian quantities in **depth order**: ``u, v, a, b, c, d``
    (conic), ``opac`` (sigmoid), ``rgb [V,3]`` and ``order`` (the argsort).
    """
    dt = means.dtype
    V = means.shape[0]
    vm = viewmat.to(dt)
    Kt = K.to(dt)
    ones = torch.ones((V, 1), dtype=dt)
    means_cam = torch.cat([means, ones], 1) @ vm.T
    means_cam = means_cam[:, :3]
    depths = means_cam[:, 2]
    fx, fy, cx, cy = Kt[0, 0], Kt[1, 1], Kt[0, 2], Kt[1, 2]
    dsafe = _gt(depths, 1e-4)
    x2d = (means_cam[:, 0] * fx) / dsafe + cx
    y2d = (means_cam[:, 1] * fy) / dsafe + cy

    qn = torch.sqrt(torch.sum(quats ** 2, 1, keepdim=True) + 1e-8)
    q = quats / qn
    r, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    R = torch.stack([
        torch.stack([1.0 - 2.0 * (y ** 2 + z ** 2), 2.0 * (x * y - r * z), 2.0 * (x * z + r * y)], -1),
        torch.stack([2.0 * (x * y + r * z), 1.0 - 2.0 * (x ** 2 + z ** 2), 2.0 * (y * z - r * x)], -1),
        torch.stack([2.0 * (x * z - r * y), 2.0 * (y * z + r * x), 1.0 - 2.0 * (x ** 2 + y ** 2)], -1),
    ], -2)
    S = torch.exp(scales)
    RS = R * S[:, None, :]                      # R @ diag(S)
    Sigma3 = RS @ RS.transpose(1, 2)

    tx, ty, tz = means_cam[:, 0], means_cam[:, 1], dsafe
    tz2 = tz ** 2
    zero = torch.zeros_like(tz)
    J = torch.stack([
        torch.stack([fx / tz, zero, -fx * tx / tz2], -1),
        torch.stack([zero, fy / tz, -fy * ty / tz2], -1),
        torch.zeros((V, 3), dtype=dt),
    ], -2)
    W = vm[:3, :3]
    JW = J @ W
    Sigma2 = (JW @ (Sigma3 @ JW.transpose(1, 2)))[:, :2, :2]
    Sigma2 = Sigma2 + torch.tensor([[0.3, 0.0], [0.0, 0.3]], dtype=dt)

    order = torch.argsort(depths.detach(), stable=True)
    S2 = Sigma2[order]
    det = S2[:, 0, 0] * S2[:, 1, 1] - S2[:, 0, 1] * S2[:, 1, 0]
    det = _gt(det, 1e-6)
    a = S2[:, 1, 1] / det
    b = -S2[:, 0, 1] / det
    c = -S2[:, 1, 0] / det
    d = S2[:, 0, 0] / det
    opac = torch.sigmoid(opacities[order]).reshape(-1)

    R_w2c = vm[:3, :3]
    T_w2c = vm[:3, 3]
    cam_pos = -(R_w2c.T @ T_w2c)
    dirs = means[order] - cam_pos[None, :]
    dirs = dirs / (torch.sqrt(torch.sum(dirs ** 2, -1, keepdim=True)) + 1e-8)
    cs = colors[order]
    rgb = cs[:, :3] * SH_C0
    if sh_mode == "full":
        rgb = sh_color_full(cs, dirs)
    elif cs.shape[1] >= 12:
        xd, yd, zd = dirs[:, 0], dirs[:, 1], dirs[:, 2]
        rgb = rgb + SH_C1 * torch.stack([
            cs[:, 3] * yd + cs[:, 4] * zd + cs[:, 5] * xd,
            cs[:, 6] * yd + cs[:, 7] * zd + cs[:, 8] * xd,
            cs[:, 9] * yd + cs[:, 10] * zd + cs[:, 11] * xd,
        ], 1)
    rgb = _clip(rgb + 0.5, 0.0, 1.0)
    return {"u": x2d[order], "v": y2d[order], "a": a, "b": b, "c": c, "d": d,
            "opac": opac, "rgb": rgb, "order": order, "depths": depths}


def pixel_centers(width, height, render_width, render_height, dtype) -> torch.Tensor:
    """rendering.py:246-256: centres ``i*sx + sx/2`` (float32 grid as in MLX)."""
    xs = torch.arange(render_width, dtype=torch.float32)
    ys = torch.arange(render_height, dtype=torch.float32)
    gx, gy = torch.meshgrid(xs, ys, indexing="xy")
    sx = float(width) / float(render_width)
    sy = float(height) / float(render_height)
    px = gx * sx + (sx * 0.5)
    py = gy * sy + (sy * 0.5)
    return torch.stack([px, py], -1).reshape(-1, 2).to(dtype)


def composite(pg: Dict[str, torch.Tensor], pix: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """rendering.py:274-300 for one chunk of pixels ``pix [P,2]``.  ``pg["mask"]``
    (optional, depth order) multiplies the clipped alphas (:289-290)."""
    xv = pix[:, None, 0] - pg["u"][None, :]
    yv = pix[:, None, 1] - pg["v"][None, :]
    isx = pg["a"][None, :] * xv + pg["b"][None, :] * yv
    isy = pg["c"][None, :] * xv + pg["d"][None, :] * yv
    mah = xv * isx + yv * isy
    g = torch.exp(-0.5 * mah)
    alpha = _clip(pg["opac"][None, :] * g, 0.0, 0.99)
    if pg.get("mask") is not None:
        alpha = alpha * pg["mask"][None, :]
    trans = torch.cumprod(1.0 - alpha, 1)
    T = torch.cat([torch.ones((pix.shape[0], 1), dtype=alpha.dtype), trans[:, :-1]], 1)
    w = alpha * T
    return w @ pg["rgb"], torch.sum(w, 1, keepdim=True)


def _sorted_mask(mask, mask_order, pg_order, dtype):
    """The alpha mask in this projection's depth order.  ``mask[j]`` belongs to
    the j-th Gaussian of ``mask_order`` (default: this projection's own depth
    order, the reference's rule)."""
    if mask is None:
        return None
    mk = _as_t(mask, dtype).reshape(-1)
    if mask_order is None:
        return mk
    by_gaussian = torch.zeros_like(mk)
    by_gaussian[torch.as_tensor(np.asarray(mask_order, np.int64))] = mk
    return by_gaussian[pg_order]


def _as_t(x, dtype):
    if isinstance(x, torch.Tensor):
        return x.detach().to(dtype)
    return torch.as_tensor(np.asarray(x)).to(dtype)


def rasterize_dense(means, quats, scales, opacities, colors, viewmat, K, width, height,
                    render_width, render_height, dtype=torch.float64, chunk: int = 512,
                    pixel_ids: Optional[np.ndarray] = None, sh_mode: str = "reference", mask=None,
                    mask_order=None):
    """Forward only.  Inputs are the gathered active rows (numpy or torch);
    ``mask`` [V] multiplies the clipped alpha of the j-th Gaussian in depth order
    (of ``mask_order`` when given, e.g. ``depth_order_f32``).
    Returns ``(colors [H,W,3], alphas [H,W,1])`` as numpy arrays, or
    ``[P,3], [P,1]`` when ``pixel_ids`` selects a subset."""
    with torch.no_grad():
        args = [_as_t(a, dtype) for a in (means, quats, scales, opacities, colors)]
        pg = project(*args, _as_t(viewmat, dtype), _as_t(K, dtype), width, height,
                     render_width, render_height, sh_mode=sh_mode)
        pg["mask"] = _sorted_mask(mask, mask_order, pg["order"], dtype)
        pix = pixel_centers(width, height, render_width, render_height, dtype)
        if pixel_ids is not None:
            pix = pix[torch.as_tensor(np.asarray(pixel_ids, np.int64))]
        P = pix.shape[0]
        if means.shape[0] == 0:
            outc = torch.zeros((P, 3), dtype=dtype)
            outa = torch.zeros((P, 1), dtype=dtype)
        else:
            cs, as_ = [], []
            for s in range(0, P, chunk):
                c_, a_ = composite(pg, pix[s:s + chunk])
                cs.append(c_)
                as_.append(a_)
            outc, outa = torch.cat(cs), torch.cat(as_)
    if pixel_ids is None:
        return (outc.reshape(render_height, render_width, 3).numpy(),
                outa.reshape(render_height, render_width, 1).numpy())
    return outc.numpy(), outa.numpy()


def rasterize_dense_vjp(means, quats, scales, opacities, colors, viewmat, K, width, height,
                        render_width, render_height, dL_dC, dL_dA=None, dtype=torch.float64,
                        chunk: int = 256, pixel_ids: Optional[np.ndarray] = None, sh_mode: str = "reference",
                        l1_target=None, mask=None, mask_order=None):
    """Forward plus vector-Jacobian product of the dense rasterizer.

    ``dL_dC``/``dL_dA`` are ``[H,W,3]``/``[H,W,1]`` (or ``[P,3]``/``[P,1]`` for
    a pixel subset).  Returns ``(C, A, grads)`` with ``grads`` keyed
    ``means, quats, scales, opacities, colors`` on the gathered rows.
    With ``l1_target`` ([H,W,3]) the loss is instead the trainer's
    ``mean(|C - target|)`` (trainer.py:273-275, over all 3 H W values), whose
    gradient is formed chunk by chunk in the same single pass (``dL_dC`` is
    ignored).  ``mask`` as in ``rasterize_dense`` (no gradient flows to it).
    """
    leaves = [_as_t(a, dtype).requires_grad_(True) for a in (means, quats, scales, opacities, colors)]
    pg = project(*leaves, _as_t(viewmat, dtype), _as_t(K, dtype), width, height,
                 render_width, render_height, sh_mode=sh_mode)
    keys = ["u", "v", "a", "b", "c", "d", "opac", "rgb"]
    det = {k: pg[k].detach().clone().requires_grad_(True) for k in keys}
    det["mask"] = _sorted_mask(mask, mask_order, pg["order"], dtype)
    acc = {k: torch.zeros_like(det[k]) for k in keys}
    pix = pixel_centers(width, height, render_width, render_height, dtype)
    if pixel_ids is not None:
        pix = pix[torch.as_tensor(np.asarray(pixel_ids, np.int64))]
    P = pix.shape[0]
    tgt = None if l1_target is None else _as_t(l1_target, dtype).reshape(P, 3)
    gC = None if tgt is not None else _as_t(dL_dC, dtype).reshape(P, 3)
    gA = None if dL_dA is None else _as_t(dL_dA, dtype).reshape(P, 1)
    cs, as_ = [], []
    for s in range(0, P, chunk):
        for k in keys:
            det[k].grad = None
        c_, a_ = composite(det, pix[s:s + chunk])
        if tgt is not None:
            loss = torch.sum(torch.abs(c_ - tgt[s:s + chunk])) / (3 * P)
        else:
            loss = torch.sum(c_ * gC[s:s + chunk])
        if gA is not None:
            loss = loss + torch.sum(a_ * gA[s:s + chunk])
        gs = torch.autograd.grad(loss, [det[k] for k in keys], allow_unused=True)
        for k, g in zip(keys, gs):
            if g is not None:
                acc[k] += g
        cs.append(c_.detach())
        as_.append(a_.detach())
    outs = [pg[k] for k in keys]
    grads = torch.autograd.grad(outs, leaves, grad_outputs=[acc[k] for k in keys], allow_unused=True)
    names = ["means", "quats", "scales", "opacities", "colors"]
    gd = {n: (torch.zeros_like(l) if g is None else g).detach().numpy() for n, g, l in zip(names, grads, leaves)}
    C = torch.cat(cs).numpy()
    A = torch.cat(as_).numpy()
    if pixel_ids is None:
        C = C.reshape(render_height, render_width, 3)
        A = A.reshape(render_height, render_width, 1)
    return C, A, gd


def rasterize_gaussians(means, quats, scales, opacities, colors, viewmat, K, width, height,
                        active_indices, render_width, render_height, dtype=torch.float64):
    """The reference entry's gather rule (rendering.py:121-146): rows of the four
    geometry inputs are taken at ``active_indices``; ``colors`` is used as is
    when it already has one row per visible Gaussian, otherwise gathered too."""
    ids = np.asarray(active_indices, np.int64)
    cols = np.asarray(colors)
    cols = cols if cols.shape[0] == ids.shape[0] else cols[ids]
    return rasterize_dense(np.asarray(means)[ids], np.asarray(quats)[ids], np.asarray(scales)[ids],
                           np.asarray(opacities)[ids], cols, viewmat, K, width, height,
                           render_width, render_height, dtype=dtype)
