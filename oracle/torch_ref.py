"""CPU ORACLE — TEST INFRASTRUCTURE ONLY (autograd restatements).

Differentiable torch restatements of the reference's pure-MLX pieces, used to
check the hand-derived sm_100a backward kernels against automatic
differentiation (the reference gets these gradients from MLX autodiff):

* ``project``     — src/mlx3d/splatting/projection.py:24-146
* ``eval_sh``     — src/mlx3d/splatting/sh.py:41-78
* ``view_dirs``   — src/mlx3d/splatting/render.py:77-78
* ``naive_render``— src/mlx3d/splatting/reference.py:16-74, the reference's own
  O(N*H*W) test oracle (small scenes only).
* ``ssim`` / ``l1_dssim``   — src/mlx3d/losses/image_metrics.py:23-85 and the
  trainer's loss, trainer.py:300-305 (depthwise conv2d, zero padding).
* ``adam_update`` — mlx.optimizers.Adam.apply_single as the trainer builds it
  (trainer.py:128), float32 numpy, one rounding per operation.
* ``geometry_loss_2dgs`` — the 2DGS geometry terms, trainer.py:186-259, on the
  naive renderer's feature composite (cameras.py:327-336 for the unprojection,
  pinhole cameras).

The product package never imports this module.
"""

from __future__ import annotations

import torch

SH_C0 = 0.28209479177387814
SH_C1 = 0.4886025119029199
SH_C2 = (1.0925484305920792, -1.0925484305920792, 0.31539156525252005, -1.0925484305920792, 0.5462742152960396)
SH_C3 = (-0.5900435899266435, 2.890611442640554, -0.4570457994644658, 0.3731763325901154, -0.4570457994644658,
         1.445305721320277, -0.5900435899266435)


def project(camera, means, quats, scales, blur=0.3, antialias=False):
    dt = means.dtype
    R = camera.R.to(dt)
    t = camera.t.to(dt)
    mx_, my_, mz_ = means[:, 0], means[:, 1], means[:, 2]
    x = mx_ * R[0, 0] + my_ * R[0, 1] + mz_ * R[0, 2] + t[0]
    y = mx_ * R[1, 0] + my_ * R[1, 1] + mz_ * R[1, 2] + t[1]
    z = mx_ * R[2, 0] + my_ * R[2, 1] + mz_ * R[2, 2] + t[2]
    z_safe = torch.clamp(z, min=1e-6)
    u = camera.fx * x / z_safe + camera.cx
    v = camera.fy * y / z_safe + camera.cy
    tan_fov_x = 0.5 * camera.width / camera.fx
    tan_fov_y = 0.5 * camera.height / camera.fy
    tx = torch.clamp(x / z_safe, -1.3 * tan_fov_x, 1.3 * tan_fov_x) * z_safe
    ty = torch.clamp(y / z_safe, -1.3 * tan_fov_y, 1.3 * tan_fov_y) * z_safe
    inv_z = 1.0 / z_safe
    inv_z2 = inv_z * inv_z
    j00 = camera.fx * inv_z
    j02 = -camera.fx * tx * inv_z2
    j11 = camera.fy * inv_z
    j12 = -camera.fy * ty * inv_z2
    t00 = j00 * R[0, 0] + j02 * R[2, 0]
    t01 = j00 * R[0, 1] + j02 * R[2, 1]
    t02 = j00 * R[0, 2] + j02 * R[2, 2]
    t10 = j11 * R[1, 0] + j12 * R[2, 0]
    t11 = j11 * R[1, 1] + j12 * R[2, 1]
    t12 = j11 * R[1, 2] + j12 * R[2, 2]
    q = quats / torch.linalg.norm(quats, dim=-1, keepdim=True)
    qw, qx, qy, qz = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    r00 = 1.0 - 2.0 * (qy * qy + qz * qz)
    r01 = 2.0 * (qx * qy - qw * qz)
    r02 = 2.0 * (qx * qz + qw * qy)
    r10 = 2.0 * (qx * qy + qw * qz)
    r11 = 1.0 - 2.0 * (qx * qx + qz * qz)
    r12 = 2.0 * (qy * qz - qw * qx)
    r20 = 2.0 * (qx * qz - qw * qy)
    r21 = 2.0 * (qy * qz + qw * qx)
    r22 = 1.0 - 2.0 * (qx * qx + qy * qy)
    sx, sy, sz = scales[:, 0], scales[:, 1], scales[:, 2]
    m00 = (t00 * r00 + t01 * r10 + t02 * r20) * sx
    m01 = (t00 * r01 + t01 * r11 + t02 * r21) * sy
    m02 = (t00 * r02 + t01 * r12 + t02 * r22) * sz
    m10 = (t10 * r00 + t11 * r10 + t12 * r20) * sx
    m11 = (t10 * r01 + t11 * r11 + t12 * r21) * sy
    m12 = (t10 * r02 + t11 * r12 + t12 * r22) * sz
    a0 = m00 * m00 + m01 * m01 + m02 * m02
    b = m00 * m10 + m01 * m11 + m02 * m12
    c0 = m10 * m10 + m11 * m11 + m12 * m12
    a = a0 + blur
    c = c0 + blur
    det = a * c - b * b
    det_safe = torch.clamp(det, min=1e-12)
    conics = torch.stack([c / det_safe, -b / det_safe, a / det_safe], dim=-1)
    if antialias and blur > 0:
        det0 = torch.clamp(a0 * c0 - b * b, min=0.0)
        comp = torch.sqrt(det0 / det_safe)
    else:
        comp = torch.ones_like(det)
    mid = 0.5 * (a + c)
    lam1 = mid + torch.sqrt(torch.clamp(mid * mid - det, min=0.01))
    radii = torch.ceil(3.0 * torch.sqrt(torch.clamp(lam1, min=0.0)))
    valid = (z > camera.znear) & (det > 0)
    radii = torch.where(valid, radii, torch.zeros_like(radii)).detach()
    comp = torch.where(valid, comp, torch.zeros_like(comp))
    return {"means2d": torch.stack([u, v], dim=-1), "conics": conics, "depths": z, "radii": radii,
            "compensation": comp}


def eval_sh(degree, sh, dirs):
    result = SH_C0 * sh[:, 0]
    if degree > 0:
        x, y, z = dirs[:, 0:1], dirs[:, 1:2], dirs[:, 2:3]
        result = result - SH_C1 * y * sh[:, 1] + SH_C1 * z * sh[:, 2] - SH_C1 * x * sh[:, 3]
        if degree > 1:
            xx, yy, zz = x * x, y * y, z * z
            xy, yz, xz = x * y, y * z, x * z
            result = (result + SH_C2[0] * xy * sh[:, 4] + SH_C2[1] * yz * sh[:, 5]
                      + SH_C2[2] * (2.0 * zz - xx - yy) * sh[:, 6] + SH_C2[3] * xz * sh[:, 7]
                      + SH_C2[4] * (xx - yy) * sh[:, 8])
            if degree > 2:
                result = (result + SH_C3[0] * y * (3.0 * xx - yy) * sh[:, 9] + SH_C3[1] * xy * z * sh[:, 10]
                          + SH_C3[2] * y * (4.0 * zz - xx - yy) * sh[:, 11]
                          + SH_C3[3] * z * (2.0 * zz - 3.0 * xx - 3.0 * yy) * sh[:, 12]
                          + SH_C3[4] * x * (4.0 * zz - xx - yy) * sh[:, 13] + SH_C3[5] * z * (xx - yy) * sh[:, 14]
                          + SH_C3[6] * x * (xx - 3.0 * yy) * sh[:, 15])
    return result + 0.5


def view_dirs(camera, means):
    center = (-(camera.R.T.to(torch.float32) @ camera.t.to(torch.float32))).to(means.dtype)
    d = means - center
    return d / torch.clamp(torch.linalg.norm(d, dim=-1, keepdim=True), min=1e-8)


def naive_render(camera, means, quats, scales, opacities, colors, background=None, antialias=False):
    """reference.py:16-74: every Gaussian at every pixel, global depth order
    (``colors`` may have any number C of channels; background (C,))."""
    dt = means.dtype
    if background is None:
        background = torch.zeros(colors.shape[1], dtype=dt)
    H, W = camera.height, camera.width
    proj = project(camera, means, quats, scales, antialias=antialias)
    order = torch.argsort(proj["depths"].detach(), stable=True)
    means2d = proj["means2d"][order]
    conics = proj["conics"][order]
    colors = colors[order]
    opac = (opacities * proj["compensation"])[order]
    radii = proj["radii"][order]
    xs = torch.arange(W, dtype=dt) + 0.5
    ys = torch.arange(H, dtype=dt) + 0.5
    px = xs[None, :].expand(H, W)
    py = ys[:, None].expand(H, W)
    dx = means2d[:, 0][:, None, None] - px[None]
    dy = means2d[:, 1][:, None, None] - py[None]
    a = conics[:, 0][:, None, None]
    b = conics[:, 1][:, None, None]
    c = conics[:, 2][:, None, None]
    power = -0.5 * (a * dx * dx + c * dy * dy) - b * dx * dy
    alpha = torch.clamp(opac[:, None, None] * torch.exp(power), max=0.99)
    alpha = torch.where(power > 0.0, torch.zeros_like(alpha), alpha)
    alpha = torch.where(alpha < 1.0 / 255.0, torch.zeros_like(alpha), alpha)
    alpha = alpha * (radii > 0)[:, None, None]
    one_minus = 1.0 - alpha
    trans = torch.cumprod(one_minus, dim=0)
    trans = torch.cat([torch.ones_like(trans[:1]), trans[:-1]], dim=0)
    keep = trans > 1e-4
    weights = alpha * trans * keep
    image = torch.sum(weights[..., None] * colors[:, None, None, :], dim=0)
    final_T = torch.prod(torch.where(keep, one_minus, torch.ones_like(one_minus)), dim=0)
    image = image + final_T[..., None] * background
    return {"image": image, "alpha": 1.0 - final_T, "final_T": final_T}


def ssim(pred, target, max_val=1.0, window_size=11, sigma=1.5):
    """image_metrics.py:29-85 for (H, W, C) images."""
    dt = pred.dtype
    x = torch.arange(window_size, dtype=torch.float32) - (window_size - 1) / 2.0
    g = torch.exp(-(x * x) / (2.0 * sigma * sigma))
    g = (g / g.sum()).to(dt)
    win = g[:, None] * g[None, :]
    C = pred.shape[-1]
    w = win[None, None].expand(C, 1, window_size, window_size)
    p = pred.permute(2, 0, 1)[None]
    t = target.permute(2, 0, 1)[None]
    filt = lambda a: torch.nn.functional.conv2d(a, w, padding=window_size // 2, groups=C)  # noqa: E731
    mu_p, mu_t = filt(p), filt(t)
    sp = filt(p * p) - mu_p * mu_p
    st = filt(t * t) - mu_t * mu_t
    spt = filt(p * t) - mu_p * mu_t
    c1, c2 = (0.01 * max_val) ** 2, (0.03 * max_val) ** 2
    cs = (2.0 * spt + c2) / (sp + st + c2)
    return ((2.0 * mu_p * mu_t + c1) / (mu_p * mu_p + mu_t * mu_t + c1) * cs).mean()


def l1_dssim(pred, target, lam=0.2):
    return (1.0 - lam) * (pred - target).abs().mean() + lam * (1.0 - ssim(pred, target))


def adam_update(p, g, m, v, lr, b1=0.9, b2=0.999, eps=1e-15):
    """One update in float32 numpy (arrays updated and returned)."""
    import numpy as np

    f = np.float32
    m = f(b1) * m + f(1.0 - b1) * g
    v = f(b2) * v + f(1.0 - b2) * (g * g)
    p = p - (f(lr) * m) / (np.sqrt(v) + f(eps))
    return p.astype(np.float32), m.astype(np.float32), v.astype(np.float32)


def project_points(camera, pts, eps=1e-8):
    """Camera.project_points (cameras.py:290-317, distortion :42-76)."""
    R, t = camera.R.to(pts.dtype), camera.t.to(pts.dtype)
    pc = pts @ R.T + t
    z = pc[..., 2]
    if camera.orthographic:
        return torch.stack([camera.fx * pc[..., 0] + camera.cx, camera.fy * pc[..., 1] + camera.cy], -1)
    inv = 1.0 / torch.where(z.abs() < eps, torch.full_like(z, eps), z)
    x, y = pc[..., 0] * inv, pc[..., 1] * inv
    d = camera.distortion
    if d is not None and not camera.fisheye:
        k1, k2, p1, p2 = d[0], d[1], d[2], d[3]
        k3 = d[4] if len(d) > 4 else 0.0
        r2 = x * x + y * y
        radial = 1.0 + r2 * (k1 + r2 * (k2 + r2 * k3))
        x, y = (x * radial + 2.0 * p1 * x * y + p2 * (r2 + 2.0 * x * x),
                y * radial + p1 * (r2 + 2.0 * y * y) + 2.0 * p2 * x * y)
    elif d is not None:
        k1, k2, k3, k4 = (list(d) + [0.0] * 4)[:4]
        r = torch.sqrt(x * x + y * y)
        th = torch.atan(r)
        th2 = th * th
        thd = th * (1.0 + th2 * (k1 + th2 * (k2 + th2 * (k3 + th2 * k4))))
        sc = thd / torch.clamp(r, min=1e-9)
        x, y = x * sc, y * sc
    return torch.stack([camera.fx * x + camera.cx, camera.fy * y + camera.cy], -1)


def project_ut(camera, means, quats, scales, blur=0.3, antialias=False):
    """project_gaussians_ut (projection.py:149-205)."""
    q = quats / torch.linalg.norm(quats, dim=-1, keepdim=True)
    w, x, y, z = q.unbind(-1)
    R = torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
                     2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
                     2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1).reshape(-1, 3, 3)
    sqrt_cov = R * scales[:, None, :]
    offsets = torch.cat([sqrt_cov.transpose(1, 2), -sqrt_cov.transpose(1, 2)], dim=1)
    sigma = means[:, None, :] + 3.0 ** 0.5 * offsets
    xy = project_points(camera, sigma.reshape(-1, 3)).reshape(means.shape[0], 6, 2)
    m2 = xy.mean(dim=1)
    d = xy - m2[:, None, :]
    a0 = (d[..., 0] * d[..., 0]).mean(1)
    b = (d[..., 0] * d[..., 1]).mean(1)
    c0 = (d[..., 1] * d[..., 1]).mean(1)
    a, c = a0 + blur, c0 + blur
    det = a * c - b * b
    ds = torch.clamp(det, min=1e-12)
    conics = torch.stack([c / ds, -b / ds, a / ds], -1)
    comp = torch.sqrt(torch.clamp(a0 * c0 - b * b, min=0.0) / ds) if (antialias and blur > 0) else torch.ones_like(det)
    mid = 0.5 * (a + c)
    radii = torch.ceil(3.0 * torch.sqrt(torch.clamp(mid + torch.sqrt(torch.clamp(mid * mid - det, min=0.01)), min=0)))
    zc = (means @ camera.R.to(means.dtype).T + camera.t.to(means.dtype))[:, 2]
    valid = (zc > camera.znear) & (det > 0)
    return {"means2d": m2, "conics": conics, "depths": zc, "radii": torch.where(valid, radii, 0 * radii).detach(),
            "compensation": torch.where(valid, comp, 0 * comp)}


def geometry_loss_2dgs(camera, means, quats, scales, opacities, antialias=False, lam_var=0.0, lam_normal=0.0,
                       min_alpha=0.05):
    """(loss, depth_variance, normal_consistency) of trainer.py:186-259 with
    ``opacities`` activated; features [z, z^2, normal] composited by the naive
    renderer and normalised by alpha (rasterize.py:535-544)."""
    dt = means.dtype
    proj = project(camera, means, quats, scales, antialias=antialias)
    q = quats / torch.linalg.norm(quats, dim=-1, keepdim=True)
    w, x, y, z = q.unbind(-1)
    normals = torch.stack([2 * (x * z + w * y), 2 * (y * z - w * x), 1 - 2 * (x * x + y * y)], -1)
    center = (-(camera.R.T.to(torch.float32) @ camera.t.to(torch.float32))).to(dt)
    view = center - means
    normals = normals / torch.clamp(torch.linalg.norm(normals, dim=-1, keepdim=True), min=1e-8)
    normals = torch.where((normals * view).sum(-1, keepdim=True) < 0, -normals, normals)
    d = proj["depths"]
    feats = torch.cat([d[:, None], (d * d)[:, None], normals], 1)
    out = naive_render(camera, means, quats, scales, opacities, feats, antialias=antialias)
    alpha = out["alpha"]
    a = alpha[..., None]
    f = torch.where(a > 1e-6, out["image"] / torch.clamp(a, min=1e-6), torch.zeros_like(out["image"]))
    valid = (alpha > min_alpha).to(dt)
    denom = torch.clamp(valid.sum(), min=1.0)
    ed, ed2 = f[..., 0], f[..., 1]
    dv = (torch.clamp(ed2 - ed * ed, min=0.0) * valid).sum() / denom
    H, W = camera.height, camera.width
    u = torch.arange(W, dtype=dt) + 0.5
    v = torch.arange(H, dtype=dt) + 0.5
    xd = (u[None, :].expand(H, W) - camera.cx) / camera.fx
    yd = (v[:, None].expand(H, W) - camera.cy) / camera.fy
    pc = torch.stack([xd * ed, yd * ed, ed], -1)
    pts = (pc - camera.t.to(dt)) @ camera.R.to(dt)
    tx = pts[:-1, 1:] - pts[:-1, :-1]
    ty = pts[1:, :-1] - pts[:-1, :-1]
    dn = torch.linalg.cross(tx, ty)
    dn = dn / torch.clamp(torch.linalg.norm(dn, dim=-1, keepdim=True), min=1e-8)
    rn = f[:-1, :-1, 2:5]
    rn = rn / torch.clamp(torch.linalg.norm(rn, dim=-1, keepdim=True), min=1e-8)
    valid4 = valid[:-1, :-1] * valid[:-1, 1:] * valid[1:, :-1] * valid[1:, 1:]
    nc = ((1.0 - (rn * dn).sum(-1).abs()) * valid4).sum() / torch.clamp(valid4.sum(), min=1.0)
    return lam_var * dv + lam_normal * nc, dv, nc
