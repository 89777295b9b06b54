"""The CPU oracle pinned against the reference's own tests (CPU only).

MLX cannot run here, so no golden vectors of the reference exist; the pins
are the known-answer and cross-check tests of src/mlx3d's
tests/test_splatting.py, re-expressed against the oracle:
  :43-54   SH degree-0 identity and DC round trip
  :57-72   centre Gaussian -> (32, 32), depth 3, radius > 0; behind camera -> 0
  :114-165 projection equals the explicit T Sigma T^T matrix formula, radii exact
  :168-195 antialias compensation = var / (var + 0.3) for an isotropic Gaussian
  :198-211 binning invariants
  :214-222, 243-277 tile compositor vs the naive renderer (reference.py), 1e-3
  :280-337 depth and feature rendering
  :340-365, 390-414 gradients vs autodiff of the naive renderer (1e-3 / 2e-3)
"""

import math

import numpy as np
import pytest
import torch

import oracle.oracle as orc
from oracle import torch_ref
from mlx3d_b200.cameras import Camera
from tests.helpers import max_rel, random_scene, t64


def _proj(cam, means, quats, scales, **kw):
    return orc.project(cam.to_native(), means, quats, scales, **kw)


def test_expf_within_two_ulp():
    xs = np.concatenate([np.linspace(-103.0, 88.0, 20001), np.linspace(-6.0, 0.0, 20001), [0.0, -1e-30, 1e-30]])
    for x in xs.astype(np.float32):
        got = orc.expf(float(x))
        ref = math.exp(float(x))
        ulp = np.spacing(np.float32(ref)) if ref > 1.2e-38 else np.float32(1.4e-45)
        assert abs(got - ref) <= 2 * float(ulp), (x, got, ref)


def test_compositor_exponential_is_bitwise_gs_expf_on_its_domain():
    assert orc.expf_nonpos_mismatches() == 0


def test_sh_dc_roundtrip_and_degree0_identity():
    rng = np.random.default_rng(1)
    rgb = rng.uniform(size=(10, 3)).astype(np.float32)
    sh = ((rgb - 0.5) / torch_ref.SH_C0).astype(np.float32)
    dirs = rng.normal(size=(10, 3)).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    out = orc.eval_sh(0, sh[:, None, :], dirs)
    np.testing.assert_allclose(out, rgb, atol=1e-5)


def test_eval_sh_matches_restatement():
    rng = np.random.default_rng(2)
    sh = rng.normal(size=(64, 16, 5)).astype(np.float32)
    dirs = rng.normal(size=(64, 3)).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    for deg in range(4):
        ref = torch_ref.eval_sh(deg, torch.tensor(sh, dtype=torch.float64), torch.tensor(dirs, dtype=torch.float64))
        np.testing.assert_allclose(orc.eval_sh(deg, sh, dirs), ref.numpy(), atol=2e-6)


def test_projection_center_gaussian():
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), width=64, height=64, fov=60.0)
    p = _proj(cam, np.zeros((1, 3)), [[1.0, 0, 0, 0]], np.full((1, 3), 0.1))
    np.testing.assert_allclose(p["means2d"][0], [32.0, 32.0], atol=1e-3)
    assert abs(float(p["depths"][0]) - 3.0) < 1e-5
    assert float(p["radii"][0]) > 0


def test_projection_culls_behind_camera():
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), width=64, height=64)
    p = _proj(cam, [[0.0, 0.0, -10.0]], [[1.0, 0, 0, 0]], np.full((1, 3), 0.1))
    assert float(p["radii"][0]) == 0.0


def test_projection_matches_matrix_formula():
    rng = np.random.default_rng(11)
    cam = Camera.look_at(eye=(0.3, -0.2, -3.0), at=(0, 0, 0), width=80, height=48, fov=55.0)
    means = (rng.normal(size=(32, 3)) * 0.4).astype(np.float32)
    quats = rng.normal(size=(32, 4)).astype(np.float32)
    scales = np.exp(rng.normal(size=(32, 3)) * 0.2 - 2.0).astype(np.float32)
    out = _proj(cam, means, quats, scales)
    m, q, s = (torch.tensor(a) for a in (means, quats, scales))
    R, t = cam.R, cam.t
    p_cam = m @ R.T + t
    x, y, z = p_cam[:, 0], p_cam[:, 1], p_cam[:, 2]
    zs = torch.clamp(z, min=1e-6)
    means2d = torch.stack([cam.fx * x / zs + cam.cx, cam.fy * y / zs + cam.cy], -1)
    tfx, tfy = 0.5 * cam.width / cam.fx, 0.5 * cam.height / cam.fy
    tx = torch.clamp(x / zs, -1.3 * tfx, 1.3 * tfx) * zs
    ty = torch.clamp(y / zs, -1.3 * tfy, 1.3 * tfy) * zs
    zero = torch.zeros_like(zs)
    iz = 1.0 / zs
    iz2 = iz * iz
    J = torch.stack([torch.stack([cam.fx * iz, zero, -cam.fx * tx * iz2], -1),
                     torch.stack([zero, cam.fy * iz, -cam.fy * ty * iz2], -1)], -2)
    from mlx3d_b200.splatting.projection import quat_scale_to_cov3d

    cov3d = quat_scale_to_cov3d(q, s)
    T = J @ R
    cov2d = T @ cov3d @ T.transpose(-1, -2)
    a, b, c = cov2d[:, 0, 0] + 0.3, cov2d[:, 0, 1], cov2d[:, 1, 1] + 0.3
    det = a * c - b * b
    ds = torch.clamp(det, min=1e-12)
    conics = torch.stack([c / ds, -b / ds, a / ds], -1)
    mid = 0.5 * (a + c)
    radii = torch.ceil(3.0 * torch.sqrt(torch.clamp(mid + torch.sqrt(torch.clamp(mid * mid - det, min=0.01)), min=0)))
    radii = torch.where((z > cam.znear) & (det > 0), radii, torch.zeros_like(radii))
    np.testing.assert_allclose(out["means2d"], means2d.numpy(), atol=1e-5)
    np.testing.assert_allclose(out["conics"], conics.numpy(), atol=1e-4)
    np.testing.assert_allclose(out["depths"], z.numpy(), atol=1e-5)
    np.testing.assert_array_equal(out["radii"], radii.numpy())
    np.testing.assert_array_equal(out["compensation"], np.ones(32, np.float32))


def test_projection_antialias_compensation_matches_isotropic_formula():
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), width=64, height=64, fov=60.0)
    scales = np.array([[0.001] * 3, [0.1] * 3], np.float32)
    out = _proj(cam, np.zeros((2, 3)), [[1.0, 0, 0, 0]] * 2, scales, antialias=True)
    var = (cam.fx * scales[:, 0] / 3.0) ** 2
    np.testing.assert_allclose(out["compensation"], var / (var + 0.3), atol=1e-5)
    comp = out["compensation"]
    assert (comp >= 0).all() and (comp <= 1).all() and comp[0] < comp[1]
    nb = _proj(cam, np.zeros((1, 3)), [[1.0, 0, 0, 0]], [[0.001] * 3], blur=0.0, antialias=True)
    np.testing.assert_array_equal(nb["compensation"], [1.0])


def test_binning_invariants_and_key_order():
    cam, means, quats, scales, opac, colors = random_scene()
    p = _proj(cam, means, quats, scales)
    counts, ids, ranges, tx, ty = orc.bin_gaussians(p["means2d"], p["radii"], p["depths"], cam.width, cam.height)
    assert (tx, ty) == (6, 4)
    assert (ranges[:, 1] >= ranges[:, 0]).all()
    assert int((ranges[:, 1] - ranges[:, 0]).sum()) == ids.shape[0] == counts.sum()
    assert ids.min() >= 0 and ids.max() < means.shape[0]
    # The reference's key tile*N + rank(depth) orders duplicates by
    # (tile, depth, Gaussian index) when the depth argsort is stable.
    tiles = np.empty_like(ids)
    for t in range(tx * ty):
        tiles[ranges[t, 0]:ranges[t, 1]] = t
    order = np.lexsort((ids, p["depths"][ids], tiles))
    np.testing.assert_array_equal(order, np.arange(ids.shape[0]))


def _naive(cam, means, quats, scales, opac, colors, bg, antialias=False):
    return torch_ref.naive_render(cam, t64(means), t64(quats), t64(scales), t64(opac), t64(colors), t64(bg),
                                  antialias=antialias)


def test_tile_compositor_matches_naive_forward():
    cam, means, quats, scales, opac, colors = random_scene()
    bg = np.array([0.1, 0.2, 0.3], np.float32)
    out = orc.render(cam.to_native(), cam.width, cam.height, means, quats, scales, opac, colors=colors, background=bg)
    ref = _naive(cam, means, quats, scales, opac, colors, bg)
    np.testing.assert_allclose(out["image"], ref["image"].numpy(), atol=1e-3)
    np.testing.assert_allclose(out["alpha"], ref["alpha"].numpy(), atol=1e-3)


def test_antialiased_render_matches_naive_and_reduces_alpha():
    cam, means, quats, scales, opac, colors = random_scene()
    opac = (opac * 0.1).astype(np.float32)
    bg = np.array([0.1, 0.2, 0.3], np.float32)
    plain = orc.render(cam.to_native(), cam.width, cam.height, means, quats, scales, opac, colors=colors,
                       background=bg)
    aa = orc.render(cam.to_native(), cam.width, cam.height, means, quats, scales, opac, colors=colors, background=bg,
                    antialias=True)
    ref = _naive(cam, means, quats, scales, opac, colors, bg, antialias=True)
    np.testing.assert_allclose(aa["image"], ref["image"].numpy(), atol=1e-3)
    np.testing.assert_allclose(aa["alpha"], ref["alpha"].numpy(), atol=1e-3)
    assert float((aa["alpha"] - plain["alpha"]).max()) <= 1e-6
    comp = aa["compensation"]
    assert (comp >= 0).all() and (comp <= 1).all() and (comp < 1).any()


def test_depth_and_normalized_feature_depth():
    cam, means, quats, scales, opac, _ = random_scene()
    W, H = cam.width, cam.height
    p = _proj(cam, means, quats, scales)
    opac_eff = opac * p["compensation"]
    _, ids, ranges, _, _ = orc.bin_gaussians(p["means2d"], p["radii"], p["depths"], W, H)
    d = orc.rasterize_fwd(p["means2d"], p["conics"], None, opac_eff, ids, ranges, W, H, depths=p["depths"])
    valid = d["alpha"] > 1e-3
    assert valid.any()
    assert np.isfinite(d["depth"][valid]).all() and d["depth"][valid].min() > 0
    f = orc.rasterize_fwd(p["means2d"], p["conics"], p["depths"][:, None], opac_eff, ids, ranges, W, H)
    alpha = f["alpha"]
    feat = np.where(alpha > 1e-6, f["image"][..., 0] / np.maximum(alpha, 1e-6), 0.0)
    np.testing.assert_allclose(alpha, d["alpha"], atol=1e-5)
    np.testing.assert_allclose(feat[valid], d["depth"][valid], atol=1e-4)


def test_feature_compositing_with_five_channels_matches_naive():
    cam, means, quats, scales, opac, _ = random_scene()
    n = means.shape[0]
    feats = np.concatenate([means, np.arange(n * 2, dtype=np.float32).reshape(n, 2) / n], 1).astype(np.float32)
    bg = np.linspace(-0.2, 0.2, 5).astype(np.float32)
    p = _proj(cam, means, quats, scales)
    _, ids, ranges, _, _ = orc.bin_gaussians(p["means2d"], p["radii"], p["depths"], cam.width, cam.height)
    out = orc.rasterize_fwd(p["means2d"], p["conics"], feats, opac * p["compensation"], ids, ranges, cam.width,
                            cam.height, background=bg)
    ref = _naive(cam, means, quats, scales, opac, feats, bg)
    assert out["image"].shape == (cam.height, cam.width, 5)
    np.testing.assert_allclose(out["image"], ref["image"].numpy(), atol=1e-3)


@pytest.mark.parametrize("use_sh", [False, True])
def test_oracle_gradients_match_naive_autodiff(use_sh):
    cam, means, quats, scales, opac, colors = random_scene()
    rng = np.random.default_rng(5)
    target = rng.uniform(size=(cam.height, cam.width, 3)).astype(np.float32)
    bg = np.zeros(3, np.float32)
    sh = None
    if use_sh:
        sh = (rng.normal(size=(means.shape[0], 16, 3)) * 0.1).astype(np.float32)
        sh[:, 0] = (colors - 0.5) / torch_ref.SH_C0
    fwd = orc.render(cam.to_native(), cam.width, cam.height, means, quats, scales, opac,
                     colors=None if use_sh else colors, sh=sh, sh_degree=3, background=bg)
    npx = cam.height * cam.width
    g_img = 2.0 * (fwd["image"] - target) / (npx * 3)
    g_alpha = np.full((cam.height, cam.width), 0.05 / npx, np.float32)
    _, g = orc.render_grads(cam, means, quats, scales, opac, colors=None if use_sh else colors, sh=sh,
                            sh_degree=3, background=bg, grad_image=g_img, grad_alpha=g_alpha, fwd=fwd)
    m, q, s, o = t64(means, True), t64(quats, True), t64(scales, True), t64(opac, True)
    if use_sh:
        shv = t64(sh, True)
        dirs = torch_ref.view_dirs(cam, m).detach()
        col = torch.clamp(torch_ref.eval_sh(3, shv, dirs), min=0.0)
    else:
        col = t64(colors, True)
    ref = torch_ref.naive_render(cam, m, q, s, o, col, t64(bg))
    loss = ((ref["image"] - t64(target)) ** 2).mean() + 0.05 * ref["alpha"].mean()
    loss.backward()
    pairs = [("means", m), ("quats", q), ("scales", s), ("opacities", o)]
    pairs.append(("sh", shv) if use_sh else ("colors", col))
    for name, leaf in pairs:
        assert max_rel(g[name], leaf.grad.numpy()) < 1e-3, name


def test_refined_tiles_render_matches_naive_and_drop_duplicates():
    """test_splatting.py:225-240: rendering with refine_tiles still matches the
    naive renderer at 1e-3; the refinement only removes duplicates."""
    cam, means, quats, scales, opac, colors = random_scene()
    bg = np.array([0.1, 0.2, 0.3], np.float32)
    out = orc.render(cam.to_native(), cam.width, cam.height, means, quats, scales, opac, colors=colors,
                     background=bg, refine_tiles=True)
    ref = _naive(cam, means, quats, scales, opac, colors, bg)
    np.testing.assert_allclose(out["image"], ref["image"].numpy(), atol=1e-3)
    np.testing.assert_allclose(out["alpha"], ref["alpha"].numpy(), atol=1e-3)
    p = _proj(cam, means, quats, scales)
    full = orc.bin_gaussians(p["means2d"], p["radii"], p["depths"], cam.width, cam.height)
    ref_ids, ref_ranges = full[1], full[2]
    ids, ranges = out["sorted_ids"], out["tile_ranges"]
    assert 0 < ids.shape[0] < ref_ids.shape[0]
    for t in range(ranges.shape[0]):
        kept = ids[ranges[t, 0]:ranges[t, 1]]
        allv = list(ref_ids[ref_ranges[t, 0]:ref_ranges[t, 1]])
        assert set(kept) <= set(allv)
        pos = [allv.index(g) for g in kept]
        assert pos == sorted(pos)  # same (depth, index) order


def _ut_cams():
    base = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), fov=60.0, width=128, height=128)
    mk = lambda **kw: Camera(R=base.R, t=base.t, fx=base.fx, fy=base.fy, cx=base.cx, cy=base.cy,  # noqa: E731
                             width=base.width, height=base.height, **kw)
    return base, mk


def test_ut_projection_respects_camera_distortion():
    """test_splatting.py:75-97 on the oracle."""
    base, mk = _ut_cams()
    cam = mk(distortion=(-0.35, 0.12, 0.002, -0.001))
    means = np.array([[0.75, 0.45, 0.0]], np.float32)
    quats = np.array([[1.0, 0, 0, 0]], np.float32)
    scales = np.full((1, 3), 1e-4, np.float32)
    ut = orc.project_ut(cam, means, quats, scales)
    center = torch_ref.project_points(cam, torch.tensor(means)).numpy()
    ewa = orc.project(cam.to_native(), means, quats, scales)
    np.testing.assert_allclose(ut["means2d"], center, atol=1e-3)
    assert np.abs(ewa["means2d"] - center).max() > 0.25
    assert ut["radii"][0] > 0


def test_ut_projection_close_to_ewa_for_pinhole_small_gaussians():
    """test_splatting.py:100-111 on the oracle."""
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), fov=55.0, width=96, height=64)
    means = np.array([[0.0, 0.0, 0.0], [0.2, -0.1, 0.3]], np.float32)
    quats = np.array([[1.0, 0, 0, 0], [0.9, 0.1, 0.2, 0.3]], np.float32)
    scales = np.full((2, 3), 1e-3, np.float32)
    ut = orc.project_ut(cam, means, quats, scales)
    ewa = orc.project(cam.to_native(), means, quats, scales)
    np.testing.assert_allclose(ut["means2d"], ewa["means2d"], atol=1e-3)
    np.testing.assert_allclose(ut["conics"], ewa["conics"], rtol=0.05)


@pytest.mark.parametrize("lens", ["pinhole", "brown", "fisheye", "ortho"])
def test_ut_oracle_matches_autograd_restatement(lens):
    base, mk = _ut_cams()
    cam = {"pinhole": base, "brown": mk(distortion=(-0.2, 0.05, 0.001, -0.002, 0.01)),
           "fisheye": mk(distortion=(0.05, -0.01, 0.002, 0.0), fisheye=True),
           "ortho": Camera(R=base.R, t=base.t, fx=40.0, fy=40.0, cx=64.0, cy=64.0, width=128, height=128,
                           orthographic=True)}[lens]
    rng = np.random.default_rng(3)
    means = (rng.normal(size=(64, 3)) * 0.5).astype(np.float32)
    quats = rng.normal(size=(64, 4)).astype(np.float32)
    scales = np.exp(rng.normal(size=(64, 3)) * 0.3 - 3).astype(np.float32)
    a = orc.project_ut(cam, means, quats, scales, antialias=True)
    b = torch_ref.project_ut(cam, t64(means), t64(quats), t64(scales), antialias=True)
    np.testing.assert_allclose(a["means2d"], b["means2d"].numpy(), atol=1e-3)
    np.testing.assert_allclose(a["conics"], b["conics"].numpy(), rtol=1e-3, atol=1e-4)
    np.testing.assert_allclose(a["compensation"], b["compensation"].numpy(), atol=1e-4)
