"""Parity of the sm_100a path against the CPU oracle (GPU only).

Bar: radii, tiles touched, sorted ids, tile ranges, means2d / conics /
colours, image / final_T / n_contrib / depth bit-exact (both sides use the
same exactly rounded float32 operation order); gradients within 1e-4
relative L2 (atomic accumulation order is nondeterministic).
"""

import ctypes
import numpy as np
import pytest
import torch

import oracle.oracle as orc
from oracle import torch_ref
from mlx3d_b200 import _native as nat
from mlx3d_b200 import splatting as gs
from mlx3d_b200.cameras import Camera
from mlx3d_b200.scenes import make_scene
from tests.helpers import random_scene, rel_l2

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-4


def cu(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a)).to("cuda", dtype)


def npy(t):
    return t.detach().cpu().numpy()


def eq(a, b, what=""):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    bad = ~((a == b) | (np.isnan(a) & np.isnan(b))) if a.dtype.kind == "f" else a != b
    assert not bad.any(), f"{what}: {int(bad.sum())} of {a.size} differ; first at {np.argwhere(bad)[:3].tolist()}"


def activated(scene):
    p = scene.params
    s, o = orc.activate(p["scales"], p["opacities"])
    sh = np.concatenate([p["sh_dc"], p["sh_rest"]], axis=1)
    return p["means"], p["quats"], s, o, sh


SCENES = {
    "random300": lambda: None,
    "c0": lambda: make_scene(0),
    "c1": lambda: make_scene(1),
    "c2_200k": lambda: make_scene(2, n=200_000),
}


def scene_inputs(name):
    if name == "random300":
        cam, means, quats, scales, opac, colors = random_scene()
        sh = np.zeros((means.shape[0], 16, 3), np.float32)
        rng = np.random.default_rng(3)
        sh[:, 1:] = rng.normal(size=(means.shape[0], 15, 3)) * 0.1
        sh[:, 0] = (colors - 0.5) / torch_ref.SH_C0
        return cam, means, quats, scales, opac, sh, 3, False
    sc = SCENES[name]()
    means, quats, scales, opac, sh = activated(sc)
    return sc.cameras[0], means, quats, scales, opac, sh, sc.config.sh_degree, sc.config.antialias


@pytest.mark.parametrize("aa", [False, True])
@pytest.mark.parametrize("name", list(SCENES))
def test_projection_bit_exact(name, aa):
    cam, means, quats, scales, *_ = scene_inputs(name)
    got = gs.project_gaussians(cam, cu(means), cu(quats), cu(scales), antialias=aa)
    ref = orc.project(cam.to_native(), means, quats, scales, antialias=aa)
    for k in ("means2d", "conics", "depths", "radii", "compensation"):
        eq(npy(got[k]), ref[k], k)


@pytest.mark.parametrize("name", list(SCENES))
def test_binning_bit_exact(name):
    cam, means, quats, scales, *_ = scene_inputs(name)
    ref = orc.project(cam.to_native(), means, quats, scales)
    ids, ranges, tx, ty = gs.bin_gaussians(cu(ref["means2d"]), cu(ref["radii"]), cu(ref["depths"]), cam.width,
                                           cam.height)
    counts, rids, rranges, rtx, rty = orc.bin_gaussians(ref["means2d"], ref["radii"], ref["depths"], cam.width,
                                                        cam.height)
    assert (tx, ty) == (rtx, rty)
    eq(npy(ids), rids, "sorted_ids")
    eq(npy(ranges), rranges, "tile_ranges")


@pytest.mark.parametrize("name", list(SCENES))
def test_render_forward_bit_exact(name):
    cam, means, quats, scales, opac, sh, deg, aa = scene_inputs(name)
    bg = np.array([0.1, 0.2, 0.3], np.float32)
    out = gs.render_gaussians(cam, cu(means), cu(quats), cu(scales), cu(opac), sh=cu(sh), sh_degree=deg,
                              background=cu(bg), antialias=aa, render_depth=True)
    ref = orc.render(cam.to_native(), cam.width, cam.height, means, quats, scales, opac, sh=sh, sh_degree=deg,
                     background=bg, antialias=aa, with_depth=True)
    for k in ("means2d", "depths", "radii", "compensation", "image", "final_T", "n_contrib", "depth"):
        eq(npy(out[k]), ref[k], k)
    eq(npy(out["alpha"]), ref["alpha"], "alpha")
    eq(npy(out["tiles_touched"]), ref["tiles_touched"], "tiles_touched")


@pytest.mark.parametrize("name", ["random300", "c0", "c1"])
def test_model_render_with_fused_activations_bit_exact(name):
    if name == "random300":
        sc = make_scene(0, n=300)
    else:
        sc = make_scene(int(name[1]))
    model = gs.GaussianModel({k: v.clone() for k, v in sc.torch_params().items()}, sh_degree=3)
    model.active_sh_degree = sc.config.sh_degree
    cam = sc.cameras[0]
    out = model.render(cam, antialias=sc.config.antialias)
    means, quats, scales, opac, sh = activated(sc)
    ref = orc.render(cam.to_native(), cam.width, cam.height, means, quats, scales, opac, sh=sh,
                     sh_degree=sc.config.sh_degree, antialias=sc.config.antialias)
    for k in ("radii", "image", "final_T", "n_contrib"):
        eq(npy(out[k]), ref[k], k)


@pytest.mark.parametrize("name", list(SCENES))
def test_rasterize_backward_matches_oracle(name):
    cam, means, quats, scales, opac, sh, deg, aa = scene_inputs(name)
    ref = orc.render(cam.to_native(), cam.width, cam.height, means, quats, scales, opac, sh=sh, sh_degree=deg,
                     antialias=aa, background=np.array([0.2, 0.1, 0.4], np.float32))
    rng = np.random.default_rng(7)
    g_img = rng.normal(size=ref["image"].shape).astype(np.float32)
    g_T = rng.normal(size=ref["final_T"].shape).astype(np.float32)
    m2d = cu(ref["means2d"]).requires_grad_()
    con = cu(ref["conics"]).requires_grad_()
    col = cu(ref["colors"]).requires_grad_()
    op = cu(ref["opacities_eff"]).requires_grad_()
    out = gs.rasterize(m2d, con, col, op, cu(ref["sorted_ids"], torch.int32), cu(ref["tile_ranges"], torch.int32),
                       cam.width, cam.height, ref["tiles_x"], ref["tiles_y"], background=cu(ref["background"]))
    eq(npy(out["image"]), ref["image"], "image")
    torch.autograd.backward([out["image"], out["final_T"]], [cu(g_img), cu(g_T)])
    g = orc.rasterize_bwd(ref["means2d"], ref["conics"], ref["colors"], ref["opacities_eff"], ref["sorted_ids"],
                          ref["tile_ranges"], cam.width, cam.height, ref["background"], ref["final_T"],
                          ref["n_contrib"], g_img, g_T)
    for k, t in (("means2d", m2d), ("conics", con), ("colors", col), ("opacities", op)):
        assert rel_l2(npy(t.grad), g[k]) < GRAD_TOL, k


@pytest.mark.parametrize("aa", [False, True])
def test_project_backward_matches_autodiff(aa):
    sc = make_scene(2, n=20_000)
    means, quats, scales, *_ = activated(sc)
    cam = sc.cameras[0]
    rng = np.random.default_rng(9)
    n = means.shape[0]
    cots = {"means2d": rng.normal(size=(n, 2)), "conics": rng.normal(size=(n, 3)), "depths": rng.normal(size=n),
            "compensation": rng.normal(size=n)}
    m, q, s = cu(means).requires_grad_(), cu(quats).requires_grad_(), cu(scales).requires_grad_()
    out = gs.project_gaussians(cam, m, q, s, antialias=aa)
    # compensation is a constant (no gradient) unless antialias is on
    keys = ["means2d", "conics", "depths"] + (["compensation"] if aa else [])
    torch.autograd.backward([out[k] for k in keys], [cu(cots[k]) for k in keys])
    tm, tq, ts = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (means, quats, scales))
    ref = torch_ref.project(cam, tm, tq, ts, antialias=aa)
    torch.autograd.backward([ref[k] for k in keys], [torch.tensor(cots[k], dtype=torch.float64) for k in keys])
    for name, a, b in (("means", m, tm), ("quats", q, tq), ("scales", s, ts)):
        assert rel_l2(npy(a.grad), b.grad.numpy()) < GRAD_TOL, name


def test_eval_sh_forward_backward():
    rng = np.random.default_rng(4)
    sh = rng.normal(size=(5000, 16, 4)).astype(np.float32)
    dirs = rng.normal(size=(5000, 3)).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    for deg in range(4):
        a, d = cu(sh).requires_grad_(), cu(dirs).requires_grad_()
        out = gs.eval_sh(deg, a, d)
        eq(npy(out), orc.eval_sh(deg, sh, dirs), f"eval_sh deg {deg}")
        g = rng.normal(size=(5000, 4))
        out.backward(cu(g))
        ta = torch.tensor(sh, dtype=torch.float64, requires_grad=True)
        td = torch.tensor(dirs, dtype=torch.float64, requires_grad=True)
        torch_ref.eval_sh(deg, ta, td).backward(torch.tensor(g))
        assert rel_l2(npy(a.grad), ta.grad.numpy()) < GRAD_TOL
        if deg > 0:
            assert rel_l2(npy(d.grad), td.grad.numpy()) < GRAD_TOL


@pytest.mark.parametrize("name", list(SCENES))
def test_render_gradients_match_oracle(name):
    cam, means, quats, scales, opac, sh, deg, aa = scene_inputs(name)
    bg = np.array([0.3, 0.2, 0.1], np.float32)
    m, q, s, o, shv = (cu(a).requires_grad_() for a in (means, quats, scales, opac, sh))
    out = gs.render_gaussians(cam, m, q, s, o, sh=shv, sh_degree=deg, background=cu(bg), antialias=aa)
    rng = np.random.default_rng(11)
    g_img = rng.normal(size=(cam.height, cam.width, 3)).astype(np.float32)
    g_alpha = rng.normal(size=(cam.height, cam.width)).astype(np.float32)
    torch.autograd.backward([out["image"], out["alpha"]], [cu(g_img), cu(g_alpha)])
    _, g = orc.render_grads(cam, means, quats, scales, opac, sh=sh, sh_degree=deg, background=bg, antialias=aa,
                            grad_image=g_img, grad_alpha=g_alpha)
    for k, t in (("means", m), ("quats", q), ("scales", s), ("opacities", o), ("sh", shv)):
        assert rel_l2(npy(t.grad), g[k]) < GRAD_TOL, k


def test_model_gradients_through_fused_activations():
    sc = make_scene(1, n=30_000)
    params = sc.torch_params(requires_grad=True)
    model = gs.GaussianModel(params, sh_degree=3)
    model.active_sh_degree = 3
    cam = sc.cameras[0]
    out = model.render(cam)
    target = sc.target()
    (out["image"] - target).abs().mean().backward()
    # reference: same loss through torch activations + render_gaussians
    p2 = sc.torch_params(requires_grad=True)
    sh = torch.cat([p2["sh_dc"], p2["sh_rest"]], 1)
    s_act, o_act = orc.activate(sc.params["scales"], sc.params["opacities"])
    # use bit-identical activations so the forward passes match exactly
    s_t = cu(s_act) + (p2["scales"] - p2["scales"].detach()) * cu(s_act)
    o_t = cu(o_act) + (p2["opacities"] - p2["opacities"].detach()) * cu(o_act * (1 - o_act))
    out2 = gs.render_gaussians(cam, p2["means"], p2["quats"], s_t, o_t, sh=sh, sh_degree=3)
    eq(npy(out["image"]), npy(out2["image"]), "image")
    (out2["image"] - target).abs().mean().backward()
    for k in params:
        assert rel_l2(npy(params[k].grad), npy(p2[k].grad)) < GRAD_TOL, k


@pytest.mark.parametrize("channels", [1, 5, 20])
def test_feature_rendering_parity(channels):
    cam, means, quats, scales, opac, *_ = scene_inputs("c0")
    rng = np.random.default_rng(channels)
    feats = rng.normal(size=(means.shape[0], channels)).astype(np.float32)
    bg = np.linspace(-0.2, 0.2, channels).astype(np.float32)
    f = cu(feats).requires_grad_()
    out = gs.render_gaussian_features(cam, cu(means), cu(quats), cu(scales), cu(opac), f, background=cu(bg))
    p = orc.project(cam.to_native(), means, quats, scales)
    oe = opac * p["compensation"]
    _, ids, ranges, _, _ = orc.bin_gaussians(p["means2d"], p["radii"], p["depths"], cam.width, cam.height)
    ref = orc.rasterize_fwd(p["means2d"], p["conics"], feats, oe, ids, ranges, cam.width, cam.height, background=bg)
    eq(npy(out["features"]), ref["image"], "features")
    eq(npy(out["alpha"]), ref["alpha"], "alpha")
    g = rng.normal(size=ref["image"].shape).astype(np.float32)
    out["features"].backward(cu(g))
    gr = orc.rasterize_bwd(p["means2d"], p["conics"], feats, oe, ids, ranges, cam.width, cam.height, bg,
                           ref["final_T"], ref["n_contrib"], g)
    assert rel_l2(npy(f.grad), gr["colors"]) < GRAD_TOL


def test_depth_rendering_parity_and_normalized_features():
    cam, means, quats, scales, opac, *_ = scene_inputs("c1")
    d = gs.render_gaussian_depth(cam, cu(means), cu(quats), cu(scales), cu(opac))
    p = orc.project(cam.to_native(), means, quats, scales)
    oe = opac * p["compensation"]
    _, ids, ranges, _, _ = orc.bin_gaussians(p["means2d"], p["radii"], p["depths"], cam.width, cam.height)
    ref = orc.rasterize_fwd(p["means2d"], p["conics"], None, oe, ids, ranges, cam.width, cam.height,
                            depths=p["depths"])
    eq(npy(d["depth"]), ref["depth"], "depth")
    eq(npy(d["alpha"]), ref["alpha"], "alpha")
    f = gs.render_gaussian_features(cam, cu(means), cu(quats), cu(scales), cu(opac), d["depths"][:, None],
                                    background=torch.tensor([10.0], device="cuda"), normalize=True)
    valid = npy(d["alpha"]) > 1e-3
    np.testing.assert_allclose(npy(f["features"][..., 0])[valid], npy(d["depth"])[valid], atol=1e-4)
    assert np.abs(npy(f["features"][..., 0])[~valid]).max(initial=0.0) < 1e-6


# ------------------------------------------------------------------ edge cases
def _render_both(cam, means, quats, scales, opac, colors, bg=None):
    out = gs.render_gaussians(cam, cu(means), cu(quats), cu(scales), cu(opac), colors=cu(colors),
                              background=None if bg is None else cu(bg))
    ref = orc.render(cam.to_native(), cam.width, cam.height, means, quats, scales, opac, colors=colors,
                     background=bg)
    for k in ("radii", "image", "final_T", "n_contrib"):
        eq(npy(out[k]), ref[k], k)
    return out, ref


def test_empty_scene():
    cam = Camera.look_at(eye=(0, 0, -3.0), width=40, height=24)
    z = np.zeros((0, 3), np.float32)
    out, _ = _render_both(cam, z, np.zeros((0, 4), np.float32), z, np.zeros(0, np.float32), z,
                          bg=np.array([0.5, 0.25, 1.0], np.float32))
    np.testing.assert_array_equal(npy(out["image"]), np.broadcast_to([0.5, 0.25, 1.0], (24, 40, 3)))
    ids, ranges, _, _ = gs.bin_gaussians(torch.zeros(0, 2, device="cuda"), torch.zeros(0, device="cuda"),
                                         torch.zeros(0, device="cuda"), 40, 24)
    assert ids.shape == (0,) and not npy(ranges).any()


def test_all_culled_and_odd_image_sizes():
    rng = np.random.default_rng(0)
    for w, h in ((1, 1), (17, 33), (31, 16)):
        cam = Camera.look_at(eye=(0, 0, -3.0), width=w, height=h, fov=40.0)
        n = 64
        means = (rng.normal(size=(n, 3)) * 0.3).astype(np.float32)
        means[: n // 2, 2] = -10.0  # behind the camera
        quats = rng.normal(size=(n, 4)).astype(np.float32)
        scales = np.exp(rng.normal(size=(n, 3)) * 0.3 - 2.0).astype(np.float32)
        opac = rng.uniform(0.05, 0.99, size=n).astype(np.float32)
        cols = rng.uniform(size=(n, 3)).astype(np.float32)
        out, ref = _render_both(cam, means, quats, scales, opac, cols)
        assert (npy(out["radii"])[: n // 2] == 0).all()


def test_huge_gaussian_covers_every_tile_and_equal_depth_ties():
    cam = Camera.look_at(eye=(0, 0, -3.0), width=200, height=120, fov=60.0)
    n = 50
    rng = np.random.default_rng(1)
    means = np.zeros((n, 3), np.float32)
    means[:, :2] = rng.uniform(-0.5, 0.5, size=(n, 2))  # all at the same depth
    quats = np.tile(np.array([[1.0, 0, 0, 0]], np.float32), (n, 1))
    scales = np.full((n, 3), 0.05, np.float32)
    scales[0] = 5.0  # covers the whole image
    opac = np.full(n, 0.3, np.float32)
    cols = rng.uniform(size=(n, 3)).astype(np.float32)
    out, ref = _render_both(cam, means, quats, scales, opac, cols)
    tx, ty = 13, 8
    assert ref["tiles_touched"][0] == tx * ty
    eq(npy(gs.bin_gaussians(out["means2d"], out["radii"], out["depths"], 200, 120)[0]), ref["sorted_ids"], "ids")


def test_full_size_c2_properties():
    """Size-independent checks at the benchmark size (1M Gaussians, 1080p)."""
    sc = make_scene(2)
    params = sc.torch_params(requires_grad=True)
    model = gs.GaussianModel(params, sh_degree=3)
    model.active_sh_degree = 3
    cam = sc.cameras[0]
    out = model.render(cam, antialias=True)
    img = out["image"]
    assert torch.isfinite(img).all() and (npy(out["alpha"]) >= 0).all() and (npy(out["alpha"]) <= 1).all()
    ids, ranges, tx, ty = gs.bin_gaussians(out["means2d"], out["radii"], out["depths"], cam.width, cam.height)
    ids, ranges = npy(ids), npy(ranges).astype(np.int64)
    depths, radii = npy(out["depths"]), npy(out["radii"])
    # every tile range is sorted by depth, then by Gaussian index
    tiles = np.repeat(np.arange(tx * ty), ranges[:, 1] - ranges[:, 0])
    assert tiles.shape[0] == ids.shape[0]
    order = np.lexsort((ids, depths[ids], tiles))
    np.testing.assert_array_equal(order, np.arange(ids.shape[0]))
    nonempty = ranges[:, 1] > ranges[:, 0]
    assert (ranges[nonempty][1:, 0] == ranges[nonempty][:-1, 1]).all()
    assert (radii[ids] > 0).all()
    # no radix-pass block gave up waiting for its predecessors
    cnt = ctypes.c_uint64(0)
    nat.call("gs_wait_failures", ctypes.byref(cnt), 1)
    assert cnt.value == 0
    # backward is linear in the output cotangent
    g = torch.randn_like(img)
    g1 = torch.autograd.grad(img, list(params.values()), g, retain_graph=True)
    g2 = torch.autograd.grad(img, list(params.values()), 2.0 * g)
    for a, b in zip(g1, g2):
        assert rel_l2(npy(b), 2.0 * npy(a)) < 1e-5


def test_full_size_c2_forward_bit_exact_and_gradients():
    """The benchmark workload itself (1M Gaussians, SH3, 1080p, antialias)
    against the oracle: forward bit-exact, gradients within 1e-4."""
    sc = make_scene(2)
    cam = sc.cameras[0]
    params = sc.torch_params(requires_grad=True)
    model = gs.GaussianModel(params, sh_degree=3)
    model.active_sh_degree = 3
    out = model.render(cam, antialias=True)
    means, quats, scales, opac, sh = activated(sc)
    fwd = orc.render(cam.to_native(), cam.width, cam.height, means, quats, scales, opac, sh=sh, sh_degree=3,
                     antialias=True)
    for k in ("radii", "image", "final_T", "n_contrib"):
        eq(npy(out[k]), fwd[k], k)
    rng = np.random.default_rng(21)
    g_img = rng.normal(size=(cam.height, cam.width, 3)).astype(np.float32)
    out["image"].backward(cu(g_img))
    _, g = orc.render_grads(cam, means, quats, scales, opac, sh=sh, sh_degree=3, antialias=True, grad_image=g_img,
                            fwd=fwd)
    s_act, o_act = scales, opac
    checks = {
        "means": (params["means"].grad, g["means"]),
        "quats": (params["quats"].grad, g["quats"]),
        "scales": (params["scales"].grad, g["scales"] * s_act),
        "opacities": (params["opacities"].grad, g["opacities"] * o_act * (1 - o_act)),
        "sh_dc": (params["sh_dc"].grad, g["sh"][:, :1]),
        "sh_rest": (params["sh_rest"].grad, g["sh"][:, 1:]),
    }
    for k, (a, b) in checks.items():
        assert rel_l2(npy(a), b) < GRAD_TOL, k


@pytest.mark.parametrize("name", ["random300", "c0", "c2_200k"])
def test_refined_binning_and_render_bit_exact(name):
    cam, means, quats, scales, opac, sh, deg, aa = scene_inputs(name)
    ref = orc.project(cam.to_native(), means, quats, scales)
    ids, ranges, _, _ = gs.bin_gaussians(cu(ref["means2d"]), cu(ref["radii"]), cu(ref["depths"]), cam.width,
                                         cam.height, conics=cu(ref["conics"]))
    _, rids, rranges, _, _ = orc.bin_gaussians(ref["means2d"], ref["radii"], ref["depths"], cam.width, cam.height,
                                               conics=ref["conics"])
    eq(npy(ids), rids, "sorted_ids")
    eq(npy(ranges), rranges, "tile_ranges")
    m, q, s, o, shv = (cu(a).requires_grad_() for a in (means, quats, scales, opac, sh))
    out = gs.render_gaussians(cam, m, q, s, o, sh=shv, sh_degree=deg, antialias=aa, refine_tiles=True)
    fwd = orc.render(cam.to_native(), cam.width, cam.height, means, quats, scales, opac, sh=sh, sh_degree=deg,
                     antialias=aa, refine_tiles=True)
    for k in ("image", "final_T", "n_contrib"):
        eq(npy(out[k]), fwd[k], k)
    g_img = np.random.default_rng(2).normal(size=fwd["image"].shape).astype(np.float32)
    out["image"].backward(cu(g_img))
    _, g = orc.render_grads(cam, means, quats, scales, opac, sh=sh, sh_degree=deg, antialias=aa, grad_image=g_img,
                            fwd=fwd)
    for k, t in (("means", m), ("quats", q), ("scales", s), ("opacities", o), ("sh", shv)):
        assert rel_l2(npy(t.grad), g[k]) < GRAD_TOL, k
