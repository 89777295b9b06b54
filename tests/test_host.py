"""Host-side logic (no GPU): cameras, argument validation, scene generation."""

import math

import numpy as np
import pytest
import torch

from mlx3d_b200 import splatting as gs
from mlx3d_b200.cameras import Camera, look_at
from mlx3d_b200.scenes import CONFIGS, make_scene


def test_camera_from_fov_and_look_at():
    cam = Camera.look_at(eye=(0, 0, -4.0), width=256, height=128, fov=60.0)
    assert cam.fx == pytest.approx(128 / (2 * math.tan(math.radians(30))))
    assert (cam.cx, cam.cy) == (128.0, 64.0)
    # camera centre recovers the eye; R is orthonormal
    np.testing.assert_allclose(cam.camera_center.numpy(), [0, 0, -4.0], atol=1e-6)
    np.testing.assert_allclose((cam.R @ cam.R.T).numpy(), np.eye(3), atol=1e-6)
    # the world origin projects to the principal point
    p = cam.world_to_camera(torch.zeros(1, 3))
    assert p[0, 2].item() == pytest.approx(4.0)


def test_native_camera_rounds_like_mixed_precision_expressions():
    cam = Camera.look_at(eye=(0.3, -0.2, -3.0), width=80, height=48, fov=55.0)
    nc = cam.to_native()
    f32 = lambda v: float(np.float32(v))  # noqa: E731
    assert nc.fx == f32(cam.fx) and nc.neg_fx == f32(-cam.fx)
    assert nc.clip_x == f32(1.3 * (0.5 * cam.width / cam.fx))
    assert nc.znear == f32(0.01)
    assert (nc.width, nc.height) == (80, 48)


def test_look_at_matches_formula():
    R, t = look_at([1.0, 2.0, -3.0], [0.0, 0.0, 0.0], [0.0, 1.0, 0.0])
    eye = torch.tensor([1.0, 2.0, -3.0])
    np.testing.assert_allclose((R @ eye + t).numpy(), 0, atol=1e-6)
    z = -eye / eye.norm()
    np.testing.assert_allclose(R[2].numpy(), z.numpy(), atol=1e-6)


def test_cpu_tensors_are_rejected():
    cam = Camera.look_at(eye=(0, 0, -3.0), width=32, height=32)
    with pytest.raises(ValueError, match="CUDA"):
        gs.project_gaussians(cam, torch.zeros(1, 3), torch.tensor([[1.0, 0, 0, 0]]), torch.ones(1, 3))
    from mlx3d_b200 import losses

    with pytest.raises(ValueError, match="CUDA"):
        losses.l1_loss(torch.zeros(4), torch.zeros(4))
    with pytest.raises(ValueError, match="shape"):
        losses.l1_loss(torch.zeros(4), torch.zeros(5))


def test_render_argument_validation():
    cam = Camera.look_at(eye=(0, 0, -3.0), width=32, height=32)
    z = torch.zeros(2, 3)
    with pytest.raises(ValueError, match="exactly one"):
        gs.render_gaussians(cam, z, torch.zeros(2, 4), z, torch.zeros(2))
    with pytest.raises(ValueError, match="projection"):
        gs.render_gaussians(cam, z, torch.zeros(2, 4), z, torch.zeros(2), colors=z, projection="bad")
    with pytest.raises(ValueError, match="features must have shape"):
        gs.render_gaussian_features(cam, z, torch.zeros(2, 4), z, torch.zeros(2), torch.zeros(2))
    with pytest.raises(ValueError, match="same first dimension"):
        gs.render_gaussian_features(cam, z, torch.zeros(2, 4), z, torch.zeros(2), torch.zeros(1, 4))
    with pytest.raises(ValueError, match="CUDA"):
        gs.render_gaussians(cam, z, torch.zeros(2, 4), z, torch.zeros(2), colors=z, projection="ut")


def test_sh_helpers():
    rgb = torch.rand(10, 3)
    torch.testing.assert_close(gs.sh_to_rgb(gs.rgb_to_sh(rgb)), rgb)
    assert gs.num_sh_bases(3) == 16


def test_scene_generator_shapes_and_determinism():
    a = make_scene(1, n=2000)
    b = make_scene(1, n=2000)
    for k in a.params:
        np.testing.assert_array_equal(a.params[k], b.params[k])
    p = a.params
    assert p["means"].shape == (2000, 3) and p["sh_rest"].shape == (2000, 15, 3)
    assert a.cameras[0].width == 1280 and a.cameras[0].height == 720
    c3 = make_scene(3, n=1000)
    assert len(c3.cameras) == 64
    eyes = np.stack([c.camera_center.numpy() for c in c3.cameras])
    np.testing.assert_allclose(np.linalg.norm(eyes, axis=1), 6.0, rtol=1e-5)
    # no view within 5 degrees of the poles (look_at up = +y)
    assert np.degrees(np.arccos(np.abs(eyes[:, 1]) / 6.0)).min() >= 5.0
    c4 = make_scene(4, n=1000, views=4)
    assert len(c4.cameras) == 4 and CONFIGS[4].with_depth
