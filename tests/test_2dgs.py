"""2DGS surfel helpers on CPU tensors (the reference's tests/test_splatting.py
:477-515 restated): the thickness clamp, surfel export, and the camera's
unprojection (cameras.py:327-336) as the inverse of project_points."""

import math

import numpy as np
import pytest
import torch

from mlx3d_b200.cameras import Camera
from mlx3d_b200.splatting import GaussianModel


def test_2dgs_constraints_clamp_local_normal_scale():
    model = GaussianModel.from_points(torch.randn(12, 3, generator=torch.Generator().manual_seed(0)), sh_degree=0)
    with torch.no_grad():
        model.params["scales"].copy_(torch.full((12, 3), math.log(0.5)))
    model.apply_2dgs_constraints(max_thickness=0.01)
    s = torch.exp(model.params["scales"]).detach().numpy()
    assert np.all(s[:, 2] <= 0.010001)
    np.testing.assert_allclose(s[:, :2], 0.5, atol=1e-6)


def test_surfel_points_filter_cap_and_orient():
    pts = torch.tensor([[float(i), 0.0, 0.0] for i in range(5)])
    model = GaussianModel.from_points(pts, sh_degree=0)
    with torch.no_grad():
        model.params["opacities"].copy_(torch.tensor([-8.0, 2.0, 1.0, 4.0, -9.0]))
        model.params["scales"].copy_(torch.log(torch.tensor(
            [[10.0, 10.0, 0.01], [0.1, 0.1, 0.01], [3.0, 3.0, 0.01], [1.0, 4.0, 0.01], [20.0, 20.0, 0.01]])))
        model.params["quats"].copy_(torch.tensor([[1.0, 0.0, 0.0, 0.0]]).repeat(5, 1))
    surfels, normals = model.surfel_points(min_opacity=0.01, max_points=2, orient_towards=(0.0, 0.0, -1.0))
    np.testing.assert_allclose(surfels[:, 0].numpy(), [2.0, 3.0], atol=1e-6)
    np.testing.assert_allclose(normals.numpy(), [[0.0, 0.0, -1.0]] * 2, atol=1e-6)
    with pytest.raises(ValueError, match="max_points"):
        model.surfel_points(max_points=0)


@pytest.mark.parametrize("lens", [None, (0.05, -0.01, 0.001, 0.002), "fisheye", "ortho"])
def test_unproject_inverts_project(lens):
    kw = {}
    if lens == "fisheye":
        kw = dict(distortion=(0.02, -0.01, 0.0, 0.0), fisheye=True)
    elif lens == "ortho":
        kw = dict(orthographic=True)
    elif lens is not None:
        kw = dict(distortion=lens)
    cam = Camera.look_at(eye=(0.5, 0.3, -4.0), fov=50.0, width=64, height=48, **kw)
    pts = torch.randn(50, 3, generator=torch.Generator().manual_seed(1)) * 0.5
    xy, z = cam.project_points(pts)
    back = cam.unproject_points(xy, z)
    np.testing.assert_allclose(back.numpy(), pts.numpy(), atol=2e-4)
