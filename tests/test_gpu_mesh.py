"""Hard mesh rasterizer on the GPU: the kernel is bit-identical to the CPU
oracle on the same binned triangles, and rasterize_meshes reproduces the
reference's behaviours (tests/test_rasterizer.py:20-86)."""

import ctypes

import numpy as np
import pytest
import torch

import oracle.oracle as orc
from mlx3d_b200 import _native as nat
from mlx3d_b200.cameras import Camera
from mlx3d_b200.renderer import interpolate_face_attributes, rasterize_meshes
from tests.helpers import ico_sphere
from tests.test_mesh_oracle import _binned

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("level,w,h", [(1, 48, 40), (3, 200, 120)])
def test_kernel_bit_exact_against_oracle(level, w, h):
    v, f = ico_sphere(level, 1.0)
    cam = Camera.look_at(eye=(2.2, 1.6, 2.2), at=(0, 0, 0), fov=45.0, width=w, height=h)
    tri_xy, tri_z, ids, ranges = _binned(cam, v, f)
    ref_p, ref_z = orc.mesh_rasterize(tri_xy, tri_z, ids, ranges, w, h, cam.znear)
    d = lambda a: torch.tensor(np.ascontiguousarray(a), device="cuda")  # noqa: E731
    gx, gz, gi, gr = d(tri_xy), d(tri_z), d(ids), d(ranges)
    p2f = torch.empty((h, w), dtype=torch.int32, device="cuda")
    zb = torch.empty((h, w), device="cuda")
    nat.call("gs_mesh_rasterize", nat.ptr(gx), nat.ptr(gz), f.shape[0], nat.ptr(gi), nat.ptr(gr), w, h,
             ctypes.c_float(cam.znear), nat.ptr(p2f), nat.ptr(zb), nat.stream())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(p2f.cpu().numpy(), ref_p)
    np.testing.assert_array_equal(zb.cpu().numpy(), ref_z)
    assert (ref_p >= 0).mean() > 0.1


def _tri():
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), fov=60.0, width=32, height=32)
    verts = torch.tensor([[-0.6, -0.5, 0.0], [0.6, -0.5, 0.0], [0.0, 0.6, 0.0]], device="cuda")
    return cam, verts, torch.tensor([[0, 1, 2]], dtype=torch.int32, device="cuda")


def test_triangle_hit_miss_and_barycentrics():
    cam, v, f = _tri()
    frag = rasterize_meshes(cam, v, f)
    assert int(frag.pix_to_face[16, 16]) == 0 and int(frag.pix_to_face[0, 0]) == -1
    assert not bool(frag.valid[0, 0])
    s = frag.bary.sum(-1)
    err = (torch.where(frag.valid, s, torch.ones_like(s)) - 1.0).abs()
    assert float(err.max()) < 1e-4
    colors = torch.eye(3, device="cuda")
    img = interpolate_face_attributes(frag, colors)
    csum = img.sum(-1)
    assert float((torch.where(frag.valid, csum, torch.ones_like(csum)) - 1.0).abs().max()) < 1e-4
    assert float(img.min()) >= -1e-5


def test_near_face_wins():
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), fov=60.0, width=16, height=16)
    v = torch.tensor([[-0.6, -0.5, 0.5], [0.6, -0.5, 0.5], [0.0, 0.6, 0.5],
                      [-0.6, -0.5, -0.5], [0.6, -0.5, -0.5], [0.0, 0.6, -0.5]], device="cuda")
    f = torch.tensor([[0, 1, 2], [3, 4, 5]], device="cuda")
    assert int(rasterize_meshes(cam, v, f).pix_to_face[8, 8]) == 1


def test_gradient_flows_to_vertices_and_matches_oracle_visibility():
    v, f = ico_sphere(2, 1.0)
    cam = Camera.look_at(eye=(2.2, 1.6, 2.2), at=(0, 0, 0), fov=45.0, width=48, height=48)
    vt = torch.tensor(v, device="cuda", requires_grad=True)
    frag = rasterize_meshes(cam, vt, torch.tensor(f, device="cuda"))
    ref_p, _ = orc.mesh_rasterize(*_binned(cam, v, f), cam.width, cam.height, cam.znear)
    # device-side binning (torch centroid / radius) may differ from numpy's in the last
    # bit; a bounding circle contains its triangle either way, so visibility agrees
    assert (frag.pix_to_face.cpu().numpy() != ref_p).sum() <= 2
    loss = interpolate_face_attributes(frag, 0.5 * vt + 0.5).sum()
    loss.backward()
    assert torch.isfinite(vt.grad).all() and float(vt.grad.abs().sum()) > 0.0


def test_mesh_outside_the_view_and_empty_mesh():
    cam, v, f = _tri()
    frag = rasterize_meshes(cam, v + torch.tensor([0.0, 0.0, -10.0], device="cuda"), f)  # behind the camera
    assert int((frag.pix_to_face >= 0).sum()) == 0
    frag = rasterize_meshes(cam, v, torch.zeros((0, 3), dtype=torch.int32, device="cuda"))
    assert int((frag.pix_to_face >= 0).sum()) == 0 and float(frag.zbuf.abs().sum()) == 0.0
