"""CPU restatement of the hard mesh rasterizer (oracle.mesh_rasterize),
pinned to the reference's behaviours (tests/test_rasterizer.py:20-57) and
to a brute-force z-buffer over all triangles.  Binning uses the oracle's
tiler on the triangles' bounding circles, as rasterizer.py:140-147 does."""

import numpy as np
import torch

import oracle.oracle as orc
from oracle import torch_ref
from mlx3d_b200.cameras import Camera
from tests.helpers import ico_sphere


def _binned(cam, verts, faces):
    xy = torch_ref.project_points(cam, torch.tensor(verts)).numpy()
    z = torch.tensor(verts) @ cam.R.T + cam.t
    z = z[:, 2].numpy()
    tri_xy, tri_z = xy[faces], z[faces]
    cen = tri_xy.mean(axis=1)
    rad = np.sqrt(((tri_xy - cen[:, None, :]) ** 2).sum(-1).max(axis=1))
    dep = tri_z.mean(axis=1)
    _, ids, ranges, _, _ = orc.bin_gaussians(cen, rad, dep, cam.width, cam.height)
    return tri_xy.astype(np.float32), tri_z.astype(np.float32), ids, ranges


def _tri():
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), fov=60.0, width=32, height=32)
    verts = np.array([[-0.6, -0.5, 0.0], [0.6, -0.5, 0.0], [0.0, 0.6, 0.0]], np.float32)
    return cam, verts, np.array([[0, 1, 2]], np.int32)


def test_triangle_hit_and_miss():
    cam, v, f = _tri()
    p2f, zb = orc.mesh_rasterize(*_binned(cam, v, f), cam.width, cam.height, cam.znear)
    assert p2f[16, 16] == 0 and p2f[0, 0] == -1
    assert zb[0, 0] == 0.0 and abs(zb[16, 16] - 3.0) < 1e-5


def test_near_face_wins():
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), fov=60.0, width=16, height=16)
    v = np.array([[-0.6, -0.5, 0.5], [0.6, -0.5, 0.5], [0.0, 0.6, 0.5],
                  [-0.6, -0.5, -0.5], [0.6, -0.5, -0.5], [0.0, 0.6, -0.5]], np.float32)
    f = np.array([[0, 1, 2], [3, 4, 5]], np.int32)
    p2f, _ = orc.mesh_rasterize(*_binned(cam, v, f), cam.width, cam.height, cam.znear)
    assert p2f[8, 8] == 1


def test_tiled_equals_brute_force_on_a_sphere():
    """Every pixel's nearest triangle from the tile lists equals the nearest
    over all triangles (ties are measure-zero here)."""
    v, f = ico_sphere(2, 1.0)
    cam = Camera.look_at(eye=(2.2, 1.6, 2.2), at=(0, 0, 0), fov=45.0, width=72, height=56)
    tri_xy, tri_z, ids, ranges = _binned(cam, v, f)
    p2f, zb = orc.mesh_rasterize(tri_xy, tri_z, ids, ranges, cam.width, cam.height, cam.znear)
    # brute force with the same per-triangle arithmetic: one "tile" holding every face
    h, w = cam.height, cam.width
    all_ids = np.arange(f.shape[0], dtype=np.int32)
    tx, ty = (w + 15) // 16, (h + 15) // 16
    full = np.tile(np.array([[0, f.shape[0]]], np.int32), (tx * ty, 1))
    ref, zref = orc.mesh_rasterize(tri_xy, tri_z, np.tile(all_ids, 1), full, w, h, cam.znear)
    assert (p2f >= 0).mean() > 0.2
    np.testing.assert_array_equal(p2f, ref)
    np.testing.assert_array_equal(zb, zref)
