"""3DGS PLY checkpoints (model.py:338-392; the reference's test_model_ply_roundtrip,
tests/test_splatting.py:545-556), on the host."""

import numpy as np
import torch

from mlx3d_b200.ply import _read_vertices
from mlx3d_b200.scenes import make_scene
from mlx3d_b200.splatting import GaussianModel


def test_ply_roundtrip_and_layout(tmp_path):
    sc = make_scene(1, n=500)
    model = GaussianModel({k: torch.from_numpy(v) for k, v in sc.params.items()}, sh_degree=3)
    path = str(tmp_path / "g.ply")
    model.save_ply(path)
    v = _read_vertices(path)
    names = list(v.dtype.names)
    assert names[:9] == ["x", "y", "z", "nx", "ny", "nz", "f_dc_0", "f_dc_1", "f_dc_2"]
    assert names[9:54] == [f"f_rest_{i}" for i in range(45)]
    assert names[54:] == ["opacity", "scale_0", "scale_1", "scale_2", "rot_0", "rot_1", "rot_2", "rot_3"]
    # f_rest is channel-major: f_rest_i = sh_rest[:, i % 15, i // 15]
    np.testing.assert_array_equal(v["f_rest_16"], sc.params["sh_rest"][:, 1, 1])
    loaded = GaussianModel.load_ply(path, device="cpu")
    assert loaded.sh_degree == 3 and loaded.active_sh_degree == 3
    for k, a in sc.params.items():
        np.testing.assert_array_equal(loaded.params[k].numpy(), a.reshape(loaded.params[k].shape))


def test_ply_infers_sh_degree_and_reads_ascii(tmp_path):
    sc = make_scene(0, n=20)  # SH degree 0
    model = GaussianModel({k: torch.from_numpy(v) for k, v in sc.params.items()}, sh_degree=0)
    path = str(tmp_path / "g0.ply")
    model.save_ply(path)
    loaded = GaussianModel.load_ply(path, sh_degree=3, device="cpu")
    assert loaded.sh_degree == 0 and loaded.params["sh_rest"].shape == (20, 0, 3)
    # the same data as an ascii PLY
    v = _read_vertices(path)
    names = v.dtype.names
    apath = str(tmp_path / "a.ply")
    with open(apath, "w") as f:
        f.write("ply\nformat ascii 1.0\ncomment test\nelement vertex 20\n")
        f.writelines(f"property float {k}\n" for k in names)
        f.write("end_header\n")
        for row in v:
            f.write(" ".join(repr(float(x)) for x in row) + "\n")
    la = GaussianModel.load_ply(apath, device="cpu")
    for k in sc.params:
        np.testing.assert_array_equal(la.params[k].numpy(), loaded.params[k].numpy())
