"""Unscented projection on the GPU vs the oracle (forward) and vs autograd of
the restated reference (backward), for all four camera models; rendering
and training with projection="ut" (tests/test_splatting.py:425-437)."""

import numpy as np
import pytest
import torch

import oracle.oracle as orc
from oracle import torch_ref
from mlx3d_b200 import splatting as gs
from mlx3d_b200.cameras import Camera
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu


def _cam(lens):
    base = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), fov=60.0, width=160, height=120)
    kw = dict(R=base.R, t=base.t, fx=base.fx, fy=base.fy, cx=base.cx, cy=base.cy, width=160, height=120)
    if lens == "pinhole":
        return base
    if lens == "brown":
        return Camera(**kw, distortion=(-0.2, 0.05, 0.001, -0.002, 0.01))
    if lens == "fisheye":
        return Camera(**kw, distortion=(0.05, -0.01, 0.002, 0.0), fisheye=True)
    kw.update(fx=50.0, fy=50.0)
    return Camera(**kw, orthographic=True)


def _inputs(n=3000, seed=0):
    rng = np.random.default_rng(seed)
    means = (rng.normal(size=(n, 3)) * 0.5).astype(np.float32)
    quats = rng.normal(size=(n, 4)).astype(np.float32)
    scales = np.exp(rng.normal(size=(n, 3)) * 0.3 - 3).astype(np.float32)
    return means, quats, scales


@pytest.mark.parametrize("lens", ["pinhole", "brown", "fisheye", "ortho"])
def test_ut_forward_matches_oracle(lens):
    cam = _cam(lens)
    means, quats, scales = _inputs()
    out = gs.project_gaussians_ut(cam, *(torch.tensor(a, device="cuda") for a in (means, quats, scales)),
                                  antialias=True)
    ref = orc.project_ut(cam, means, quats, scales, antialias=True)
    for k in ("means2d", "conics", "depths", "radii", "compensation"):
        got = out[k].cpu().numpy()
        if lens == "fisheye":  # arctan of the device and host libm may differ by an ulp
            np.testing.assert_allclose(got, ref[k], rtol=1e-5, atol=1e-5, err_msg=k)
        else:
            np.testing.assert_array_equal(got, ref[k], err_msg=k)


@pytest.mark.parametrize("lens", ["pinhole", "brown", "fisheye", "ortho"])
def test_ut_backward_matches_autodiff(lens):
    cam = _cam(lens)
    means, quats, scales = _inputs(2000, 1)
    rng = np.random.default_rng(5)
    n = means.shape[0]
    cots = {"means2d": rng.normal(size=(n, 2)), "conics": rng.normal(size=(n, 3)), "depths": rng.normal(size=n),
            "compensation": rng.normal(size=n)}
    m, q, s = (torch.tensor(a, device="cuda", requires_grad=True) for a in (means, quats, scales))
    out = gs.project_gaussians_ut(cam, m, q, s, antialias=True)
    keys = list(cots)
    torch.autograd.backward([out[k] for k in keys], [torch.tensor(cots[k], device="cuda", dtype=torch.float32)
                                                     for k in keys])
    tm, tq, ts = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (means, quats, scales))
    ref = torch_ref.project_ut(cam, tm, tq, ts, antialias=True)
    torch.autograd.backward([ref[k] for k in keys], [torch.tensor(cots[k]) for k in keys])
    for name, a, b in (("means", m, tm), ("quats", q, tq), ("scales", s, ts)):
        assert rel_l2(a.grad.cpu().numpy(), b.grad.numpy()) < 1e-4, name


def test_render_and_trainer_support_ut_projection():
    torch.manual_seed(16)
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), width=24, height=24, fov=60.0)
    model = gs.GaussianModel.from_points((torch.randn(18, 3) * 0.25).cuda(), sh_degree=0)
    out = model.render(cam, projection="ut")
    assert out["image"].shape == (24, 24, 3) and not torch.isnan(out["image"]).any()
    with pytest.raises(ValueError, match="projection"):
        model.render(cam, projection="bad")
    with pytest.raises(ValueError, match="projection"):
        gs.GaussianTrainer(model, gs.TrainerConfig(projection="bad"))
    target = torch.rand(24, 24, 3, device="cuda")
    trainer = gs.GaussianTrainer(model, gs.TrainerConfig(projection="ut", densify_from=10_000))
    info = trainer.step(cam, target)
    assert np.isfinite(info["loss"])
