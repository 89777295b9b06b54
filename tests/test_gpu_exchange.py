"""View-batched per-Gaussian backward and the screen-space gradient
exchange (GPU, one device).

gs_preprocess_backward_views over V views must equal the sum of V
single-view backward passes (gs_preprocess_backward through the fused
render); ScreenGradientExchange on one rank must give the ordinary
backward's gradients.  Float sums in another order: 1e-5 relative L2.
"""

import numpy as np
import pytest
import torch

from mlx3d_b200 import _native as nat
from mlx3d_b200.cameras import Camera
from mlx3d_b200.distributed import ScreenGradientExchange
from mlx3d_b200.scenes import _eye_from_angles, make_scene
from mlx3d_b200.splatting import GaussianModel
from mlx3d_b200.splatting import render as R
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _model(n=30_000, aa=True):
    sc = make_scene(1, n=n)
    model = GaussianModel({k: v.clone().requires_grad_(True) for k, v in sc.torch_params(device="cuda").items()},
                          sh_degree=3)
    model.active_sh_degree = 3
    cams = [Camera.look_at(eye=_eye_from_angles(4.0, 30.0 + 50.0 * v, 20.0 - 10 * v), fov=60.0, width=320,
                           height=200) for v in range(3)]
    return model, cams, aa


def _view_loss(model, cam, aa, v):
    out = model.render(cam, antialias=aa)
    g = torch.Generator(device="cuda").manual_seed(v)
    w = torch.rand(out["image"].shape, device="cuda", generator=g)
    return (out["image"] * w).sum() + 0.3 * out["alpha"].sum()


def test_view_batched_backward_equals_sum_of_single_view_backwards():
    model, cams, aa = _model()
    names = list(model.params)
    for p in model.params.values():
        p.grad = None
    for v, cam in enumerate(cams):
        _view_loss(model, cam, aa, v).backward()
    ref = {k: model.params[k].grad.clone() for k in names}

    captured = []
    R.set_screen_grad_hook(lambda cfg, cot, params: captured.append((cfg, cot, params)))
    try:
        for p in model.params.values():
            p.grad = None
        for v, cam in enumerate(cams):
            _view_loss(model, cam, aa, v).backward()
    finally:
        R.set_screen_grad_hook(None)
    assert all(p.grad is None for p in model.params.values())  # the hook took over
    cfg0, _, params = captured[0]
    means, quats, scales, opac, sh_a, sh_b = params
    n = means.shape[0]
    g_screen = torch.stack([torch.cat([c[0], c[1], c[2], c[3].reshape(-1, 1)], 1) for _, c, _ in captured])
    cams_dev = torch.frombuffer(bytearray(b"".join(bytes(c.cam) for c, _, _ in captured)),
                                dtype=torch.uint8).cuda()
    out = {k: torch.empty_like(t) for k, t in zip(("means", "quats", "scales", "opacities", "sh_a", "sh_b"),
                                                   params)}
    dc, dcs, rest, rests = R._sh_layout(cfg0, sh_a, sh_b)
    nat.call("gs_preprocess_backward_views", cams_dev.data_ptr(), len(cams), nat.ptr(means), nat.ptr(quats),
             nat.ptr(scales), nat.ptr(opac), dc, dcs, rest, rests, cfg0.sh_degree, n, cfg0.blur,
             int(cfg0.antialias), cfg0.flags, g_screen.data_ptr(), n * 9, nat.ptr(out["means"]),
             nat.ptr(out["quats"]), nat.ptr(out["scales"]), nat.ptr(out["opacities"]), nat.ptr(out["sh_a"]),
             nat.ptr(out["sh_b"]), nat.stream())
    torch.cuda.synchronize()
    pairs = {"means": "means", "quats": "quats", "scales": "scales", "opacities": "opacities", "sh_dc": "sh_a",
             "sh_rest": "sh_b"}
    for k in names:
        err = rel_l2(out[pairs[k]].cpu().numpy(), ref[k].cpu().numpy())
        assert err < TOL, (k, err)


def test_exchange_on_one_rank_equals_ordinary_backward():
    model, cams, aa = _model(n=20_000, aa=False)
    for p in model.params.values():
        p.grad = None
    _view_loss(model, cams[1], aa, 5).backward()
    ref = {k: p.grad.clone() for k, p in model.params.items()}
    for p in model.params.values():
        p.grad = None
    ex = ScreenGradientExchange()
    with ex.capture():
        _view_loss(model, cams[1], aa, 5).backward()
    got = ex.reduce()
    torch.cuda.synchronize()
    assert got["range"] == (0, 20_000)
    for k, gk in (("means", "means"), ("quats", "quats"), ("scales", "scales"), ("opacities", "opacities"),
                  ("sh_dc", "sh_a"), ("sh_rest", "sh_b")):
        err = rel_l2(got[gk].cpu().numpy(), ref[k].cpu().numpy())
        assert err < TOL, (k, err)


def test_peer_exchange_on_one_rank_equals_ordinary_backward():
    """The peer-memory variant (compositor backward writing into a CUDA IPC
    buffer, the view-batched backward reading it through a pointer table)
    on one rank: same gradients as the ordinary backward."""
    from mlx3d_b200.distributed import PeerScreenExchange

    model, cams, aa = _model(n=20_000, aa=True)
    for p in model.params.values():
        p.grad = None
    _view_loss(model, cams[2], aa, 9).backward()
    ref = {k: p.grad.clone() for k, p in model.params.items()}
    for p in model.params.values():
        p.grad = None
    ex = PeerScreenExchange()
    ex.prepare(20_000, "cuda")
    try:
        for _ in range(3):  # both buffer slots, then the first again
            with ex.capture():
                _view_loss(model, cams[2], aa, 9).backward()
            got = ex.reduce()
            torch.cuda.synchronize()
            for k, gk in (("means", "means"), ("quats", "quats"), ("scales", "scales"), ("opacities", "opacities"),
                          ("sh_dc", "sh_a"), ("sh_rest", "sh_b")):
                err = rel_l2(got[gk].cpu().numpy(), ref[k].cpu().numpy())
                assert err < TOL, (k, err)
    finally:
        ex.close()
