"""Training-step pieces on the GPU: fused L1 + D-SSIM loss and gradient,
multi-tensor Adam, and the trainer's schedule / convergence behaviour
(the reference's test_trainer_* tests in tests/test_splatting.py:652-699)."""

import numpy as np
import pytest
import torch

from oracle import torch_ref
from mlx3d_b200 import _native as nat
from mlx3d_b200 import losses
from mlx3d_b200 import splatting as gs
from mlx3d_b200.cameras import Camera
from mlx3d_b200.scenes import make_scene
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(37, 53, 3), (64, 64, 1), (1080, 1920, 3)])
def test_l1_dssim_loss_and_gradient_match_autodiff(shape):
    rng = np.random.default_rng(shape[0])
    pred = rng.uniform(size=shape).astype(np.float32)
    target = np.clip(pred + rng.normal(0, 0.1, size=shape), 0, 1).astype(np.float32)
    p = torch.tensor(pred, device="cuda", requires_grad=True)
    loss, l1, s = losses.l1_dssim_loss(p, torch.tensor(target, device="cuda"), 0.2)
    loss.backward()
    tp = torch.tensor(pred, dtype=torch.float64, requires_grad=True)
    tt = torch.tensor(target, dtype=torch.float64)
    ref_ssim = torch_ref.ssim(tp, tt)
    ref = 0.8 * (tp - tt).abs().mean() + 0.2 * (1.0 - ref_ssim)
    ref.backward()
    assert abs(float(s) - float(ref_ssim)) < 1e-5
    assert abs(float(loss) - float(ref)) < 1e-5
    assert rel_l2(p.grad.cpu().numpy(), tp.grad.numpy()) < 1e-4


@pytest.mark.parametrize("n", [1, 1000, 1080 * 1920 * 3])
def test_l1_loss_and_gradient_match_torch(n):
    rng = np.random.default_rng(n)
    pred = rng.uniform(size=n).astype(np.float32)
    target = rng.uniform(size=n).astype(np.float32)
    target[: n // 7] = pred[: n // 7]  # ties: zero subgradient
    p = torch.tensor(pred, device="cuda", requires_grad=True)
    loss = losses.l1_loss(p, torch.tensor(target, device="cuda"))
    (3.0 * loss).backward()
    tp = torch.tensor(pred, dtype=torch.float64, requires_grad=True)
    ref = (tp - torch.tensor(target, dtype=torch.float64)).abs().mean()
    (3.0 * ref).backward()
    assert abs(float(loss) - float(ref)) <= 1e-6 * max(1.0, abs(float(ref)))
    np.testing.assert_allclose(p.grad.cpu().numpy(), tp.grad.numpy(), rtol=1e-6, atol=0)
    # deterministic: same bits on a second evaluation
    assert float(losses.l1_loss(p, torch.tensor(target, device="cuda"))) == float(loss)


def test_l1_dssim_gradient_of_each_output_term():
    rng = np.random.default_rng(5)
    pred = rng.uniform(size=(40, 50, 3)).astype(np.float32)
    target = rng.uniform(size=(40, 50, 3)).astype(np.float32)
    p = torch.tensor(pred, device="cuda", requires_grad=True)
    loss, l1, s = losses.l1_dssim_loss(p, torch.tensor(target, device="cuda"), 0.3)
    (2.0 * loss + 0.5 * l1 - 1.5 * s).backward()
    tp = torch.tensor(pred, dtype=torch.float64, requires_grad=True)
    tt = torch.tensor(target, dtype=torch.float64)
    rs = torch_ref.ssim(tp, tt)
    rl1 = (tp - tt).abs().mean()
    (2.0 * (0.7 * rl1 + 0.3 * (1.0 - rs)) + 0.5 * rl1 - 1.5 * rs).backward()
    assert rel_l2(p.grad.cpu().numpy(), tp.grad.numpy()) < 1e-4


def test_ssim_of_identical_images_is_one_and_gradient_flows():
    x = torch.rand(32, 48, 3, device="cuda", requires_grad=True)
    s = losses.ssim(x, x.detach())
    assert abs(float(s) - 1.0) < 1e-5
    s.backward()
    assert torch.isfinite(x.grad).all()


def test_adam_step_is_bit_exact_against_restatement():
    rng = np.random.default_rng(1)
    sizes, lrs = [1000, 7, 4099], [1e-2, 5e-3, 1.6e-4]
    host = [dict(p=rng.normal(size=n).astype(np.float32), g=rng.normal(size=n).astype(np.float32),
                 m=np.zeros(n, np.float32), v=np.zeros(n, np.float32)) for n in sizes]
    dev = [{k: torch.tensor(v, device="cuda") for k, v in h.items()} for h in host]
    for step in (1, 2, 3):
        groups = (nat.GsAdamGroup * 3)()
        for i, (d, lr) in enumerate(zip(dev, lrs)):
            groups[i] = nat.GsAdamGroup(d["p"].data_ptr(), d["g"].data_ptr(), d["m"].data_ptr(), d["v"].data_ptr(),
                                        d["p"].numel(), lr)
        nat.call("gs_adam_step", groups, 3, 0.9, 0.999, 1e-15, 0, step, nat.stream())
        for h, lr in zip(host, lrs):
            h["p"], h["m"], h["v"] = torch_ref.adam_update(h["p"], h["g"], h["m"], h["v"], lr)
    torch.cuda.synchronize()
    for h, d in zip(host, dev):
        for k in ("p", "m", "v"):
            np.testing.assert_array_equal(d[k].cpu().numpy(), h[k])


def _model(n, seed, sh_degree=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    pts = (torch.randn(n, 3, generator=g) * 0.4).cuda()
    cols = torch.rand(n, 3, generator=g).cuda()
    return gs.GaussianModel.from_points(pts, cols, sh_degree=sh_degree)


def test_trainer_position_lr_decays():
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), width=24, height=24, fov=60.0)
    target = torch.rand(24, 24, 3, device="cuda")
    trainer = gs.GaussianTrainer(
        _model(20, 7),
        gs.TrainerConfig(lr_means=1e-2, lr_means_final=1e-4, lr_means_max_steps=2, densify_from=10_000,
                         sh_increase_every=10_000),
        scene_extent=2.0,
    )
    lr0 = trainer.learning_rates()["means"]
    info1, info2, info3 = (trainer.step(cam, target) for _ in range(3))
    assert abs(lr0 - 2e-2) < 1e-6
    assert abs(info1["lr_means"] - lr0) < 1e-8
    assert info3["lr_means"] < info2["lr_means"] < info1["lr_means"]
    assert abs(info3["lr_means"] - 2e-4) < 1e-7


def test_trainer_converges_single_view_and_tracks_screen_gradients():
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), width=48, height=48, fov=60.0)
    with torch.no_grad():
        target = _model(30, 3).render(cam)["image"].detach()
    model = _model(60, 4)
    trainer = gs.GaussianTrainer(model, gs.TrainerConfig(densify_from=1))
    losses_ = [trainer.step(cam, target)["loss"] for _ in range(60)]
    assert losses_[-1] < losses_[0] * 0.6, (losses_[0], losses_[-1])
    assert trainer.grad_accum.shape == (60,) and float(trainer.grad_count.max()) > 0
    assert float(trainer.grad_accum.sum()) > 0


def test_data_parallel_step_on_one_rank_equals_summed_views():
    """step_views over two views == the mean of the two single-view losses'
    gradients, applied once (no process group: world size 1)."""
    sc = make_scene(0, n=2000)
    cams = [sc.cameras[0], Camera.look_at(eye=(1.0, 0.5, -3.5), width=256, height=256, fov=60.0)]
    tgts = [sc.target(0), sc.target(1)]
    m1 = gs.GaussianModel(sc.torch_params(), sh_degree=0)
    m2 = gs.GaussianModel(sc.torch_params(), sh_degree=0)
    t1 = gs.GaussianTrainer(m1, gs.TrainerConfig(densify_from=10_000))
    info = t1.step_views(cams, tgts)
    assert info["views"] == 2 and np.isfinite(info["loss"])
    # manual: average the two views' losses, one Adam update
    for p in m2.params.values():
        p.requires_grad_(True)
    total = 0
    for cam, tgt in zip(cams, tgts):
        out = m2.render(cam)
        total = total + losses.l1_dssim_loss(out["image"], tgt)[0] / 2
    total.backward()
    t2 = gs.GaussianTrainer(m2, gs.TrainerConfig(densify_from=10_000))  # keeps the gradients
    t2._adam()
    for k in m1.params:
        assert rel_l2(m1.params[k].detach().cpu().numpy(), m2.params[k].detach().cpu().numpy()) < 1e-6, k


def test_trainer_densification_runs():
    """trainer.py:366-400 through GaussianTrainer.step (tests/test_splatting.py:705-717)."""
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), width=32, height=32)
    target = torch.rand(32, 32, 3, device="cuda")
    model = _model(40, 4)
    trainer = gs.GaussianTrainer(model, gs.TrainerConfig(densify_from=2, densify_every=5,
                                                         densify_grad_threshold=1e-9))
    events = []
    for _ in range(12):
        info = trainer.step(cam, target)
        if info["densify"] is not None:
            events.append(info["densify"])
    assert np.isfinite(info["loss"])
    assert len(events) == 2 and events[0]["cloned"] + events[0]["split"] > 0
    n = model.num_gaussians
    assert info["num_gaussians"] == n
    assert trainer.grad_accum.shape == (n,) and trainer.grad_count.shape == (n,)
    for k in ("means", "scales", "quats", "opacities", "sh_dc", "sh_rest"):
        assert trainer._m[k].shape == model.params[k].shape == trainer._v[k].shape
        assert model.params[k].is_cuda and model.params[k].requires_grad


def test_trainer_preserves_moments_after_densify_resize():
    """trainer.py:139-159 (tests/test_splatting.py:720-751)."""
    model = _model(8, 8)
    trainer = gs.GaussianTrainer(model, gs.TrainerConfig(densify_from=10_000))
    old_m = torch.arange(24, dtype=torch.float32, device="cuda").reshape(8, 3)
    trainer._m["means"] = old_m.clone()
    trainer._v["means"] = old_m + 100.0
    keep = torch.tensor([1, 3, 6], device="cuda")
    model.select(keep)
    model.append({k: torch.zeros((2, *v.shape[1:]), device="cuda") for k, v in model.params.items()})
    trainer._resize_moments(keep, 2)
    zeros = torch.zeros(2, 3, device="cuda")
    assert torch.equal(trainer._m["means"], torch.cat([old_m[keep], zeros]))
    assert torch.equal(trainer._v["means"], torch.cat([old_m[keep] + 100.0, zeros]))
    assert trainer._m["opacities"].shape == (5,)


def test_trainer_mcmc_relocation_keeps_count_and_resets_moments():
    """trainer.py:366-377 (tests/test_splatting.py:754-781)."""
    cam = Camera.look_at(eye=(0, 0, -3.0), at=(0, 0, 0), width=32, height=32)
    target = torch.rand(32, 32, 3, device="cuda")
    model = _model(40, 13)
    n0 = model.num_gaussians
    cfg = gs.TrainerConfig(method="mcmc", densify_from=1, densify_every=2, densify_grad_threshold=1e-9,
                           mcmc_relocate_frac=0.25, mcmc_min_opacity=0.2, mcmc_jitter_scale=0.0,
                           mcmc_noise_scale=0.0)
    trainer = gs.GaussianTrainer(model, cfg)
    event = None
    for _ in range(3):
        info = trainer.step(cam, target)
        if info["densify"] is not None:
            event = info["densify"]
    assert model.num_gaussians == n0
    assert event is not None and event["relocated"] > 0
    assert torch.isfinite(trainer._m["means"]).all()


def test_chunked_adam_equals_one_launch():
    """The multi-GPU step updates the parameters chunk by chunk as the
    all-reduce pieces arrive (chunks cut across parameter tensors); the result
    must be bit-identical to one launch over all parameters."""
    from mlx3d_b200.distributed import GradientReducer

    sc = make_scene(1, n=3001)

    def trainer():
        m = gs.GaussianModel({k: v.clone() for k, v in sc.torch_params(device="cuda").items()}, sh_degree=3)
        return gs.GaussianTrainer(m, gs.TrainerConfig())

    t1, t2 = trainer(), trainer()
    g = torch.Generator(device="cuda").manual_seed(4)
    for step in range(2):
        grads = {k: torch.randn(p.shape, device="cuda", generator=g) for k, p in t1.model.params.items()}
        for k, p in t1.model.params.items():
            p.grad = grads[k].clone()
        t1._adam()
        plist = [t2.model.params[k] for k in ("means", "scales", "quats", "opacities", "sh_dc", "sh_rest")]
        for k, p in t2.model.params.items():
            p.grad = grads[k].clone()
        red = GradientReducer()
        red.stage(plist)
        flat, chunks = red.launch_chunks(5)
        assert len(chunks) == 5 and chunks[-1][1] == flat.numel()
        t2._adam_chunked(flat, chunks)
        torch.cuda.synchronize()
        for k in t1.model.params:
            assert torch.equal(t1.model.params[k], t2.model.params[k]), k
            assert torch.equal(t1._m[k], t2._m[k]) and torch.equal(t1._v[k], t2._v[k]), k
