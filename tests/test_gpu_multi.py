"""Multi-GPU exchange paths (GPU, needs 2 devices; skipped otherwise).

Two ranks (one process per GPU, NCCL) each render their own view of the
same Gaussians; the summed gradient each rank holds for its slice must be
the same with the peer-memory exchange, the NCCL all-to-all exchange and a
plain all-reduce of the parameter gradients (1e-5 relative L2: float sums
in different orders).
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs 2 GPUs")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, results):
    import torch.distributed as dist

    from mlx3d_b200.cameras import Camera
    from mlx3d_b200.distributed import (PeerScreenExchange, ScreenGradientExchange, allreduce_gradients,
                                        world)
    from mlx3d_b200.scenes import _eye_from_angles, make_scene
    from mlx3d_b200.splatting import GaussianModel
    from tests.helpers import rel_l2

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=torch.device("cuda", rank))
    try:
        sc = make_scene(1, n=30_001)  # odd count: the slices differ in length
        model = GaussianModel({k: v.clone().requires_grad_(True)
                               for k, v in sc.torch_params(device="cuda").items()}, sh_degree=3)
        model.active_sh_degree = 3
        cam = Camera.look_at(eye=_eye_from_angles(4.0, 30.0 + 70.0 * rank, 15.0), fov=60.0, width=320, height=200)

        def loss():
            out = model.render(cam, antialias=True)
            return (out["image"] * (0.5 + rank)).sum()

        for p in model.params.values():
            p.grad = None
        loss().backward()
        allreduce_gradients(model.params)
        ref = {k: p.grad.clone() for k, p in model.params.items()}
        errs = {}
        for name, ex in (("screen", ScreenGradientExchange()), ("peer", PeerScreenExchange())):
            if name == "peer":
                ex.prepare(30_001, "cuda")
            for p in model.params.values():
                p.grad = None
            for _ in range(2):
                with ex.capture():
                    loss().backward()
                got = ex.reduce()
            lo, hi = got["range"]
            for k, gk in (("means", "means"), ("quats", "quats"), ("scales", "scales"),
                          ("opacities", "opacities"), ("sh_dc", "sh_a"), ("sh_rest", "sh_b")):
                errs[(name, k)] = rel_l2(got[gk].cpu().numpy(), ref[k][lo:hi].cpu().numpy())
            if name == "peer":
                ex.close()
        results[rank] = errs
    finally:
        dist.destroy_process_group()


@needs_two
def test_two_gpu_exchanges_match_allreduce():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
            assert p.exitcode == 0
        for r in (0, 1):
            for key, err in results[r].items():
                assert err < 1e-5, (r, key, err)


def _trainer_worker(rank, port, results):
    import torch.distributed as dist

    from mlx3d_b200.distributed import shard_views
    from mlx3d_b200.scenes import make_scene
    from mlx3d_b200.splatting import GaussianModel, GaussianTrainer, TrainerConfig
    from tests.helpers import rel_l2

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=torch.device("cuda", rank))
    try:
        sc = make_scene(3, n=40_000, views=5)
        cams = sc.cameras
        targets = [sc.target(i, device="cuda") for i in range(len(cams))]

        def trainer():
            m = GaussianModel({k: v.clone() for k, v in sc.torch_params(device="cuda").items()}, sh_degree=3)
            m.active_sh_degree = 3
            t = GaussianTrainer(m, TrainerConfig(densify_from=10**9))
            seen = {}

            def record(flat, chunks):  # the summed gradient, instead of the update
                for _, _, w in chunks:
                    if w is not None:
                        w.wait()
                off = 0
                for k in ("means", "scales", "quats", "opacities", "sh_dc", "sh_rest"):
                    n = m.params[k].numel()
                    seen[k] = flat[off:off + n].view_as(m.params[k]).clone()
                    off += n

            t._adam_chunked = record
            return t, seen

        tr, got = trainer()
        mine = shard_views(list(range(len(cams))), rank, 2)
        tr.step_views([cams[i] for i in mine], [targets[i] for i in mine], total_views=len(cams))
        ref, _ = trainer()
        ref._views_backward(cams, targets, 1.0 / len(cams), 2)  # all views on this rank, no collective
        results[rank] = {k: rel_l2(got[k].cpu().numpy(), p.grad.cpu().numpy()) for k, p in ref.model.params.items()}
    finally:
        dist.destroy_process_group()


@needs_two
def test_two_gpu_training_step_gradients_equal_all_views_on_one_gpu():
    """GaussianTrainer.step_views on 2 ranks (gradients written straight into
    the flat all-reduce buffer, all-reduced over NCCL) equals the gradient of
    all views accumulated on one GPU."""
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_trainer_worker, args=(r, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
            assert p.exitcode == 0
        for r in (0, 1):
            for k, err in results[r].items():
                assert err < 1e-5, (r, k, err)
