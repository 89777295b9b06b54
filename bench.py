#!/usr/bin/env python
"""Benchmark of the splatting hot path on B200.

Workload (benchmark config C2, the configuration the headline metric is
quoted on): 1,000,000 Gaussians, SH degree 3, 1920x1080, fov 50, antialias on.  One
step = GaussianModel.render(camera) forward (fused preprocess, binning,
compositing) + L1 loss against a U(0,1) target + backward to every raw
parameter (means, quats, log-scales, opacity logits, sh_dc, sh_rest).
Under torchrun with N ranks each rank renders its own view of the same
scene (weak scaling) and the per-Gaussian gradients (59 floats each) are
summed over ranks with one NCCL all-reduce, launched under the next view's
backward (the step has no optimizer; --sync-allreduce waits every step).

Prints one JSON line (rank 0).  `value` is whole-job milliseconds per frame:
the max-over-ranks step time divided by the frames (views) the job rendered
per step.  `--impl reference` times the CPU oracle (a restatement of the
reference's algorithm; mlx3D itself needs Apple's MLX/Metal) instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fwd+bwd ms/frame @1080p 1M Gaussians SH3; views/s at 1/2/4/8 B200"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=2, help="scene config (2 = the headline workload)")
    ap.add_argument("--n", type=int, default=None, help="override the Gaussian count (profiling runs)")
    ap.add_argument("--views", type=int, default=None, help="override the view count (configs 3 and 4)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-inputs", choices=["target", "all"], default="target",
                    help="what the e2e measurement copies from the host every step")
    ap.add_argument("--rank-views", choices=["same", "ring"], default="same",
                    help="multi-GPU C2: every rank renders the C2 camera (identical per-GPU work), or rank r "
                         "renders azimuth 30 + 45 r (views of unequal cost)")
    ap.add_argument("--no-multiview", action="store_true",
                    help="skip the C4 render and C3 training measurements that follow the C2 headline")
    ap.add_argument("--mv-steps", type=int, default=2, help="timed steps of each multi-view measurement")
    ap.add_argument("--streams", type=int, default=2, help="CUDA streams the C4 views are pipelined over")
    ap.add_argument("--sync-allreduce", action="store_true",
                    help="multi-GPU C2: every step waits for its own gradient exchange (no overlap)")
    ap.add_argument("--exchange", choices=["peer", "screen", "allreduce"], default="peer",
                    help="multi-GPU C2: screen-space cotangents read from the other GPUs' memory by the "
                         "view-batched per-Gaussian backward (peer), or exchanged by an NCCL all-to-all first "
                         "(screen); both leave the summed gradient reduce-scattered.  Or an all-reduce of the "
                         "parameter gradients (allreduce)")
    return ap.parse_args()


# --------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event (throttle) reasons every 10 ms through
    NVML while the timed region runs (read-only queries)."""

    # NVML clocks-event reason bits
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.sm: list[float] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self.stop = threading.Event()
        self.thread = None
        self.nv = None

    def __enter__(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[self.gpu]) if vis else self.gpu
            self.h = nv.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
            self.nv = nv
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception:  # no NVML: clocks stay unreported
            self.nv = None
        return self

    def _sample(self):
        nv = self.nv
        self.sm.append(float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)))
        try:
            bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except AttributeError:
            bits = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
        for b, name in self.REASONS.items():
            if bits & b:
                self.reasons.add(name)

    def _run(self):
        self._sample()
        while not self.stop.wait(0.01):
            self._sample()

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=2)
            self._sample()

    def summary(self) -> dict:
        sm = self.sm
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(sm)}


# ------------------------------------------------------------ distributed glue
def dist_setup(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = "nccl" if args.impl == "ours" else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo")
    elif torch.cuda.is_available() and args.impl == "ours":
        torch.cuda.set_device(local)
    return world, rank, local


def view_camera(scene, rank: int):
    """Rank r renders the scene from azimuth 30 + 45 r degrees (rank 0 is the
    config's own camera)."""
    from mlx3d_b200.cameras import Camera
    from mlx3d_b200.scenes import _eye_from_angles

    cfg = scene.config
    if rank == 0:
        return scene.cameras[0]
    radius = float(scene.cameras[0].camera_center.norm())
    eye = _eye_from_angles(radius, 30.0 + 45.0 * rank, 20.0)
    return Camera.look_at(eye=eye, fov=cfg.fov, width=cfg.width, height=cfg.height)


# ---------------------------------------------------------------- our arm
# Algorithmic bytes per unit of each entry point: the bytes the entry point
# must read and write once (inputs, outputs, and the passes its algorithm
# needs), counted from the array sizes.
def stage_bytes(stage: str, n: int, d: int, pixels: int, sh_rest_floats: int) -> float:
    sh = 4 * (3 + sh_rest_floats)
    if stage == "gs_preprocess_forward":
        return n * (12 + 16 + 12 + 4 + sh) + n * (8 + 12 + 4 + 4 + 4 + 12 + 4 + 4)
    if stage == "gs_preprocess_backward":
        return n * (12 + 16 + 12 + 4 + sh) + n * (8 + 12 + 12 + 4) + n * (12 + 16 + 12 + 4 + sh)
    if stage == "gs_bin_begin":
        # depth keys (read depth+count, write key+val), 4 single-kernel radix
        # passes over N (read key+value, write key+value), scan reading counts
        # through the permutation twice and writing offsets
        return n * 16 + 4 * n * 16 + n * (8 + 8 + 4)
    if stage == "gs_bin_end":
        # duplication (read perm, offset, means2d, radius; write key+value per
        # duplicate), two single-kernel tile-sort passes over D, ranges (read keys)
        return n * 20 + d * 8 + 2 * d * 16 + d * 4
    if stage == "gs_rasterize_forward":
        return d * 40 + pixels * 20
    if stage == "gs_rasterize_backward":
        return d * 40 + pixels * 24 + n * 36
    return 0.0


def run_ours(args, world, rank, local):
    import numpy as np
    import torch
    import torch.distributed as dist

    from mlx3d_b200 import _native as nat
    from mlx3d_b200.scenes import make_scene
    from mlx3d_b200.splatting import GaussianModel

    dev = torch.device("cuda", local)
    scene = make_scene(args.config, n=args.n)
    cfg = scene.config
    cam = view_camera(scene, rank if args.rank_views == "ring" else 0)
    params = scene.torch_params(device=dev, requires_grad=True)
    model = GaussianModel(params, sh_degree=3)
    model.active_sh_degree = cfg.sh_degree
    target = scene.target(view=rank, device=dev)

    from mlx3d_b200.distributed import GradientReducer, allreduce_gradients
    from mlx3d_b200.losses import l1_loss

    # Multi-GPU: the step has no optimizer, so nothing reads the summed
    # gradient before the next view is rendered.  Step k's gradients are
    # staged into a flat buffer at its end; their all-reduce is launched once
    # step k+1's forward is enqueued, so it runs on NCCL's stream under step
    # k+1's backward, and step k+1 waits for it at the end of its backward
    # (GradientReducer, two flat buffers).  The last one is waited for before
    # the timed region closes.  --sync-allreduce makes every step wait for
    # its own all-reduce instead.
    from mlx3d_b200.distributed import PeerScreenExchange, ScreenGradientExchange

    reducer = GradientReducer()
    screen = world > 1 and args.exchange in ("screen", "peer")
    exchange = PeerScreenExchange() if args.exchange == "peer" else ScreenGradientExchange()
    if screen and args.exchange == "peer":
        exchange.prepare(params["means"].shape[0], dev)
    overlap = world > 1 and not screen and not args.sync_allreduce
    # screen exchange: step k's all-to-all runs on NCCL's stream under step
    # k+1's forward; its per-Gaussian backward is launched once step k+1's
    # forward is enqueued (the step has no optimizer, nothing reads the
    # gradient earlier); the last one completes inside the timed region
    screen_overlap = screen and not args.sync_allreduce

    def step(model_=model, target_=target):
        pl = list(model_.params.values())
        for p in pl:
            p.grad = None
        out = model_.render(cam, antialias=cfg.antialias)
        if overlap:
            reducer.launch()
        if screen_overlap:
            while exchange.in_flight():
                exchange.finish()
        loss = l1_loss(out["image"], target_)
        if screen:
            # the gradient ends reduce-scattered: this rank holds the sum over
            # all ranks' views for its slice of the Gaussians
            with exchange.capture():
                loss.backward()
            if screen_overlap:
                exchange.start()
            else:
                exchange.reduce()
            return loss
        if overlap:
            with reducer.sink(pl):  # gradients land in the next flat all-reduce buffer
                loss.backward()
        else:
            loss.backward()
        if overlap:
            while reducer.in_flight():
                reducer.finish()
            reducer.stage(pl)
        elif world > 1:
            allreduce_gradients(pl)
        return loss

    def drain():
        while reducer.in_flight():
            reducer.finish()
        while exchange.in_flight():
            exchange.finish()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        step()
    drain()
    torch.cuda.synchronize()
    lib = nat.load()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # The clock sampler starts (NVML set-up takes a while, and differs per
    # process) before the barrier, so every rank records its start event
    # right after the same barrier.
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        launches0 = lib.gs_kernel_launch_count()
        start.record()
        for _ in range(args.steps):
            step()
        drain()
        end.record()
        torch.cuda.synchronize()
    barrier()
    launches = lib.gs_kernel_launch_count() - launches0
    ms_step = start.elapsed_time(end) / args.steps
    t = torch.tensor([ms_step], device=dev)
    rank_ms = [ms_step]
    if world > 1:
        every = torch.empty((world,), device=dev)
        dist.all_gather_into_tensor(every, t)
        rank_ms = [round(float(x), 4) for x in every.tolist()]
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item())

    # ---- per-entry-point device time (CUDA events around each library call,
    # on the launching stream), a separate pass after the timed region.
    stage_ms: dict[str, list[float]] = {}
    orig_call = nat.call

    def timed_call(name, *a):
        s = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        orig_call(name, *a)
        e1.record(s)
        stage_ms.setdefault(name, []).append((e0, e1))

    nat.call = timed_call
    try:
        prof_steps = 3
        for _ in range(prof_steps):
            step()
        drain()
        torch.cuda.synchronize()
    finally:
        nat.call = orig_call
    stages = {k: sum(a.elapsed_time(b) for a, b in v) / prof_steps for k, v in stage_ms.items()}
    # this rank's device time inside library calls per step (its compute,
    # without waits for other ranks), gathered for the line
    comp = torch.tensor([sum(stages.values())], device=dev)
    rank_compute = [round(float(comp.item()), 4)]
    if world > 1:
        every = torch.empty((world,), device=dev)
        dist.all_gather_into_tensor(every, comp)
        rank_compute = [round(float(x), 4) for x in every.tolist()]
    with torch.no_grad():
        out = model.render(cam, antialias=cfg.antialias)
        from mlx3d_b200.splatting.tiles import bin_gaussians

        ids, _, _, _ = bin_gaussians(out["means2d"], out["radii"], out["depths"], cam.width, cam.height)
        d = int(ids.shape[0])
        visible = int((out["radii"] > 0).sum().item())
    n = scene.params["means"].shape[0]
    pixels = cam.width * cam.height
    rest = scene.params["sh_rest"].shape[1] * 3
    dom = max(stages, key=stages.get)
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    alg = stage_bytes(dom, n, d, pixels, rest)
    achieved = alg / (stages[dom] * 1e-3) / 1e9
    stage_rows = {
        k: {"ms": round(v, 4), "alg_gb_s": round(stage_bytes(k, n, d, pixels, rest) / (v * 1e-3) / 1e9, 1)}
        for k, v in sorted(stages.items(), key=lambda kv: -kv[1])
    }
    traffic = None
    tf = ROOT / "profiles" / "dram_traffic_c2.json"
    if tf.exists() and cfg.index == 2 and args.n is None:
        traffic = json.loads(tf.read_text()).get(dom)

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        # Every step copies its inputs from pinned host memory and reads the
        # loss back; the copy of step k+1 runs on a copy stream under step k's
        # kernels (HostStager double-buffers the device side).  The inputs of a
        # render + loss + backward step are the camera (kernel arguments) and
        # the target image; the Gaussians are the model, resident in HBM across
        # steps like a network's weights (--e2e-inputs all also re-copies
        # every parameter each step).
        from mlx3d_b200.staging import HostStager

        host = {"target": target.cpu().pin_memory()}
        if args.e2e_inputs == "all":
            host.update({k: v.detach().cpu().pin_memory() for k, v in params.items()})
        loss_host = torch.empty((), dtype=torch.float32).pin_memory()
        stager = HostStager(host, dev, requires_grad=tuple(k for k in params if k in host))
        h2d = stager.h2d_bytes()
        models = []
        for slot in stager.slots:
            if args.e2e_inputs == "all":
                m = GaussianModel({k: slot[k] for k in params}, sh_degree=3)
                m.active_sh_degree = cfg.sh_degree
            else:
                m = model
            models.append(m)

        def e2e_run(k_steps):
            stager.copy_stream.wait_stream(torch.cuda.current_stream())
            stager.prefetch(host)
            for k in range(k_steps):
                if k + 1 < k_steps:
                    stager.prefetch(host)
                i, slot = stager.acquire()
                loss = step(models[i], slot["target"])
                loss_host.copy_(loss.detach(), non_blocking=True)
                stager.release(i)
            drain()

        e2e_run(max(3, args.warmup))
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        e2e_run(args.steps)
        e1.record()
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": round(float(te.item()) / world, 4), "unit": "ms/frame", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": 4,
               "inputs": ("target image copied host->device every step (pinned, double-buffered); the Gaussian "
                          "parameters stay resident in HBM as model state" if args.e2e_inputs == "target" else
                          "target image and all Gaussian parameters copied host->device every step")}

    if isinstance(exchange, PeerScreenExchange):
        exchange.close()  # collective: unmaps the peers' buffers on every rank
    if rank != 0:
        return None
    clk = clocks.summary()
    line = {
        "metric": METRIC,
        "value": round(ms_step / world, 4),
        "unit": "ms/frame",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "views_per_s": round(1000.0 * world / ms_step, 2),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded PCG64 scene of BASELINE config %d)" % cfg.index,
        "config": {
            "workload": f"C{cfg.index}: {n:,} Gaussians, SH{cfg.sh_degree}, {cam.width}x{cam.height}, "
                        f"fov {cfg.fov:g}, antialias={cfg.antialias}; GaussianModel.render + L1 + backward",
            "gaussians": n,
            "width": cam.width,
            "height": cam.height,
            "views_per_step": world,
            "rank_views": ("every rank renders the C2 camera (identical per-GPU work)" if args.rank_views == "same"
                           else "rank r renders azimuth 30 + 45 r (unequal per-view cost)") if world > 1 else None,
            "duplicates": d,
            "visible_gaussians": visible,
            "parallelism": ((f"views sharded over {world} GPU(s); screen-space cotangents (9 floats per "
                             f"Gaussian) "
                             + ("read by each rank's view-batched per-Gaussian backward straight from the other "
                                "GPUs' memory (CUDA IPC mappings, peer loads over NVLink; one 1-float NCCL "
                                "all-reduce per step as the barrier)" if args.exchange == "peer" else
                                "exchanged by one NCCL all-to-all per step, then one view-batched per-Gaussian "
                                "backward per rank")
                             + f" over its 1/{world} of the Gaussians: the summed gradient ends reduce-scattered "
                               f"across ranks")
                            if screen else
                            (f"views sharded over {world} GPU(s); per-Gaussian gradient all-reduce (NCCL, one "
                             f"flat 59-float-per-Gaussian buffer per step, "
                             + ("waited for by the same step)" if args.sync_allreduce else
                                "overlapped with the next step's render; all complete inside the timed region)")))
                           + ("" if not screen else ("; each step's exchange overlaps the next step's forward, the "
                                                     "last completes inside the timed region" if screen_overlap
                                                     else "; each step waits for its own exchange"))
                           if world > 1 else "single GPU",
            "l2": "no flush: per-step working set (parameters %.0f MB + gradients + image buffers) exceeds the "
                  "126 MB L2" % (sum(v.nbytes for v in scene.params.values()) / 1e6),
        },
        "e2e": e2e,
        "gpu_launches": int(launches),
        "clocks": clk,
        "rank_ms_per_step": rank_ms,
        "rank_compute_ms_per_step": rank_compute,
        "stages_ms": stage_rows,
        "roofline": {
            "kernel": dom,
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": hbm_peak,
            "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4),
            "peak_source": peak_src,
            "traffic": traffic,
            "algorithmic_bytes": alg,
        },
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(scene, cam, cfg, steps=1, warmup=1)
    if cam is scene.cameras[0] and (args.n is None or args.n <= 2_000_000):
        # The compositors are FP32-issue bound, not HBM bound.  Their
        # algorithmic work is that of the reference's loops: 21 FLOP per
        # pixel-Gaussian pair its forward loop evaluates, 45 FLOP per pair
        # it composites (backward), counted exactly on this frame by the
        # oracle (forward only, host cores), over the kernels' live
        # CUDA-event times.  Peak: nominal dense FP32, 148 SMs x 128 lanes
        # x 2 FLOP x 1.965 GHz (the measured peaks file has no FP32 figure).
        pairs = getattr(cpu_baseline, "last_pairs", None) if world == 1 and not args.no_cpu_baseline else None
        if pairs is None:
            pairs = oracle_pairs(scene, cam, cfg)
        n_eval, n_comp = pairs
        peak = 148 * 128 * 2 * 1.965e9 / 1e12
        rf = {}
        for k, flops in (("gs_rasterize_forward", 21.0 * n_eval), ("gs_rasterize_backward", 45.0 * n_comp)):
            t = stages.get(k)
            if t:
                ach = flops / (t * 1e-3) / 1e12
                rf[k] = {"achieved": round(ach, 2), "peak": round(peak, 1), "unit": "TFLOP/s",
                         "frac": round(ach / peak, 4), "peak_source": "nominal", "flops": flops}
        line["roofline_fp32"] = dict(rf, pairs_evaluated=n_eval, pairs_composited=n_comp)
        if dom in rf:
            hbm = line["roofline"]
            line["roofline"] = dict(rf[dom], kernel=dom, bound="fp32_issue", traffic=traffic,
                                    algorithmic_bytes=alg, hbm_achieved_gbs=hbm["achieved"], hbm_peak_gbs=hbm_peak,
                                    hbm_frac=hbm["frac"], hbm_peak_source=peak_src)
    return line


# ------------------------------------------------------- CPU oracle baseline
def _oracle_frame(scene, cam, cfg, threads=0):
    import numpy as np

    import oracle.oracle as orc

    p = scene.params
    s, o = orc.activate(p["scales"], p["opacities"])
    sh = np.concatenate([p["sh_dc"], p["sh_rest"]], axis=1)
    fwd = orc.render(cam.to_native(), cam.width, cam.height, p["means"], p["quats"], s, o, sh=sh,
                     sh_degree=cfg.sh_degree, antialias=cfg.antialias, threads=threads)
    target = scene.target(view=0, device="cpu").numpy()
    g_img = (np.sign(fwd["image"] - target) / fwd["image"].size).astype(np.float32)
    orc.render_grads(cam, p["means"], p["quats"], s, o, sh=sh, sh_degree=cfg.sh_degree, antialias=cfg.antialias,
                     grad_image=g_img, threads=threads, fwd=fwd)
    return fwd


def oracle_pairs(scene, cam, cfg):
    """(pairs evaluated, pairs composited) of the reference's forward loop on
    this frame, counted by the oracle's forward (host cores)."""
    import numpy as np

    import oracle.oracle as orc

    p = scene.params
    s, o = orc.activate(p["scales"], p["opacities"])
    sh = np.concatenate([p["sh_dc"], p["sh_rest"]], axis=1)
    fwd = orc.render(cam.to_native(), cam.width, cam.height, p["means"], p["quats"], s, o, sh=sh,
                     sh_degree=cfg.sh_degree, antialias=cfg.antialias)
    return fwd["pairs_evaluated"], fwd["pairs_composited"]


def cpu_baseline(scene, cam, cfg, steps=1, warmup=0):
    import torch

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    for _ in range(warmup):
        _oracle_frame(scene, cam, cfg)
    t0 = time.perf_counter()
    for _ in range(steps):
        fwd = _oracle_frame(scene, cam, cfg)
    ms = (time.perf_counter() - t0) * 1000.0 / steps
    cpu_baseline.last_pairs = (fwd["pairs_evaluated"], fwd["pairs_composited"])
    return {"value": round(ms, 1), "unit": "ms/frame", "cores": cores, "kind": "port",
            "sample": f"{steps} full frame(s) after {warmup} warm-up frame(s) of the same workload: C++ oracle (OpenMP, {cores} threads) for "
                      "projection, SH, binning and both compositors; torch float64 autograd (CPU) for the "
                      "per-Gaussian backward"}


def run_reference(args, world, rank):
    if rank != 0:
        return None
    from mlx3d_b200.scenes import make_scene

    scene = make_scene(args.config, n=args.n)
    cam = scene.cameras[0]
    cfg = scene.config
    steps = max(1, min(args.steps, 3))
    warm = min(args.warmup, 1)
    for _ in range(warm):
        _oracle_frame(scene, cam, cfg)
    cb = cpu_baseline(scene, cam, cfg, steps=steps, warmup=0)
    cb["sample"] += f"; {steps} timed step(s) of the {args.steps} requested (each a full frame), {warm} warm-up"
    n = scene.params["means"].shape[0]
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": cb["value"],
        "unit": "ms/frame",
        "n_gpus": world,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": cb["value"],
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded PCG64 scene of BASELINE config %d)" % cfg.index,
        "config": {"workload": f"C{cfg.index}: {n:,} Gaussians, SH{cfg.sh_degree}, {cam.width}x{cam.height}; "
                               "render + L1 + backward on the CPU oracle (mlx3D needs Apple MLX/Metal, which "
                               "cannot run here)"},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "ms/frame", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------- multi-view configurations
def run_multiview(args, world, rank, local, config=None, steps=None, warmup=None, views=None):
    """C3 (data-parallel training step: every rank renders its shard of the 64
    views, L1 + D-SSIM, gradient all-reduce, one Adam update) or C4 (render
    only, with depth: every rank renders its shard of the 256 views).  Strong
    scaling: the view batch is fixed, ranks split it.  Metric: views/s."""
    config = args.config if config is None else config
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    views = args.views if views is None else views
    import torch
    import torch.distributed as dist

    from mlx3d_b200 import _native as nat
    from mlx3d_b200.distributed import shard_views
    from mlx3d_b200.scenes import make_scene
    from mlx3d_b200.splatting import GaussianModel, GaussianTrainer, TrainerConfig

    dev = torch.device("cuda", local)
    scene = make_scene(config, n=args.n if config == args.config else None, views=views)
    cfg = scene.config
    idx = shard_views(list(range(len(scene.cameras))), rank, world)
    cams = [scene.cameras[i] for i in idx]
    params = scene.torch_params(device=dev)
    model = GaussianModel(params, sh_degree=3)
    model.active_sh_degree = cfg.sh_degree
    dups = []
    if cfg.index == 3:
        targets = [scene.target(i, device=dev) for i in idx]
        trainer = GaussianTrainer(model, TrainerConfig(antialias=cfg.antialias, densify_from=10**9,
                                                       opacity_reset_every=10**9, sh_increase_every=10**9))

        def step():
            trainer.step_views(cams, targets, total_views=len(scene.cameras))
    else:
        # views pipelined over two CUDA streams (GaussianModel.render_views);
        # every output is produced on the device and dropped
        def step():
            model.render_views(cams, antialias=cfg.antialias, render_depth=True, streams=args.streams,
                               on_output=lambda i, out: dups.append(out["n_duplicates"]))

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dups.clear()
    lib = nat.load()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:  # started before the barrier (see run_ours)
        barrier()
        torch.cuda.synchronize()
        l0 = lib.gs_kernel_launch_count()
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    barrier()
    launches = lib.gs_kernel_launch_count() - l0
    t = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
    keys = torch.tensor([float(sum(dups)) / max(steps, 1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(keys)
    ms = float(t.item())
    views = len(scene.cameras)
    if rank != 0:
        return None
    n = scene.params["means"].shape[0]
    what = "training step (L1 + D-SSIM, all-reduce, Adam)" if cfg.index == 3 else "render + depth, forward only"
    line = {
        "metric": f"C{cfg.index} views/s ({what})",
        "value": round(1000.0 * views / ms, 2),
        "unit": "views/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded PCG64 scene of BASELINE config %d)" % cfg.index,
        "config": {"workload": f"C{cfg.index}: {n:,} Gaussians, SH{cfg.sh_degree}, {views} views "
                               f"{cfg.width}x{cfg.height}, fov {cfg.fov:g}, antialias={cfg.antialias}; {what}",
                   "views_per_step": views, "parallelism": f"views sharded over {world} GPU(s)",
                   "l2": "no flush: per-step working set exceeds the 126 MB L2"},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
    }
    if cfg.index == 4:
        line["sort_keys_per_s"] = round(float(keys.item()) / (ms * 1e-3), 1)
    return line


def main():
    args = parse_args()
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        line = run_reference(args, world, rank)
    elif args.config in (3, 4):
        line = run_multiview(args, world, rank, local)
    else:
        line = run_ours(args, world, rank, local)
        if not args.no_multiview and args.n is None:
            # The north star's scaling targets are quoted on C4 (256-view 4K
            # render with depth) and C3 (64-view training step): measured at
            # the same N right after the headline, full views and resolution,
            # fewer timed steps (each step is a whole view batch).
            import torch

            torch.cuda.empty_cache()
            mv = {}
            for c in (4, 3):
                r = run_multiview(args, world, rank, local, config=c, steps=max(1, args.mv_steps),
                                  warmup=3, views=None)
                torch.cuda.empty_cache()
                if r is not None:
                    mv[f"C{c}"] = {k: r[k] for k in ("metric", "value", "unit", "ms_per_step", "steps", "warmup",
                                                     "higher_is_better", "scaling", "config", "gpu_launches",
                                                     "clocks", "sort_keys_per_s") if k in r}
            if line is not None:
                line["multiview"] = mv
    if line is not None:
        print(json.dumps(line), flush=True)
    import torch.distributed as dist

    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
