"""View sharding and the gradient all-reduce with two gloo ranks on CPU."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mlx3d_b200.distributed import allreduce_gradients, shard_views


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world_size, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world_size)
    try:
        views = list(range(7))
        mine = shard_views(views)
        params = {"means": torch.zeros(5, 3, requires_grad=True), "opacities": torch.zeros(5, requires_grad=True),
                  "unused": torch.zeros(2, requires_grad=True)}
        # each rank's gradient: the sum over its views of view-dependent values
        params["means"].grad = torch.stack([torch.full((3,), float(v)) for v in range(5)]) * sum(mine)
        params["opacities"].grad = torch.ones(5) * (rank + 1)
        allreduce_gradients(params)
        results[rank] = (mine, params["means"].grad.clone(), params["opacities"].grad.clone(),
                         params["unused"].grad.clone())
    finally:
        dist.destroy_process_group()


def test_two_rank_view_sharding_and_gradient_sum():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        r0, r1 = results[0], results[1]
    assert r0[0] == [0, 2, 4, 6] and r1[0] == [1, 3, 5]
    total = sum(range(7))
    expect = torch.stack([torch.full((3,), float(v)) for v in range(5)]) * total
    for r in (r0, r1):
        torch.testing.assert_close(r[1], expect)
        torch.testing.assert_close(r[2], torch.full((5,), 3.0))
        torch.testing.assert_close(r[3], torch.zeros(2))


def test_shard_views_validates_rank():
    assert shard_views([1, 2, 3], 0, 1) == [1, 2, 3]
    with pytest.raises(ValueError):
        shard_views([1], 2, 2)


def _reducer_worker(rank, world_size, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world_size)
    try:
        from mlx3d_b200.distributed import GradientReducer

        red = GradientReducer()
        params = [torch.zeros(4, requires_grad=True), torch.zeros(2, 3, requires_grad=True)]
        sums = []
        for step in range(5):  # two reductions in flight at most, finished in order
            params[0].grad = torch.full((4,), float(10 * step + rank))
            params[1].grad = torch.full((2, 3), float(step * (rank + 1)))
            if red.in_flight() == 2:
                sums.append(red.finish().clone())
            if step % 2:
                red.start(params)
            else:  # staged only: launched by the next launch() or finish()
                red.stage(params)
                if step == 2:
                    red.launch()
        while red.in_flight():
            sums.append(red.finish().clone())
        results[rank] = sums
    finally:
        dist.destroy_process_group()


def test_two_rank_pipelined_gradient_reducer():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_reducer_worker, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        for r in (0, 1):
            sums = results[r]
            assert len(sums) == 5
            for step, s in enumerate(sums):
                expect = torch.cat([torch.full((4,), float(20 * step + 1)), torch.full((6,), float(3 * step))])
                torch.testing.assert_close(s, expect)


def test_gradient_sink_hands_out_views_of_the_next_flat_buffer():
    """GradientReducer.sink routes the fused render's gradient allocations
    (render._grad_like) into the buffer the next stage() fills; stage() then
    copies nothing for them (CPU tensors, world size 1)."""
    from mlx3d_b200.distributed import GradientReducer
    from mlx3d_b200.splatting import render as R

    params = {"means": torch.randn(5, 3), "opacities": torch.randn(5)}
    red = GradientReducer()
    with red.sink(params):
        gm = R._grad_like("means", params["means"])
        go = R._grad_like("opacities", params["opacities"], zero=True)
        other = R._grad_like("means", torch.randn(5, 3))  # not a parameter: a fresh tensor
    assert R._grad_sink is None  # uninstalled on exit
    gm.copy_(torch.full((5, 3), 2.0))
    params["means"].grad, params["opacities"].grad = gm, go
    red.stage(params)
    flat = red.finish()
    assert gm.data_ptr() == flat.data_ptr() and go.data_ptr() == flat.data_ptr() + 15 * 4
    assert other.data_ptr() != flat.data_ptr()
    torch.testing.assert_close(flat, torch.cat([torch.full((15,), 2.0), torch.zeros(5)]))


def _leaving_worker(rank, world_size, port, mode, results):
    """Rank 1 takes part in step 0, then leaves (announced, or by exiting);
    rank 0 must get PeerLost before step 1's collective, not hang in it."""
    import time as _time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world_size)
    from mlx3d_b200.distributed import PeerLost, PeerMonitor

    mon = PeerMonitor(timeout=1.0)
    params = {"means": torch.zeros(3, requires_grad=True)}
    params["means"].grad = torch.ones(3)
    mon.beat(0)
    allreduce_gradients(params)
    if rank == 1:
        if mode == "leave":
            mon.leave()
        results[rank] = "left"
        # between steps, nothing in flight; wait until rank 0 reported (the
        # store lives in rank 0's process), then exit without cleanup
        deadline = _time.monotonic() + 60
        while 0 not in results.keys() and _time.monotonic() < deadline:
            _time.sleep(0.05)
        os._exit(0)
    t0 = _time.monotonic()
    try:
        mon.beat(1)
        allreduce_gradients(params)
        results[rank] = ("no error", float(params["means"].grad[0]))
    except PeerLost as e:
        results[rank] = ("PeerLost", e.rank, str(e), _time.monotonic() - t0)
    os._exit(0)


@pytest.mark.parametrize("mode", ["leave", "exit"])
def test_survivor_learns_that_a_rank_left_between_steps(mode):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, mode, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        r0 = results[0]
    assert r0[0] == "PeerLost" and r0[1] == 1, r0
    if mode == "leave":
        assert "left before step 1" in r0[2] and r0[3] < 1.0
    else:
        assert "no heartbeat" in r0[2] and r0[3] < 10.0


def test_peer_monitor_single_rank_and_store_failure():
    from mlx3d_b200.distributed import PeerLost, PeerMonitor

    class BrokenStore:
        def set(self, k, v):
            raise ConnectionError("closed")

    store = dist.HashStore()
    PeerMonitor(store=store, rank=0, world_size=1).beat(0)  # alone: returns at once
    lone = PeerMonitor(store=store, rank=0, world_size=2, timeout=0.05)
    with pytest.raises(PeerLost, match="no heartbeat"):
        lone.beat(1)
    with pytest.raises(PeerLost, match="unreachable"):
        PeerMonitor(store=BrokenStore(), rank=0, world_size=2, timeout=0.1).beat(0)


def _exchange_worker(rank, world_size, port, results):
    """ScreenGradientExchange host logic on gloo ranks (CPU): padding, the
    all-to-all of the 9-float cotangent rows, the camera all-gather and the
    slice handed to the view-batched backward (the kernel call itself is
    recorded instead of run: there is no GPU here)."""
    import types

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world_size)
    try:
        from mlx3d_b200 import _native as nat
        from mlx3d_b200.distributed import ScreenGradientExchange

        n = 7  # not a multiple of the world size: the last slice is shorter
        cam = nat.GsCamera()
        cam.fx = float(rank + 1)
        cfg = types.SimpleNamespace(cam=cam, sh_mode="split", sh_degree=1, blur=0.3, antialias=False, flags=3)
        means, quats, scales = torch.zeros(n, 3), torch.zeros(n, 4), torch.zeros(n, 3)
        opac, sh_dc, sh_rest = torch.zeros(n), torch.zeros(n, 1, 3), torch.zeros(n, 3, 3)
        # cotangent row i of rank r: [100 r + i, ...] so every received row names its origin
        base = (100.0 * rank + torch.arange(n, dtype=torch.float32)).reshape(n, 1)
        cot = (base.repeat(1, 2), base.repeat(1, 3) + 0.1, base.repeat(1, 3) + 0.2, base[:, 0] + 0.3)
        calls = []
        nat.call = lambda name, *a: calls.append((name, a))
        nat.stream = lambda: None
        ex = ScreenGradientExchange()
        ex._captured = (cfg, cot, (means, quats, scales, opac, sh_dc, sh_rest))
        out = ex.reduce()
        name, a = calls[0]
        lo, hi = out["range"]
        recv = ex._slots[0][1].clone()
        results[rank] = (name, lo, hi, a[1], recv.tolist(), a[11], a[16])
    finally:
        dist.destroy_process_group()


def test_two_rank_screen_gradient_exchange_routes_rows_by_slice():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        res = {r: results[r] for r in (0, 1)}
    per = 4  # ceil(7 / 2)
    for r in (0, 1):
        name, lo, hi, n_views, recv, n_slice, view_stride = res[r]
        assert name == "gs_preprocess_backward_views" and n_views == 2
        assert (lo, hi) == ((0, 4) if r == 0 else (4, 7)) and n_slice == hi - lo and view_stride == per * 9
        for v in (0, 1):  # view v's block holds rank v's rows of this slice, padded with zeros
            for k in range(per):
                row = recv[v][k]
                i = lo + k
                if i < 7:
                    assert row[0] == 100.0 * v + i and abs(row[2] - (100.0 * v + i + 0.1)) < 1e-4
                    assert abs(row[8] - (100.0 * v + i + 0.3)) < 1e-4
                else:
                    assert row == [0.0] * 9
