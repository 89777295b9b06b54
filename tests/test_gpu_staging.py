"""Double-buffered host-to-device staging: every acquired slot holds exactly
the host data prefetched for it, in order, while compute runs on the other."""

import pytest
import torch

from mlx3d_b200.staging import HostStager

pytestmark = pytest.mark.gpu


def test_stager_delivers_each_steps_inputs_in_order():
    n_steps = 6
    hosts = [{"a": torch.full((1 << 20,), float(k)).pin_memory(),
              "b": torch.arange(1000, dtype=torch.int32).add(k).pin_memory()} for k in range(n_steps)]
    st = HostStager(hosts[0], "cuda")
    seen = []
    st.copy_stream.wait_stream(torch.cuda.current_stream())
    st.prefetch(hosts[0])
    for k in range(n_steps):
        if k + 1 < n_steps:
            st.prefetch(hosts[k + 1])
        i, slot = st.acquire()
        torch.cuda._sleep(2_000_000)  # keep the compute stream busy while the next copy lands
        seen.append((float(slot["a"].sum()) / slot["a"].numel(), int(slot["b"][0])))
        st.release(i)
    torch.cuda.synchronize()
    assert seen == [(float(k), k) for k in range(n_steps)]
    assert st.h2d_bytes() == (1 << 20) * 4 + 1000 * 4


def test_stager_rejects_pageable_host_memory_and_overfill():
    st = HostStager({"a": torch.zeros(8)}, "cuda")
    with pytest.raises(ValueError):
        st.prefetch({"a": torch.zeros(8)})
    h = {"a": torch.zeros(8).pin_memory()}
    st.prefetch(h)
    st.prefetch(h)
    with pytest.raises(RuntimeError):
        st.prefetch(h)


def test_gradient_sink_writes_render_gradients_into_the_reducer_buffer():
    from mlx3d_b200.distributed import GradientReducer
    from mlx3d_b200.scenes import make_scene
    from mlx3d_b200.splatting import GaussianModel

    sc = make_scene(1, n=5000)
    cam = sc.cameras[0]
    target = sc.target(0)

    def grads(use_sink):
        params = sc.torch_params(requires_grad=True)
        model = GaussianModel(params, sh_degree=3)
        model.active_sh_degree = 3
        red = GradientReducer()
        out = model.render(cam)
        loss = (out["image"] - target).abs().mean()
        if use_sink:
            with red.sink(params):
                loss.backward()
        else:
            loss.backward()
        ptrs = {k: p.grad.data_ptr() for k, p in params.items()}
        grads_ = {k: p.grad.clone() for k, p in params.items()}
        red.stage(params)
        flat = red.finish()
        return params, flat, ptrs, grads_

    p1, f1, ptr1, g1 = grads(True)
    p2, f2, ptr2, g2 = grads(False)
    torch.cuda.synchronize()
    # with the sink every gradient was a view of the reducer's flat buffer ...
    lo, hi = f1.data_ptr(), f1.data_ptr() + f1.numel() * 4
    assert all(lo <= v < hi for v in ptr1.values())
    # ... and stage() detached those views from the parameters (the buffer is
    # reduced in place next); copied gradients stay attached
    assert all(p.grad is None for p in p1.values())
    assert all(p.grad is not None for p in p2.values())
    # (atomic accumulation order differs between two backward passes)
    assert float((f1 - f2).norm() / f2.norm()) < 1e-5
    for k in p1:
        assert float((g1[k] - g2[k]).norm() / g2[k].norm().clamp_min(1e-30)) < 1e-5, k
