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
