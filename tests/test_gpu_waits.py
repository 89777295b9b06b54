"""Bounded device waits of the binning report an error instead of hanging.

The radix passes and the offsets scan of gs_bin_begin / gs_bin_end wait for
earlier blocks (decoupled look-back); each wait is bounded.  With the poll
limit set to 0 (gs_set_wait_limit, a test hook) every look-back that has to
wait gives up at once, so these tests exercise the failure path without
stalling the GPU: nothing here spins longer than a normal binning does.

Checked: gs_bin_status returns GS_ERR_TIMEOUT with the failing stages'
bits, gs_wait_failures counted the give-ups, every tile range is the empty
[0, 0) (so a compositor reads no stale ids), the public bin_gaussians raises
RuntimeError, and after the limit is restored the same inputs bin exactly as
the oracle does (the sort these waits implement: tiles.py:166-182).
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle.oracle as orc
from mlx3d_b200 import _native as nat
from mlx3d_b200 import splatting as gs
from mlx3d_b200.scenes import make_scene

pytestmark = pytest.mark.gpu

DEFAULT_LIMIT = 1 << 22


@pytest.fixture
def zero_wait_limit():
    lib = nat.load()
    nat.call("gs_set_wait_limit", 0)
    try:
        yield lib
    finally:
        nat.call("gs_set_wait_limit", DEFAULT_LIMIT)


def _c0_projection():
    sc = make_scene(0)
    cam = sc.cameras[0]
    p = sc.torch_params(device="cuda")
    proj = gs.project_gaussians(cam, p["means"], p["quats"], torch.exp(p["scales"]))
    return cam, proj


def _raw_binning(lib, cam, proj):
    """gs_tile_counts + gs_bin_total + gs_bin_begin + gs_bin_end through the C ABI."""
    n = proj["means2d"].shape[0]
    s = torch.cuda.current_stream().cuda_stream
    W, H = cam.width, cam.height
    tiles = ((W + 15) // 16) * ((H + 15) // 16)
    counts = torch.empty((n,), dtype=torch.int32, device="cuda")
    nat.call("gs_tile_counts", proj["means2d"].data_ptr(), proj["radii"].data_ptr(), n, W, H, counts.data_ptr(), s)
    tot = torch.zeros((2,), dtype=torch.int64, device="cuda")
    nat.call("gs_bin_total", counts.data_ptr(), n, tot.data_ptr(), s)
    d = int(tot[0].item())
    ws_n = torch.empty((lib.gs_bin_workspace_n_bytes(n),), dtype=torch.uint8, device="cuda")
    ws_d = torch.empty((lib.gs_bin_workspace_d_bytes(d),), dtype=torch.uint8, device="cuda")
    ids = torch.full((d,), -1, dtype=torch.int32, device="cuda")
    ranges = torch.full((tiles, 2), -5, dtype=torch.int32, device="cuda")
    nat.call("gs_bin_begin", proj["depths"].data_ptr(), counts.data_ptr(), n, ws_n.data_ptr(), ws_n.numel(),
             tot[1:].data_ptr(), s)
    nat.call("gs_bin_end", proj["means2d"].data_ptr(), proj["radii"].data_ptr(), n, d, W, H, ws_n.data_ptr(),
             ws_n.numel(), ws_d.data_ptr(), ws_d.numel(), ids.data_ptr(), ranges.data_ptr(), s)
    st = ctypes.c_uint32(0)
    status = lib.gs_bin_status(ws_n.data_ptr(), ws_n.numel(), n, ctypes.byref(st), s)
    return status, st.value, ids, ranges, d


def test_timed_out_wait_reports_error_and_empties_ranges(zero_wait_limit):
    lib = zero_wait_limit
    cam, proj = _c0_projection()
    cnt = ctypes.c_uint64(0)
    nat.call("gs_wait_failures", ctypes.byref(cnt), 1)  # reset
    status, bits, ids, ranges, d = _raw_binning(lib, cam, proj)
    torch.cuda.synchronize()
    assert d > 0
    assert status == nat.GS_ERR_TIMEOUT, lib.gs_last_error()
    assert bits & 1, bits  # the depth sort of C0 has several partitions: its look-backs gave up
    assert b"gave up" in lib.gs_last_error()
    nat.call("gs_wait_failures", ctypes.byref(cnt), 1)
    assert cnt.value > 0
    assert (ranges.cpu().numpy() == 0).all()
    # the public API raises instead of returning the empty binning
    with pytest.raises(RuntimeError, match="gave up"):
        gs.bin_gaussians(proj["means2d"], proj["radii"], proj["depths"], cam.width, cam.height)
    nat.call("gs_wait_failures", ctypes.byref(cnt), 1)


def test_binning_is_exact_again_after_the_limit_is_restored():
    lib = nat.load()
    cam, proj = _c0_projection()
    cnt = ctypes.c_uint64(0)
    nat.call("gs_wait_failures", ctypes.byref(cnt), 1)
    status, bits, ids, ranges, d = _raw_binning(lib, cam, proj)
    assert status == nat.GS_OK and bits == 0
    counts, rids, rranges, _, _ = orc.bin_gaussians(proj["means2d"].cpu().numpy(), proj["radii"].cpu().numpy(),
                                                    proj["depths"].cpu().numpy(), cam.width, cam.height)
    np.testing.assert_array_equal(ids.cpu().numpy(), rids)
    np.testing.assert_array_equal(ranges.cpu().numpy(), rranges)
    nat.call("gs_wait_failures", ctypes.byref(cnt), 0)
    assert cnt.value == 0


def test_render_path_raises_on_the_next_frame(zero_wait_limit):
    """The fused render copies the binning status to the host without
    waiting; the next binning on this thread raises it."""
    sc = make_scene(0)
    model = gs.GaussianModel({k: v.clone() for k, v in sc.torch_params().items()}, sh_degree=3)
    model.active_sh_degree = 0
    cam = sc.cameras[0]
    out = model.render(cam)
    torch.cuda.synchronize()
    # nothing was composited: every tile range is empty
    assert float(out["final_T"].min()) == 1.0
    nat.call("gs_set_wait_limit", DEFAULT_LIMIT)
    with pytest.raises(RuntimeError, match="gave up"):
        model.render(cam)
    out = model.render(cam)  # the status was consumed; this frame is fine
    assert float(out["final_T"].min()) < 1.0
    cnt = ctypes.c_uint64(0)
    nat.call("gs_wait_failures", ctypes.byref(cnt), 1)
