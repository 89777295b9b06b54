"""gs_bin_gaussians_static: binning for callers that cannot allocate.

Applications that embed this renderer but do not own the GPU's memory (the
memory belongs to a host engine or a fixed-pool allocator) cannot hand the
library a freshly allocated workspace.  The static entry point takes its
scratch space from a fixed 20 MiB device array inside the library instead.
This test calls it through the C ABI twice in a row, on two different
scenes (so the second call runs on the first call's leftover scratch), and
checks that its sorted ids and tile ranges equal those of the ordinary,
workspace-taking entry points (binning is integer work: exact equality).
"""

import ctypes

import numpy as np
import pytest
import torch

from mlx3d_b200 import _native as nat
from mlx3d_b200 import splatting as gs
from mlx3d_b200.scenes import make_scene

pytestmark = pytest.mark.gpu


def _projected(index, n):
    sc = make_scene(index, n=n)
    cam = sc.cameras[0]
    p = sc.torch_params(device="cuda")
    proj = gs.project_gaussians(cam, p["means"], p["quats"], torch.exp(p["scales"]))
    return cam, proj


def _static_bin(proj, width, height, capacity):
    lib = nat.load()
    n = proj["means2d"].shape[0]
    tiles = ((width + 15) // 16) * ((height + 15) // 16)
    ids = torch.full((capacity,), -7, dtype=torch.int32, device="cuda")
    ranges = torch.full((tiles, 2), -7, dtype=torch.int32, device="cuda")
    d = ctypes.c_int64(-1)
    status = lib.gs_bin_gaussians_static(
        proj["means2d"].data_ptr(), proj["radii"].data_ptr(), proj["depths"].data_ptr(), n, width, height, capacity,
        ids.data_ptr(), ranges.data_ptr(), ctypes.byref(d), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return status, d.value, ids, ranges


def _wait_failures(reset):
    cnt = ctypes.c_uint64(0)
    nat.call("gs_wait_failures", ctypes.byref(cnt), int(reset))
    return cnt.value


def test_static_binning_matches_workspace_binning_on_two_calls():
    _wait_failures(reset=True)
    for index, n in ((1, 100_000), (0, 10_000)):
        cam, proj = _projected(index, n)
        ref_ids, ref_ranges, _, _ = gs.bin_gaussians(proj["means2d"], proj["radii"], proj["depths"], cam.width,
                                                     cam.height)
        d_ref = ref_ids.shape[0]
        assert d_ref > 0
        status, d, ids, ranges = _static_bin(proj, cam.width, cam.height, capacity=d_ref + 17)
        assert status == nat.GS_OK, nat.load().gs_last_error()
        assert d == d_ref
        np.testing.assert_array_equal(ids[:d].cpu().numpy(), ref_ids.cpu().numpy())
        np.testing.assert_array_equal(ranges.cpu().numpy(), ref_ranges.cpu().numpy())
        assert (ids[d:].cpu().numpy() == -7).all()  # nothing written past D
    # no look-back of the sorts gave up (a give-up could leave partial output)
    assert _wait_failures(reset=False) == 0


def test_static_binning_of_no_gaussians():
    tiles = 4 * 3
    ranges = torch.full((tiles, 2), -7, dtype=torch.int32, device="cuda")
    d = ctypes.c_int64(-1)
    status = nat.load().gs_bin_gaussians_static(None, None, None, 0, 64, 48, 0, None, ranges.data_ptr(),
                                                 ctypes.byref(d), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert status == nat.GS_OK and d.value == 0
    assert (ranges.cpu().numpy() == 0).all()


def test_static_binning_rejects_sizes_beyond_its_limits():
    cam, proj = _projected(0, 10_000)
    d_ref = gs.bin_gaussians(proj["means2d"], proj["radii"], proj["depths"], cam.width, cam.height)[0].shape[0]
    status, d, _, _ = _static_bin(proj, cam.width, cam.height, capacity=d_ref - 1)
    assert status == nat.GS_ERR_CAPACITY and d == d_ref
    assert b"needed" in nat.load().gs_last_error()
    # more duplicates than the static limit: every Gaussian made 40x wider
    wide = dict(proj, radii=proj["radii"] * 40.0)
    status, d, _, _ = _static_bin(wide, cam.width, cam.height, capacity=1)
    assert status == nat.GS_ERR_CAPACITY and d > 1048576, (status, d)
    assert b"static limit" in nat.load().gs_last_error()
    lib = nat.load()
    big = 131072 + 1
    dd = ctypes.c_int64()
    status = lib.gs_bin_gaussians_static(None, None, None, big, 64, 64, 0, None, None, ctypes.byref(dd), None)
    assert status == nat.GS_ERR_CAPACITY
    assert b"static limit" in lib.gs_last_error()
