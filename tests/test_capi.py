"""The C-ABI library: loads without a GPU, exports every symbol declared in
include/*.h, and rejects bad arguments before touching the device."""

import ctypes
import re
from pathlib import Path

import pytest

from mlx3d_b200 import _native as nat

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(gs_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = nat.load()
    declared = _declared_symbols()
    assert len(declared) >= 15
    for name in declared:
        assert hasattr(lib, name), name
    # the Python binding covers all of them too
    assert set(declared) <= set(nat.exported_symbols())


def test_version_and_error_channel():
    lib = nat.load()
    assert lib.gs_version() >= 100
    assert isinstance(lib.gs_last_error(), bytes)


def test_invalid_arguments_are_rejected_without_device_work():
    lib = nat.load()
    # NULL camera
    st = lib.gs_project_forward(None, None, None, None, 4, 0.3, 0, None, None, None, None, None, None)
    assert st == nat.GS_ERR_INVALID_ARG
    assert b"camera" in lib.gs_last_error()
    cam = nat.GsCamera()
    cam.width, cam.height = 0, 10
    st = lib.gs_project_forward(ctypes.byref(cam), None, None, None, 4, 0.3, 0, None, None, None, None, None, None)
    assert st == nat.GS_ERR_INVALID_ARG
    # tiles_x that does not match the image
    st = lib.gs_rasterize_forward(None, None, None, 3, None, None, None, None, None, 32, 32, 3, 2, None, None, None,
                                  None, None)
    assert st == nat.GS_ERR_INVALID_ARG
    assert b"tiles_x" in lib.gs_last_error()
    # a too-small binning workspace is a capacity error
    d = ctypes.c_int64()
    st = lib.gs_bin_begin(None, None, 1000, None, 0, ctypes.addressof(d), None)
    assert st == nat.GS_ERR_CAPACITY
    # duplicate count beyond int32
    st = lib.gs_bin_end(None, None, 10, 1 << 31, 16, 16, None, 0, None, 0, None, None, None)
    assert st == nat.GS_ERR_CAPACITY
    # SH degree out of range
    st = lib.gs_eval_sh_forward(4, None, 1, 16, 3, None, None, None)
    assert st == nat.GS_ERR_INVALID_ARG


def test_call_maps_status_to_exceptions():
    with pytest.raises(ValueError, match="degree"):
        nat.call("gs_eval_sh_forward", 5, None, 1, 16, 3, None, None, None)


def test_workspace_sizes_grow_with_inputs():
    lib = nat.load()
    sizes = [lib.gs_bin_workspace_n_bytes(n) for n in (0, 1, 1000, 10**6, 6 * 10**6)]
    assert sizes == sorted(sizes) and sizes[-1] >= 5 * 4 * 6 * 10**6
    dsz = [lib.gs_bin_workspace_d_bytes(d) for d in (0, 1, 10**7)]
    assert dsz == sorted(dsz) and dsz[-1] >= 16 * 10**7
