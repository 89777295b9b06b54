"""ctypes binding of the sm_100a C-ABI library ``_lib/libgsplat_b200.so``.

Every product entry point of this package goes through this module; there is
no CPU or PyTorch fallback.  Loading fails loudly when the library has not
been built (``python -m mlx3d_b200.build``), and every call checks that its
tensors are CUDA float32 / int32 and contiguous.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p, c_char_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libgsplat_b200.so"

GS_OK = 0
GS_ERR_INVALID_ARG = 1
GS_ERR_CUDA = 2
GS_ERR_CAPACITY = 3
GS_ERR_TIMEOUT = 4

GS_ACT_EXP_SCALES = 1
GS_ACT_SIGMOID_OPACITY = 2


class GsCamera(ctypes.Structure):
    """Mirror of ``gs_camera`` in include/gsplat_b200.h."""

    _fields_ = [
        ("R", c_float * 9),
        ("t", c_float * 3),
        ("fx", c_float),
        ("fy", c_float),
        ("cx", c_float),
        ("cy", c_float),
        ("neg_fx", c_float),
        ("neg_fy", c_float),
        ("clip_x", c_float),
        ("clip_y", c_float),
        ("znear", c_float),
        ("center", c_float * 3),
        ("width", c_int32),
        ("height", c_int32),
    ]


class GsLens(ctypes.Structure):
    """Mirror of ``gs_lens`` in include/gsplat_b200.h."""

    _fields_ = [("orthographic", c_int32), ("fisheye", c_int32), ("n_dist", c_int32), ("dist", c_float * 5)]


class GsAdamGroup(ctypes.Structure):
    """Mirror of ``gs_adam_group`` in include/gsplat_b200.h."""

    _fields_ = [
        ("param", c_void_p),
        ("grad", c_void_p),
        ("m", c_void_p),
        ("v", c_void_p),
        ("n", c_int64),
        ("lr", c_float),
    ]


GS_ADAM_MAX_GROUPS = 8

# name -> (restype, argtypes)
_P = c_void_p
_SIGS = {
    "gs_version": (c_int, []),
    "gs_last_error": (c_char_p, []),
    "gs_kernel_launch_count": (ctypes.c_uint64, []),
    "gs_project_forward": (c_int, [POINTER(GsCamera), _P, _P, _P, c_int64, c_float, c_int, _P, _P, _P, _P, _P, _P]),
    "gs_project_backward": (
        c_int,
        [POINTER(GsCamera), _P, _P, _P, c_int64, c_float, c_int, _P, _P, _P, _P, _P, _P, _P, _P],
    ),
    "gs_eval_sh_forward": (c_int, [c_int, _P, c_int64, c_int, c_int, _P, _P, _P]),
    "gs_eval_sh_backward": (c_int, [c_int, _P, c_int64, c_int, c_int, _P, _P, _P, _P, _P]),
    "gs_preprocess_forward": (
        c_int,
        [POINTER(GsCamera), _P, _P, _P, _P, _P, c_int64, _P, c_int64, c_int, c_int64, c_float, c_int, c_int]
        + [_P] * 8
        + [_P],
    ),
    "gs_preprocess_backward": (
        c_int,
        [POINTER(GsCamera), _P, _P, _P, _P, _P, c_int64, _P, c_int64, c_int, c_int64, c_float, c_int, c_int]
        + [_P] * 6
        + [_P] * 6
        + [_P],
    ),
    "gs_preprocess_backward_views": (
        c_int,
        [_P, c_int, _P, _P, _P, _P, _P, c_int64, _P, c_int64, c_int, c_int64, c_float, c_int, c_int, _P, c_int64]
        + [_P] * 6
        + [_P],
    ),
    "gs_preprocess_backward_views_peer": (
        c_int,
        [_P, c_int, _P, _P, _P, _P, _P, c_int64, _P, c_int64, c_int, c_int64, c_float, c_int, c_int, _P]
        + [_P] * 6
        + [_P],
    ),
    "gs_peer_alloc": (c_int, [c_size_t, ctypes.POINTER(c_void_p), _P]),
    "gs_peer_open": (c_int, [_P, ctypes.POINTER(c_void_p)]),
    "gs_peer_close": (c_int, [_P]),
    "gs_peer_free": (c_int, [_P]),
    "gs_tile_counts": (c_int, [_P, _P, c_int64, c_int, c_int, _P, _P]),
    "gs_bin_workspace_n_bytes": (c_size_t, [c_int64]),
    "gs_bin_workspace_d_bytes": (c_size_t, [c_int64]),
    "gs_wait_failures": (c_int, [_P, c_int]),
    "gs_set_wait_limit": (c_int, [c_int]),
    "gs_bin_status": (c_int, [_P, c_size_t, c_int64, ctypes.POINTER(ctypes.c_uint32), _P]),
    "gs_bin_status_offset": (c_size_t, [c_int64]),
    "gs_mesh_rasterize": (c_int, [_P, _P, c_int64, _P, _P, c_int, c_int, c_float, _P, _P, _P]),
    "gs_bin_total": (c_int, [_P, c_int64, _P, _P]),
    "gs_bin_begin": (c_int, [_P, _P, c_int64, _P, c_size_t, _P, _P]),
    "gs_bin_end": (c_int, [_P, _P, c_int64, c_int64, c_int, c_int, _P, c_size_t, _P, c_size_t, _P, _P, _P]),
    "gs_project_ut_forward": (
        c_int, [POINTER(GsCamera), POINTER(GsLens), _P, _P, _P, c_int64, c_float, c_int, _P, _P, _P, _P, _P, _P]
    ),
    "gs_project_ut_backward": (
        c_int,
        [POINTER(GsCamera), POINTER(GsLens), _P, _P, _P, c_int64, c_float, c_int, _P, _P, _P, _P, _P, _P, _P, _P],
    ),
    "gs_tile_counts_refined": (c_int, [_P, _P, _P, c_int64, c_int, c_int, _P, _P]),
    "gs_bin_end_refined": (
        c_int, [_P, _P, _P, c_int64, c_int64, c_int, c_int, _P, c_size_t, _P, c_size_t, _P, _P, _P]
    ),
    "gs_bin_gaussians_static": (
        c_int, [_P, _P, _P, c_int64, c_int, c_int, c_int64, _P, _P, ctypes.POINTER(c_int64), _P]
    ),
    "gs_l1_ssim_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "gs_l1_ssim_forward": (
        c_int, [_P, _P, c_int, c_int, c_int, c_float, c_float, c_int, c_float, _P, c_size_t, _P, _P]
    ),
    "gs_l1_ssim_backward": (
        c_int, [_P, _P, c_int, c_int, c_int, c_float, c_float, c_int, c_float, _P, c_size_t, c_float, _P, _P]
    ),
    "gs_l1_ssim_backward_dev": (
        c_int, [_P, _P, c_int, c_int, c_int, c_float, c_int, c_float, _P, c_size_t, _P, c_float, c_int, _P, _P]
    ),
    "gs_l1_workspace_bytes": (c_size_t, [c_int64]),
    "gs_l1_forward": (c_int, [_P, _P, c_int64, _P, c_size_t, _P, _P]),
    "gs_l1_backward": (c_int, [_P, _P, c_int64, _P, _P, _P]),
    "gs_adam_step": (c_int, [POINTER(GsAdamGroup), c_int, ctypes.c_double, ctypes.c_double, c_float, c_int, c_int64, _P]),
    "gs_rasterize_forward": (
        c_int,
        [_P, _P, _P, c_int, _P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P],
    ),
    "gs_rasterize_backward": (
        c_int,
        [_P, _P, _P, c_int, _P, c_int64, _P, _P, _P, c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    ),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"mlx3d_b200: CUDA library not built ({LIB_PATH}); run `python -m mlx3d_b200.build`"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def call(name: str, *args) -> None:
    """Call ``name`` and raise on a non-zero status (ValueError for bad
    arguments, RuntimeError otherwise)."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != GS_OK:
        msg = (lib.gs_last_error() or b"").decode(errors="replace")
        if status == GS_ERR_INVALID_ARG:
            raise ValueError(f"{name}: {msg}")
        raise RuntimeError(f"{name} failed (status {status}): {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def require_cuda(name: str, t: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    """Return ``t`` as a contiguous CUDA tensor of ``dtype`` (converting the
    dtype like the reference's ``astype(mx.float32)``); CPU tensors are an
    error: this package has no CPU path."""
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (got device {t.device}); mlx3d_b200 has no CPU path")
    if t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


class _CudaArray:
    """Minimal __cuda_array_interface__ exporter for a raw device pointer."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(int(d) for d in shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None}


def wrap_device(ptr: int, shape: tuple, device, dtype=torch.float32) -> torch.Tensor:
    """A tensor aliasing device memory this library allocated (no copy; the
    memory must outlive the tensor)."""
    typestr = {torch.float32: "<f4", torch.int32: "<i4", torch.int64: "<i8", torch.uint8: "|u1"}[dtype]
    return torch.as_tensor(_CudaArray(ptr, shape, typestr), device=device)
