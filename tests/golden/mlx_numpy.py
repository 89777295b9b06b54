"""A float32 numpy stand-in for the parts of ``mlx.core`` that mlx3D's
projection, SH, binning, camera, naive-renderer and density-control modules
call.

Test infrastructure only: ``make_golden.py`` installs it as ``mlx.core`` so
that the reference's own Python source (imported from the reference checkout
in the build container) runs without MLX, which has no Linux wheel.  Every
operation is evaluated elementwise in IEEE float32 (numpy does not contract
a*b+c into FMAs), with MLX's typing rules where they differ from numpy's:

* Python scalars and lists become float32 / int32 arrays (MLX's defaults);
* ``cumsum`` keeps the input's integer type;
* ``argsort`` is stable (MLX's tie order is not documented: unpinned);
  ``argpartition`` is numpy's (the order inside MLX's selection is not
  documented either: only the selected set is compared);
* ``random.normal`` draws from numpy's global generator;
* ``linalg.norm`` over an axis and small matrix products sum their terms
  left to right without FMA (MLX's reduction order is not documented:
  unpinned);
* ``exp`` is numpy's float32 exponential (MLX's differs in the last bit on
  some inputs; only the naive renderer uses it, compared with a tolerance).

Only what those modules use is provided; any other attribute raises when it
is called, so a silent stand-in never hides an unemulated operation.
"""

from __future__ import annotations

import numpy as np

float32 = np.float32
float16 = np.float16
float64 = np.float64
int32 = np.int32
int64 = np.int64
uint32 = np.uint32
uint8 = np.uint8
bool_ = np.bool_
int8 = np.int8
int16 = np.int16
uint16 = np.uint16


class _At:
    def __init__(self, arr, idx):
        self.arr, self.idx = arr, idx

    def _apply(self, ufunc, v):
        out = np.array(self.arr, copy=True)
        ufunc.at(out, _np(self.idx), _np(v).astype(out.dtype, copy=False))
        return out.view(array)

    def add(self, v):
        return self._apply(np.add, v)

    def minimum(self, v):
        return self._apply(np.minimum, v)

    def maximum(self, v):
        return self._apply(np.maximum, v)

    def multiply(self, v):
        return self._apply(np.multiply, v)


class _AtIndexer:
    def __init__(self, arr):
        self.arr = arr

    def __getitem__(self, idx):
        return _At(self.arr, idx)


class array(np.ndarray):
    """mx.array: an ndarray with MLX's constructor defaults and ``.at``."""

    def __new__(cls, data, dtype=None):
        if isinstance(data, np.ndarray):
            a = np.asarray(data, dtype=dtype)
        else:
            a = np.asarray(data)
            if dtype is None:
                if a.dtype.kind == "f":
                    dtype = np.float32
                elif a.dtype.kind in "iu":
                    dtype = np.int32
            a = a.astype(dtype) if dtype is not None else a
        return np.ascontiguousarray(a).view(cls)

    @property
    def at(self):
        return _AtIndexer(self)


def _np(x):
    return x.view(np.ndarray) if isinstance(x, np.ndarray) else x


def _wrap(x):
    return np.asarray(x).view(array)


def _f32(x):
    if isinstance(x, np.ndarray):
        return x
    a = np.asarray(x)
    return a.astype(np.float32) if a.dtype.kind == "f" else a


# ------------------------------------------------------------- constructors
def zeros(shape, dtype=float32):
    return _wrap(np.zeros(shape, dtype=dtype))


def ones(shape, dtype=float32):
    return _wrap(np.ones(shape, dtype=dtype))


def full(shape, vals, dtype=None):
    if dtype is None:
        dtype = np.float32 if isinstance(vals, float) else np.asarray(vals).dtype
    return _wrap(np.full(shape, vals, dtype=dtype))


def zeros_like(a):
    return _wrap(np.zeros_like(_np(a)))


def ones_like(a):
    return _wrap(np.ones_like(_np(a)))


def eye(n, m=None, k=0, dtype=float32):
    return _wrap(np.eye(n, m, k, dtype=dtype))


def arange(*args, dtype=None):
    if dtype is None:
        dtype = np.float32 if any(isinstance(a, float) for a in args) else np.int32
    return _wrap(np.arange(*args, dtype=dtype))


# ------------------------------------------------------------- elementwise
def _ew(fn):
    def f(*a, **k):
        return _wrap(fn(*[_f32(_np(x)) for x in a], **k))

    return f


maximum = _ew(np.maximum)
minimum = _ew(np.minimum)
sqrt = _ew(np.sqrt)
floor = _ew(np.floor)
ceil = _ew(np.ceil)
abs = _ew(np.abs)  # noqa: A001
tan = _ew(np.tan)
arctan = _ew(np.arctan)
sin = _ew(np.sin)
cos = _ew(np.cos)
exp = _ew(np.exp)


def sigmoid(a):
    a = _f32(_np(a))
    return _wrap((1.0 / (1.0 + np.exp(-a))).astype(a.dtype))


def argpartition(a, kth, axis=-1):
    return _wrap(np.argpartition(_np(a), kth, axis=axis).astype(np.int32))


class random:  # noqa: N801
    """Draws from numpy's global generator (seeded by the caller)."""

    @staticmethod
    def normal(shape=(), dtype=float32, loc=0.0, scale=1.0, key=None):
        return _wrap((np.random.normal(size=shape) * scale + loc).astype(dtype))


def where(c, a, b):
    a, b = _f32(_np(a)), _f32(_np(b))
    return _wrap(np.where(_np(c), a, b))


def clip(a, a_min, a_max):
    a = _np(a)
    lo = None if a_min is None else np.asarray(a_min).astype(a.dtype)
    hi = None if a_max is None else np.asarray(a_max).astype(a.dtype)
    return _wrap(np.clip(a, lo, hi))


def stop_gradient(a):
    return a


# ---------------------------------------------------------------- shape ops
def stack(arrs, axis=0):
    return _wrap(np.stack([_np(a) for a in arrs], axis=axis))


def concatenate(arrs, axis=0):
    return _wrap(np.concatenate([_np(a) for a in arrs], axis=axis))


def broadcast_to(a, shape):
    return _wrap(np.broadcast_to(_np(a), shape))


def swapaxes(a, a1, a2):
    return _wrap(np.swapaxes(_np(a), a1, a2))


# --------------------------------------------------------------- reductions
def _seq_reduce(a, axis, op, keepdims=False):
    """Left-to-right reduction along one axis (no pairwise summation)."""
    a = _np(a)
    if axis is None:
        a = a.reshape(-1)
        axis = 0
    a = np.moveaxis(a, axis, 0)
    acc = a[0].copy()
    for i in range(1, a.shape[0]):
        acc = op(acc, a[i])
    if keepdims:
        acc = np.expand_dims(acc, axis)
    return _wrap(acc)


def sum(a, axis=None, keepdims=False):  # noqa: A001
    return _seq_reduce(a, axis, np.add, keepdims)


def prod(a, axis=None, keepdims=False):
    return _seq_reduce(a, axis, np.multiply, keepdims)


def mean(a, axis=None, keepdims=False):
    a = _np(a)
    n = a.size if axis is None else a.shape[axis]
    return _wrap(_np(sum(a, axis, keepdims)) / np.float32(n))


def cumsum(a, axis=None):
    a = _np(a)
    if axis is None:
        a, axis = a.reshape(-1), 0
    return _wrap(np.cumsum(a, axis=axis, dtype=a.dtype))


def cumprod(a, axis=None):
    a = _np(a)
    if axis is None:
        a, axis = a.reshape(-1), 0
    return _wrap(np.cumprod(a, axis=axis, dtype=a.dtype))


def argsort(a, axis=-1):
    return _wrap(np.argsort(_np(a), axis=axis, kind="stable").astype(np.int32))


class linalg:  # noqa: N801
    @staticmethod
    def norm(a, axis=None, keepdims=False):
        a = _np(a)
        sq = a * a
        return sqrt(_seq_reduce(sq, axis if axis is not None else None, np.add, keepdims))

    @staticmethod
    def cross(a, b, axis=-1):
        a, b = _np(a), _np(b)
        x = a[..., 1] * b[..., 2] - a[..., 2] * b[..., 1]
        y = a[..., 2] * b[..., 0] - a[..., 0] * b[..., 2]
        z = a[..., 0] * b[..., 1] - a[..., 1] * b[..., 0]
        return _wrap(np.stack([x, y, z], axis=-1))


def _matmul(a, b):
    """Small float32 matrix products, terms summed left to right, no FMA."""
    a, b = _np(a), _np(b)
    vec_b = b.ndim == 1
    if vec_b:
        b = b[:, None]
    vec_a = a.ndim == 1
    if vec_a:
        a = a[None, :]
    k = a.shape[-1]
    acc = a[..., :, 0:1] * b[..., 0:1, :]
    for i in range(1, k):
        acc = acc + a[..., :, i:i + 1] * b[..., i:i + 1, :]
    if vec_b:
        acc = acc[..., 0]
    if vec_a:
        acc = acc[..., 0, :] if not vec_b else acc[..., 0]
    return _wrap(acc)


array.__matmul__ = lambda self, other: _matmul(self, other)
array.__rmatmul__ = lambda self, other: _matmul(other, self)
matmul = _matmul


def __getattr__(name):
    def _missing(*a, **k):
        raise NotImplementedError(f"mlx.core.{name} is not emulated by the numpy stand-in")

    return _missing
