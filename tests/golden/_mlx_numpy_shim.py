"""A NumPy stand-in for the parts of ``mlx.core`` / ``mlx.nn`` that the
reference's eager ConvRot functions use -- fixture generation only.

MLX is not installable in this container (Darwin/arm64 wheels, no network), so
``make_golden.py`` installs this module as ``mlx`` and then imports the
reference's ``convrot_mlx`` package unchanged.  The eager functions then run
their own code (butterfly order, packing, quantization, epilogue order) with
the arithmetic below:

* dtypes follow MLX promotion: a Python scalar is weakly typed and takes the
  array's dtype; float16 with bfloat16 promotes to float32.
* every float16 / bfloat16 op is computed in float32 and rounded to the dtype
  (round to nearest even), i.e. a correctly rounded 16-bit op;
* ``round`` is round-half-to-even; float -> int casts truncate.

The Metal kernels (``mx.fast.metal_kernel``) are not emulated: calling one
raises.
"""

from __future__ import annotations

import math
import sys
import types

import numpy as np


class Dtype:
    def __init__(self, name, np_store, kind, size):
        self.name = name
        self.np_store = np_store  # numpy dtype holding the values
        self.kind = kind  # "f", "i", "u", "b"
        self.size = size

    def __repr__(self):
        return f"mlx.core.{self.name}"


bool_ = Dtype("bool_", np.bool_, "b", 1)
int8 = Dtype("int8", np.int8, "i", 1)
uint8 = Dtype("uint8", np.uint8, "u", 1)
int32 = Dtype("int32", np.int32, "i", 4)
int64 = Dtype("int64", np.int64, "i", 8)
float16 = Dtype("float16", np.float32, "f", 2)
bfloat16 = Dtype("bfloat16", np.float32, "f", 2)
float32 = Dtype("float32", np.float32, "f", 4)

_NP_TO_DTYPE = {
    np.dtype(np.bool_): bool_,
    np.dtype(np.int8): int8,
    np.dtype(np.uint8): uint8,
    np.dtype(np.int32): int32,
    np.dtype(np.int64): int64,
    np.dtype(np.float16): float16,
    np.dtype(np.float32): float32,
    np.dtype(np.float64): float32,
}


def _round_bf16(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) >> np.uint64(16)) << np.uint64(16)
    out = r.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.float32(np.nan)
    return out


def _store(values, dtype: Dtype):
    """Convert raw numeric values to the storage of ``dtype`` (with rounding)."""

    v = np.asarray(values)
    if dtype is bfloat16:
        return _round_bf16(v.astype(np.float32))
    if dtype is float16:
        return v.astype(np.float32).astype(np.float16).astype(np.float32)
    if dtype is float32:
        return v.astype(np.float32)
    if dtype.kind in "iu":
        if v.dtype.kind == "f":
            with np.errstate(invalid="ignore"):
                v = np.trunc(v)
        return v.astype(dtype.np_store)
    return v.astype(np.bool_)


def _promote(a: Dtype, b: Dtype) -> Dtype:
    if a is b:
        return a
    if a.kind == "f" and b.kind == "f":
        if a.size == 4 or b.size == 4:
            return float32
        return float32  # float16 with bfloat16
    if a.kind == "f":
        return a
    if b.kind == "f":
        return b
    if a.kind == "b":
        return b
    if b.kind == "b":
        return a
    return a if a.size >= b.size else b


def _scalar_dtype(array_dtype: Dtype, scalar) -> Dtype:
    if isinstance(scalar, bool):
        return array_dtype
    if isinstance(scalar, int):
        return array_dtype if array_dtype.kind != "b" else int32
    if isinstance(scalar, float):
        return array_dtype if array_dtype.kind == "f" else float32
    raise TypeError(f"unsupported scalar {scalar!r}")


class array:  # noqa: N801 - mirrors mlx.core.array
    def __init__(self, values, dtype: Dtype | None = None):
        if isinstance(values, array):
            dt = dtype or values.dtype
            self._v = _store(values._v, dt)
            self.dtype = dt
            return
        v = np.asarray(values)
        if dtype is None:
            if isinstance(values, float):
                dtype = float32
            elif isinstance(values, bool):
                dtype = bool_
            elif isinstance(values, int):
                dtype = int32
            else:
                dtype = _NP_TO_DTYPE[v.dtype]
        self._v = _store(v, dtype)
        self.dtype = dtype

    # -- construction helpers -------------------------------------------------
    @classmethod
    def _wrap(cls, values, dtype):
        out = cls.__new__(cls)
        out._v = _store(values, dtype)
        out.dtype = dtype
        return out

    # -- metadata ---------------------------------------------------------------
    @property
    def shape(self):
        return tuple(self._v.shape)

    @property
    def ndim(self):
        return self._v.ndim

    @property
    def size(self):
        return self._v.size

    @property
    def T(self):  # noqa: N802
        return array._wrap(self._v.T, self.dtype)

    def __array__(self, dtype=None, copy=None):
        v = self._v
        if self.dtype is float16:
            v = v.astype(np.float16)
        return v if dtype is None else v.astype(dtype)

    def item(self):
        return self._v.item()

    def tolist(self):
        return np.asarray(self).tolist()

    def astype(self, dtype):
        return array._wrap(self._v, dtype)

    def reshape(self, *shape):
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        return array._wrap(self._v.reshape(shape), self.dtype)

    def __getitem__(self, index):
        return array._wrap(self._v[index], self.dtype)

    # -- arithmetic -----------------------------------------------------------
    def _binary(self, other, fn, reverse=False):
        if isinstance(other, array):
            dt = _promote(self.dtype, other.dtype)
            ov = other._v
        else:
            dt = _scalar_dtype(self.dtype, other)
            ov = other
        a = _store(self._v, dt) if dt is not self.dtype else self._v
        b = _store(np.asarray(ov), dt)
        if reverse:
            a, b = b, a
        if dt.kind == "f":
            with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
                res = fn(a.astype(np.float32), b.astype(np.float32)).astype(np.float32)
        else:
            res = fn(a.astype(np.int64), b.astype(np.int64))
        return array._wrap(res, dt)

    def _compare(self, other, fn):
        ov = other._v if isinstance(other, array) else other
        return array._wrap(fn(self._v, ov), bool_)

    def __add__(self, o):
        return self._binary(o, np.add)

    def __radd__(self, o):
        return self._binary(o, np.add, True)

    def __sub__(self, o):
        return self._binary(o, np.subtract)

    def __rsub__(self, o):
        return self._binary(o, np.subtract, True)

    def __mul__(self, o):
        return self._binary(o, np.multiply)

    def __rmul__(self, o):
        return self._binary(o, np.multiply, True)

    def __truediv__(self, o):
        if self.dtype.kind != "f" and not (isinstance(o, array) and o.dtype.kind == "f"):
            return self.astype(float32)._binary(o, np.divide)
        return self._binary(o, np.divide)

    def __and__(self, o):
        return self._binary(o, np.bitwise_and)

    def __or__(self, o):
        return self._binary(o, np.bitwise_or)

    def __lshift__(self, o):
        return self._binary(o, np.left_shift)

    def __rshift__(self, o):
        return self._binary(o, np.right_shift)

    def __neg__(self):
        return array._wrap(-self._v, self.dtype)

    def __ge__(self, o):
        return self._compare(o, np.greater_equal)

    def __gt__(self, o):
        return self._compare(o, np.greater)

    def __le__(self, o):
        return self._compare(o, np.less_equal)

    def __lt__(self, o):
        return self._compare(o, np.less)

    def __eq__(self, o):  # noqa: D105
        return self._compare(o, np.equal)

    def __matmul__(self, o):
        dt = _promote(self.dtype, o.dtype)
        if dt.kind != "f":
            raise TypeError("integer matmul is not used by the eager contract")
        res = (self._v.astype(np.float64) @ o._v.astype(np.float64)).astype(np.float32)
        return array._wrap(res, dt)


def _as_array(x, like: Dtype | None = None):
    if isinstance(x, array):
        return x
    if like is not None:
        return array(np.asarray(x), dtype=_scalar_dtype(like, x) if np.isscalar(x) else None)
    return array(x)


def stack(arrays, axis=0):
    dt = arrays[0].dtype
    return array._wrap(np.stack([a._v for a in arrays], axis=axis), dt)


def where(cond, x, y):
    if isinstance(x, array):
        dt = x.dtype if not isinstance(y, array) else _promote(x.dtype, y.dtype)
    elif isinstance(y, array):
        dt = y.dtype
    else:
        dt = float32
    xv = x._v if isinstance(x, array) else x
    yv = y._v if isinstance(y, array) else y
    return array._wrap(np.where(cond._v, xv, yv), dt)


def abs(x):  # noqa: A001
    return array._wrap(np.abs(x._v), x.dtype)


def max(x, axis=None, keepdims=False):  # noqa: A001
    return array._wrap(np.max(x._v, axis=axis, keepdims=keepdims), x.dtype)


def maximum(a, b):
    return a._binary(b, np.maximum) if isinstance(a, array) else b._binary(a, np.maximum)


def clip(x, lo, hi):
    dt = x.dtype
    return array._wrap(np.clip(x._v, lo, hi), dt)


def round(x, decimals=0):  # noqa: A001
    if decimals:
        raise NotImplementedError
    return array._wrap(np.rint(x._v), x.dtype)


def zeros(shape, dtype=float32):
    return array._wrap(np.zeros(shape), dtype)


def ones(shape, dtype=float32):
    return array._wrap(np.ones(shape), dtype)


def full(shape, value, dtype=float32):
    return array._wrap(np.full(shape, value), dtype)


def isfinite(x):
    return array._wrap(np.isfinite(x._v), bool_)


def all(x):  # noqa: A001
    return array._wrap(np.all(x._v), bool_)


def eval(*args):  # noqa: A001
    return None


def compile(fn):  # noqa: A001
    return fn


def _metal_kernel(**kwargs):
    raise RuntimeError("Metal kernels cannot run under the NumPy stand-in")


fast = types.SimpleNamespace(metal_kernel=_metal_kernel)


class _Module:
    def __init__(self, *args, **kwargs):
        pass


class _Linear(_Module):
    def __init__(self, input_dims, output_dims, bias=True):
        super().__init__()
        self.weight = zeros((output_dims, input_dims))
        if bias:
            self.bias = zeros((output_dims,))


def install() -> None:
    """Register this module as ``mlx`` / ``mlx.core`` / ``mlx.nn``."""

    core = sys.modules[__name__]
    mlx_pkg = types.ModuleType("mlx")
    nn = types.ModuleType("mlx.nn")
    nn.Module = _Module
    nn.Linear = _Linear
    mlx_pkg.core = core
    mlx_pkg.nn = nn
    sys.modules["mlx"] = mlx_pkg
    sys.modules["mlx.core"] = core
    sys.modules["mlx.nn"] = nn


__all__ = ["install", "array", "math"]
