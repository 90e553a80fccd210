"""NumPy-backed stand-in for the subset of ``mlx.core`` the reference's kernel
tests and benchmarks use: ``array``, ``eval``, the dtypes ``float32``,
``int32``, ``int8``, ``uint32``, and ``abs``, ``maximum``, ``round``,
``clip``, ``argsort``, ``take_along_axis``, ``softmax``, ``arange``, plus
``.astype``, ``.max(axis, keepdims)``, ``@``, ``.shape``.  ``fast.metal_kernel``
does not exist here: Metal kernels are replaced by the CUDA library.
Evaluation is eager, so ``eval`` is a no-op.
"""
from __future__ import annotations

import numpy as _np

float32 = _np.float32
float16 = _np.float16
int32 = _np.int32
int8 = _np.int8
uint32 = _np.uint32
int64 = _np.int64


def _unwrap(a):
    return a._a if isinstance(a, array) else a


class array:
    """Eager array wrapping a NumPy ndarray."""

    __array_priority__ = 100

    def __init__(self, obj, dtype=None):
        a = _unwrap(obj)
        self._a = _np.array(a, dtype=dtype) if dtype is not None else _np.array(a)

    # NumPy interop: np.array(mx_array) works as in MLX
    def __array__(self, dtype=None, copy=None):
        return self._a if dtype is None else self._a.astype(dtype)

    @property
    def shape(self):
        return self._a.shape

    @property
    def dtype(self):
        return self._a.dtype

    @property
    def ndim(self):
        return self._a.ndim

    @property
    def size(self):
        return self._a.size

    @property
    def T(self):
        return array(self._a.T)

    def astype(self, dtype):
        return array(self._a.astype(dtype))

    def max(self, axis=None, keepdims=False):
        return array(self._a.max(axis=axis, keepdims=keepdims))

    def min(self, axis=None, keepdims=False):
        return array(self._a.min(axis=axis, keepdims=keepdims))

    def sum(self, axis=None, keepdims=False):
        return array(self._a.sum(axis=axis, keepdims=keepdims))

    def tolist(self):
        return self._a.tolist()

    def item(self):
        return self._a.item()

    def __len__(self):
        return len(self._a)

    def __getitem__(self, k):
        return array(self._a[_unwrap(k)])

    def __repr__(self):
        return f"array({self._a!r})"

    def _bin(self, other, op):
        return array(op(self._a, _unwrap(other)))

    def __matmul__(self, o): return self._bin(o, _np.matmul)
    def __rmatmul__(self, o): return array(_np.matmul(_unwrap(o), self._a))
    def __add__(self, o): return self._bin(o, _np.add)
    def __radd__(self, o): return self._bin(o, _np.add)
    def __sub__(self, o): return self._bin(o, _np.subtract)
    def __rsub__(self, o): return array(_np.subtract(_unwrap(o), self._a))
    def __mul__(self, o): return self._bin(o, _np.multiply)
    def __rmul__(self, o): return self._bin(o, _np.multiply)
    def __truediv__(self, o): return self._bin(o, _np.true_divide)
    def __rtruediv__(self, o): return array(_np.true_divide(_unwrap(o), self._a))
    def __neg__(self): return array(-self._a)
    def __eq__(self, o): return self._bin(o, _np.equal)
    def __lt__(self, o): return self._bin(o, _np.less)
    def __gt__(self, o): return self._bin(o, _np.greater)


def eval(*args):  # noqa: A001 - mirrors mlx.core.eval
    return None


def abs(a):  # noqa: A001
    return array(_np.abs(_unwrap(a)))


def maximum(a, b):
    return array(_np.maximum(_unwrap(a), _unwrap(b)))


def round(a):  # noqa: A001
    return array(_np.round(_unwrap(a)))


def clip(a, lo, hi):
    return array(_np.clip(_unwrap(a), lo, hi))


def argsort(a, axis=-1):
    return array(_np.argsort(_unwrap(a), axis=axis, kind="stable"))


def take_along_axis(a, idx, axis=-1):
    return array(_np.take_along_axis(_unwrap(a), _unwrap(idx), axis=axis))


def softmax(a, axis=-1):
    x = _unwrap(a)
    m = x.max(axis=axis, keepdims=True)
    e = _np.exp(x - m)
    return array(e / e.sum(axis=axis, keepdims=True))


def arange(*args, dtype=None):
    return array(_np.arange(*args, dtype=dtype))


def zeros(shape, dtype=float32):
    return array(_np.zeros(shape, dtype=dtype))


class _Fast:
    @staticmethod
    def metal_kernel(*args, **kwargs):
        raise NotImplementedError(
            "Metal kernels do not exist on this platform; the kernels come from "
            "aethermoe_b200.kernels (CUDA, sm_100a)")


fast = _Fast()
