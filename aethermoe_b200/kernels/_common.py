"""Array conversion and the bounded identity caches shared by the shim modules."""
from __future__ import annotations

import collections

import numpy as np


def to_numpy(a, dtype=None):
    """NumPy view/copy of a NumPy array, an ``mlx.core`` array (compat shim)
    or a CPU torch tensor."""
    if hasattr(a, "detach") and hasattr(a, "cpu"):
        a = a.detach().cpu().numpy()
    out = np.asarray(a)
    if dtype is not None and out.dtype != dtype:
        out = out.astype(dtype)
    return np.ascontiguousarray(out)


def wrap_like(ref, *arrays):
    """Returns ``arrays`` as the array type of ``ref`` (compat ``mx.array`` or NumPy)."""
    cls = type(ref)
    if getattr(cls, "__module__", "").startswith("mlx"):
        return tuple(cls(a) for a in arrays)
    return arrays


class IdentityCache:
    """Cache keyed by object identity holding a strong reference to the key
    objects (so a freed id cannot be reused for a different array while the
    entry lives), bounded LRU -- the reference's caches
    (``fused_gating_metal.py:320-344``, ``quantized_gemm.py:148-167``) with the
    unbounded growth they flag (``fused_gating_metal.py:140-146``) removed."""

    def __init__(self, limit=64):
        self.limit = limit
        self._d = collections.OrderedDict()

    def get(self, keys, make):
        key = tuple(id(k) for k in keys)
        hit = self._d.get(key)
        if hit is not None and all(a is b for a, b in zip(hit[0], keys)):
            self._d.move_to_end(key)
            return hit[1]
        value = make()
        self._d[key] = (tuple(keys), value)
        while len(self._d) > self.limit:
            self._d.popitem(last=False)
        return value

    def clear(self):
        self._d.clear()
