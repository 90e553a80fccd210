"""Drop-in for the reference's ``src/kernels/fused_gating_metal.py``.

``fused_gating(hidden, gate_weight, gate_bias, k)`` with the reference's
argument order, output layout (``idx [N,k] int32``, ``val [N,k] float32``,
descending logit order, ties to the lowest expert id) and errors
(``ValueError`` for ``num_experts > MAX_EXPERTS`` or an invalid ``k``,
``fused_gating_metal.py:380-388``).  The kernel is the B200 gating kernel of
``libaethermoe.so`` in EXACT mode: its logits are bit-identical to the
reference's NumPy specification ``fused_kernel_simulation``
(``prototype/math_proto.py:19-50``).
"""
from __future__ import annotations

import ctypes

import numpy as np

from .. import _lib
from ._common import IdentityCache, to_numpy, wrap_like

MAX_EXPERTS = _lib.MAX_EXPERTS  # fused_gating_metal.py:230
MAX_TOPK = _lib.MAX_TOPK        # fused_gating_metal.py:231

_gate_cache = IdentityCache()


def _packed_gate(gate_weight, gate_bias, device):
    def make():
        return _lib.Gate(to_numpy(gate_weight, np.float32), to_numpy(gate_bias, np.float32), device)
    return _gate_cache.get((gate_weight, gate_bias), make)


def gating(hidden, gate_weight, gate_bias, k, mode=_lib.GATING_EXACT, k_extra=0, device=0):
    """Host-buffer gating through ``aem_gating_host``; NumPy in, NumPy out."""
    h = to_numpy(hidden)
    if h.ndim != 2:
        raise ValueError("hidden must be [N, D]")
    n_tokens, d_model = h.shape
    w_shape = np.shape(gate_weight)
    if len(w_shape) != 2 or w_shape[0] != d_model:
        raise ValueError(f"gate_weight must be [{d_model}, E], got {w_shape}")
    num_experts = w_shape[1]
    if num_experts > MAX_EXPERTS:
        raise ValueError(
            f"num_experts={num_experts} exceeds this kernel's compile-time "
            f"MAX_EXPERTS={MAX_EXPERTS}")
    if k > MAX_TOPK or k > num_experts or k < 1:
        raise ValueError(f"k={k} invalid for num_experts={num_experts} (MAX_TOPK={MAX_TOPK})")
    if h.dtype == np.float32:
        xd = _lib.F32
    elif h.dtype.name == "bfloat16" or h.dtype == np.uint16:
        xd = _lib.BF16
    else:
        h = h.astype(np.float32)
        xd = _lib.F32
    gate = _packed_gate(gate_weight, gate_bias, device)
    ksel = k + k_extra
    idx = np.empty((n_tokens, ksel), dtype=np.int32)
    val = np.empty((n_tokens, k), dtype=np.float32)
    if n_tokens:
        _lib.check(_lib.lib().aem_gating_host(
            _lib.context(device), gate.handle, h.ctypes.data, xd, n_tokens, k, k_extra, mode,
            idx.ctypes.data, val.ctypes.data), "fused_gating")
    return idx, val


def fused_gating(hidden, gate_weight, gate_bias, k: int):
    """Args mirror ``reference_gating`` (``fused_gating_metal.py:361-376``).

    Returns ``(topk_idx [N,k] int32, topk_val [N,k] float32)``.
    """
    idx, val = gating(hidden, gate_weight, gate_bias, k, mode=_lib.GATING_EXACT)
    return wrap_like(hidden, idx, val)
