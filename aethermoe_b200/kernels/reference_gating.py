"""Drop-in for the reference's ``src/kernels/reference_gating.py``.

``reference_gating(hidden, gate_weight, gate_bias, k)`` -- the reference's
"unfused" tier (matmul + argsort + softmax over the k selected,
``reference_gating.py:25-57``).  On B200 both tiers run the same gating
kernel; this one uses its FAST mode (fused multiply-add logits, like a
library matmul whose summation order is unspecified), so it plays the role
the MLX matmul path plays in the reference: an independent arithmetic path
whose expert SETS and softmax values must agree with ``fused_gating``.
"""
from __future__ import annotations

from .. import _lib
from ._common import wrap_like
from .fused_gating_metal import gating


def reference_gating(hidden, gate_weight, gate_bias, k: int):
    """Returns ``(topk_idx [N,k] int32, topk_val [N,k] float32)``, sorted by
    descending logit (``reference_gating.py:34-36``)."""
    idx, val = gating(hidden, gate_weight, gate_bias, k, mode=_lib.GATING_FAST)
    return wrap_like(hidden, idx, val)
