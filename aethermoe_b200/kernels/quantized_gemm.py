"""Drop-in for the reference's ``src/kernels/quantized_gemm.py``.

* ``quantize_weights(w[D,E]) -> (q int8 [D,E], scale [1,E])`` -- per-output-column
  symmetric INT8 (``quantized_gemm.py:70-76``), computed by the library's
  quantise kernel, bit-exact with the float32 NumPy formula.
* ``dequantize_naive`` / ``naive_quantized_matmul`` -- the reference's
  "dequantise the whole matrix, then matmul" tier (``:79-92``), kept as the
  library-GEMM baseline: elementwise dequantisation and a float32 cuBLAS
  matmul through torch on the GPU.
* ``fused_quantized_matmul(x[N,D], q[D,E], scale[1,E]) -> [N,E] float32``
  (``:184-226``) -- the B200 tensor-core INT8 GEMM of ``libaethermoe.so``
  (weights packed once per array, cached by identity like ``:148-167``).
"""
from __future__ import annotations

import numpy as np

from .. import _lib
from ._common import IdentityCache, to_numpy, wrap_like

SIMDGROUPS_PER_TG = 8  # quantized_gemm.py:65 (launch shape of the Metal kernel; unused here)

_qweight_cache = IdentityCache()


def quantize_weights(weight_fp32):
    """``weight_fp32: [D, E] -> (q_int8: [D, E], scale: [1, E])``."""
    w = to_numpy(weight_fp32, np.float32)
    if w.ndim != 2:
        raise ValueError("weight must be [D, E]")
    k, n = w.shape
    q = np.empty((k, n), dtype=np.int8)
    s = np.empty((1, n), dtype=np.float32)
    _lib.check(_lib.lib().aem_quantize_int8_host(_lib.context(0), w.ctypes.data, k, n,
                                                 q.ctypes.data, s.ctypes.data), "quantize_weights")
    return wrap_like(weight_fp32, q, s)


def _torch_cuda():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("naive_quantized_matmul runs on the GPU (no CUDA device)")
    return torch


def dequantize_naive(q_int8, scale):
    """Materialises ``q.astype(float32) * scale`` (``quantized_gemm.py:79-83``) on the GPU."""
    torch = _torch_cuda()
    q = torch.as_tensor(to_numpy(q_int8, np.int8), device="cuda")
    s = torch.as_tensor(to_numpy(scale, np.float32), device="cuda")
    out = (q.to(torch.float32) * s).cpu().numpy()
    return wrap_like(q_int8, out)[0]


def naive_quantized_matmul(x_fp32, q_int8, scale):
    """Dequantise-then-matmul (``quantized_gemm.py:86-92``): float32 cuBLAS on the GPU."""
    torch = _torch_cuda()
    x = torch.as_tensor(to_numpy(x_fp32, np.float32), device="cuda")
    q = torch.as_tensor(to_numpy(q_int8, np.int8), device="cuda")
    s = torch.as_tensor(to_numpy(scale, np.float32), device="cuda")
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        out = (x @ (q.to(torch.float32) * s)).cpu().numpy()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return wrap_like(x_fp32, out)[0]


def _packed(q_int8, scale):
    def make():
        q = to_numpy(q_int8, np.int8)
        s = to_numpy(scale, np.float32)
        return _lib.QWeight(q, s.reshape(1, -1), 0)
    return _qweight_cache.get((q_int8, scale), make)


def fused_quantized_matmul(x_fp32, q_int8, scale):
    """``x_fp32 [N, D]``, ``q_int8 [D, E]``, ``scale [1, E]`` -> ``out [N, E]`` float32."""
    x = to_numpy(x_fp32)
    if x.ndim != 2:
        raise ValueError("x must be [N, D]")
    n_tokens, d_model = x.shape
    qs = np.shape(q_int8)
    if len(qs) != 2:
        raise ValueError("q_int8 must be [D, E]")
    d_model2, num_experts = qs
    if d_model != d_model2:
        raise ValueError(f"shape mismatch: x has D={d_model}, q_weight has D={d_model2}")
    if x.dtype.name == "bfloat16":
        xd = _lib.BF16
    else:
        x = x.astype(np.float32, copy=False)
        xd = _lib.F32
    w = _packed(q_int8, scale)
    out = np.empty((n_tokens, num_experts), dtype=np.float32)
    if n_tokens:
        _lib.check(_lib.lib().aem_qgemm_host(_lib.context(0), w.handle, 0, x.ctypes.data, xd,
                                             n_tokens, out.ctypes.data), "fused_quantized_matmul")
    return wrap_like(x_fp32, out)[0]
