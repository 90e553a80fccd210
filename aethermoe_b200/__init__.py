"""AetherMoE MoE-layer hot path for NVIDIA B200 (sm_100a).

The compute lives in ``libaethermoe.so`` (hand-written CUDA, C ABI in
``include/aem.h``).  This package is the host-side mirror of the reference's
Python kernel API:

* ``aethermoe_b200.kernels.fused_gating_metal.fused_gating``
* ``aethermoe_b200.kernels.reference_gating.reference_gating``
* ``aethermoe_b200.kernels.quantized_gemm.{quantize_weights, dequantize_naive,
  naive_quantized_matmul, fused_quantized_matmul}``

plus the composed layer (``aethermoe_b200.moe``): a single-GPU MoE layer and
the expert-parallel layer over NCCL.
"""
from ._lib import (AemError, AemTimeout, CAPACITY_UNLIMITED, GATING_EXACT, GATING_FAST, Gate,
                   MoeConfig, QWeight, check, context, device_count, lib)

__all__ = ["AemError", "AemTimeout", "CAPACITY_UNLIMITED", "GATING_EXACT", "GATING_FAST", "Gate",
           "MoeConfig", "QWeight", "check", "context", "device_count", "lib"]
__version__ = "0.1.0"
