"""ctypes loaders for the compiled CPU checkers -- TEST INFRASTRUCTURE ONLY.

``liboracle.so`` is the C restatement of the capacity rule
(``oracle/capacity_rule.c``); ``_ref/libref_router.so`` is the reference's own
``Router`` compiled from ``src/orchestration/router.hpp`` by ``oracle/Makefile``.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
UNLIMITED = (1 << 64) - 1
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_lib = None
_ref = None


def _load_oracle():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(os.path.join(_HERE, "liboracle.so"))
        lib.oracle_capacity_assign.argtypes = [_u32p, _u32p, _u32p, ctypes.c_uint64,
                                               ctypes.c_uint64, _u32p]
        lib.oracle_capacity_assign.restype = ctypes.c_int
        lib.oracle_moe_route.argtypes = [_i32p, ctypes.c_uint64, ctypes.c_uint32,
                                         ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64, _u32p]
        lib.oracle_moe_route.restype = ctypes.c_int
        _lib = lib
    return _lib


def ref_available():
    return os.path.exists(os.path.join(_HERE, "_ref", "libref_router.so"))


def _load_ref():
    global _ref
    if _ref is None:
        lib = ctypes.CDLL(os.path.join(_HERE, "_ref", "libref_router.so"))
        lib.ref_route_batch.argtypes = [_u32p, _u32p, _u32p, ctypes.c_void_p, ctypes.c_uint64,
                                        ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32,
                                        _u32p, _u32p, ctypes.c_void_p]
        lib.ref_route_batch.restype = ctypes.c_int
        lib.ref_last_error.restype = ctypes.c_char_p
        _ref = lib
    return _ref


def _cap(capacity):
    return UNLIMITED if capacity is None else int(capacity)


def capacity_assign(primary, secondary, batch_position, capacity):
    """C restatement of ``Router::assign_effective_experts`` (router.hpp:249-266)."""
    p = np.ascontiguousarray(primary, dtype=np.uint32)
    s = np.ascontiguousarray(secondary, dtype=np.uint32)
    pos = np.ascontiguousarray(batch_position, dtype=np.uint32)
    out = np.zeros(p.shape[0], dtype=np.uint32)
    rc = _load_oracle().oracle_capacity_assign(p, s, pos, p.shape[0], _cap(capacity), out)
    if rc != 0:
        raise MemoryError("oracle_capacity_assign")
    return out.astype(np.int32)


def moe_route(idx_ext, k, num_experts, capacity):
    """Slot-major MoE routing (see ``aem_oracle.moe_units``) in C."""
    idx = np.ascontiguousarray(idx_ext, dtype=np.int32)
    t = idx.shape[0]
    out = np.zeros(t * k, dtype=np.uint32)
    rc = _load_oracle().oracle_moe_route(idx, t, idx.shape[1], k, num_experts, _cap(capacity), out)
    if rc != 0:
        raise MemoryError("oracle_moe_route")
    return out.astype(np.int32)


def ref_route_batch(primary, secondary, batch_position, capacity, num_experts, num_shards,
                    payload=None):
    """Runs the reference ``Router::route_batch`` (router.hpp:67-100) in-process.

    Returns ``(effective_expert, processed_by_shard, negated_payload)`` per
    batch position.
    """
    p = np.ascontiguousarray(primary, dtype=np.uint32)
    s = np.ascontiguousarray(secondary, dtype=np.uint32)
    pos = np.ascontiguousarray(batch_position, dtype=np.uint32)
    n = p.shape[0]
    eff = np.zeros(n, dtype=np.uint32)
    shard = np.zeros(n, dtype=np.uint32)
    pay_in = None if payload is None else np.ascontiguousarray(payload, dtype=np.float32)
    pay_out = np.zeros(n, dtype=np.float32)
    lib = _load_ref()
    rc = lib.ref_route_batch(p, s, pos, None if pay_in is None else pay_in.ctypes.data, n,
                             _cap(capacity), num_experts, num_shards, eff, shard,
                             pay_out.ctypes.data)
    if rc != 0:
        raise RuntimeError(lib.ref_last_error().decode())
    return eff.astype(np.int32), shard.astype(np.int32), pay_out
