"""The C-ABI library: builds, loads, exports every symbol ``include/aem.h``
declares, and its host-only logic and argument checks work without a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

import aethermoe_b200 as aem
from aethermoe_b200 import _lib
from aethermoe_b200.moe import ep_plan_bases
import aem_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "aem.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(aem_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(_lib.LIB_PATH)
    names = _declared()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # and the Python binding covers all of them
    assert set(names) <= set(_lib.exported_symbols()) | {"aem_device_status"}


def test_version_and_device_count_without_gpu():
    assert aem.lib().aem_version().startswith(b"aethermoe-b200")
    assert aem.device_count() >= 0


def test_ep_plan_bases_matches_oracle():
    rng = np.random.default_rng(0)
    for R, k, e in [(1, 2, 8), (2, 6, 64), (8, 6, 64), (4, 3, 16)]:
        counts = rng.integers(0, 500, size=(R, k, e))
        for r in range(R):
            np.testing.assert_array_equal(ep_plan_bases(counts, r), O.ep_slot_bases(counts, r))


def test_ep_plan_bases_rejects_bad_rank():
    with pytest.raises(ValueError):
        ep_plan_bases(np.zeros((2, 2, 4), np.int64), 2)


def test_capacity_route_argument_checks():
    L = aem.lib()
    assert L.aem_capacity_route(None, None, None, 10, 0, 5, None, None, 0, None) == _lib.AEM_EINVAL
    assert L.aem_capacity_route(None, None, None, 10, 300, 5, None, None, 0, None) == _lib.AEM_EINVAL
    assert L.aem_capacity_route(None, None, None, 0, 8, 5, None, None, 0, None) == _lib.AEM_OK
    assert L.aem_capacity_route_workspace(1000, 8) > 0


def test_pack_without_b200_is_unsupported():
    if aem.device_count() > 0:
        pytest.skip("a B200 is present")
    h = ctypes.c_void_p()
    w = np.zeros((4, 2), np.float32)
    st = aem.lib().aem_gate_pack(w.ctypes.data, None, 4, 2, 0, ctypes.byref(h))
    assert st == _lib.AEM_EUNSUPPORTED
    assert "sm_100" in _lib.last_error()


def test_gate_pack_rejects_too_many_experts():
    h = ctypes.c_void_p()
    w = np.zeros((4, 300), np.float32)
    st = aem.lib().aem_gate_pack(w.ctypes.data, None, 4, 300, 0, ctypes.byref(h))
    assert st == _lib.AEM_EINVAL
    assert "MAX_EXPERTS" in _lib.last_error()


def test_shim_validates_like_reference():
    from aethermoe_b200.kernels.fused_gating_metal import fused_gating
    from aethermoe_b200.kernels.quantized_gemm import fused_quantized_matmul
    h = np.zeros((2, 4), np.float32)
    with pytest.raises(ValueError):
        fused_gating(h, np.zeros((4, 300), np.float32), np.zeros(300, np.float32), 2)
    with pytest.raises(ValueError):
        fused_gating(h, np.zeros((4, 8), np.float32), np.zeros(8, np.float32), 9)
    with pytest.raises(ValueError):
        fused_quantized_matmul(h, np.zeros((5, 3), np.int8), np.ones((1, 3), np.float32))


def test_mlx_compat_surface():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "aethermoe_b200", "compat"))
    try:
        import mlx.core as mx
    finally:
        sys.path.pop(0)
    a = mx.array(np.arange(6, dtype=np.float32).reshape(2, 3))
    assert np.array(a @ a.T).shape == (2, 2)
    assert a.max(axis=0, keepdims=True).shape == (1, 3)
    assert np.array(mx.argsort(-a, axis=-1))[0].tolist() == [2, 1, 0]
    with pytest.raises(NotImplementedError):
        mx.fast.metal_kernel(name="x")
