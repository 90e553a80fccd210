"""Asynchronous host-buffer steps (aem_moe_submit_host + aem_context_wait):
a stream of steps with uploads and downloads overlapping the compute gives
the same outputs as the synchronous aem_moe_forward_host, step by step."""
import ctypes

import numpy as np
import pytest

import aem_oracle as O

pytestmark = pytest.mark.gpu


def _layer(rng, d=256, f=512, e=16, k=4, cap=60):
    from aethermoe_b200.moe import MoELayer
    qu = rng.integers(-127, 128, size=(e, d, f), dtype=np.int8)
    qd = rng.integers(-127, 128, size=(e, f, d), dtype=np.int8)
    su = (rng.random(size=(e, 1, f)) * 1e-4 + 2e-4).astype(np.float32)
    sd = (rng.random(size=(e, 1, d)) * 1e-4 + 2e-4).astype(np.float32)
    gw = (rng.normal(size=(d, e)) / np.sqrt(d)).astype(np.float32)
    return MoELayer(gw, O.zipf_bias(e), qu, su, qd, sd, k, capacity=cap)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_submitted_steps_equal_synchronous_steps(cuda, dtype):
    import torch
    from aethermoe_b200 import _lib
    rng = np.random.default_rng(23)
    layer = _layer(rng)
    T, d = 200, layer.d_model
    ctx = _lib.context(0)
    L = _lib.lib()
    code = _lib.F32 if dtype == "f32" else _lib.BF16
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    xs = [torch.randn((T, d), generator=torch.Generator().manual_seed(i)).to(tdt).pin_memory()
          for i in range(3)]
    outs = [torch.empty((T, d), dtype=torch.float32).pin_memory() for _ in range(7)]
    tickets = []
    for i in range(7):  # more steps than slots: submits wait for the oldest
        t = ctypes.c_uint64()
        _lib.check(L.aem_moe_submit_host(ctx, layer.handle, xs[i % 3].data_ptr(), code, T,
                                         outs[i].data_ptr(), _lib.F32, ctypes.byref(t)))
        tickets.append(t.value)
    assert tickets == sorted(tickets) and len(set(tickets)) == 7
    for t in reversed(tickets):  # any order; already-finished steps return at once
        _lib.check(L.aem_context_wait(ctx, t))
    for i in range(7):
        ref = torch.empty((T, d), dtype=torch.float32)
        _lib.check(L.aem_moe_forward_host(ctx, layer.handle, xs[i % 3].data_ptr(), code, T,
                                          ref.data_ptr(), _lib.F32))
        np.testing.assert_allclose(outs[i].numpy(), ref.numpy(), rtol=1e-5, atol=1e-6)
    # a ticket that was never handed out is an argument error
    assert L.aem_context_wait(ctx, tickets[-1] + 100) == 1
    layer.close()
