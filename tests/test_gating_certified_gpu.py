"""CERTIFIED gating on the B200: indices bit-identical to EXACT (and so to
``fused_kernel_simulation``, prototype/math_proto.py:19-50) on every row.

Fast logits carry a rigorous bound on their distance from the EXACT logits;
rows whose selection the bound cannot decide -- near ties, exact ties, NaN,
+-inf -- are recomputed on the device with the EXACT arithmetic.  Checked
here: indices against EXACT across the small-batch (d split over threads)
and large-batch kernels, values within float32 rounding, the recomputation
firing on the reference's near-tie fixtures and producing EXACT's output
bit for bit there, and the bound certifying nearly every ordinary row.
"""
import numpy as np
import pytest

import aem_oracle as O
import cases

pytestmark = pytest.mark.gpu


def _run(cuda, gate, x, k, extra, mode):
    """aem_gating on device buffers; x float32 numpy or (uint16 bf16 bits)."""
    import torch
    from aethermoe_b200 import _lib
    n = x.shape[0]
    if x.dtype == np.uint16:
        xt = torch.from_numpy(x.view(np.int16)).to(cuda).view(torch.bfloat16)
        code = _lib.BF16
    else:
        xt = torch.from_numpy(np.ascontiguousarray(x)).to(cuda)
        code = _lib.F32
    idx = torch.empty((n, k + extra), dtype=torch.int32, device=cuda)
    val = torch.empty((n, k), dtype=torch.float32, device=cuda)
    _lib.check(_lib.lib().aem_gating(gate.handle, xt.data_ptr(), code, n, k, extra, mode,
                                     idx.data_ptr(), val.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream), "aem_gating")
    torch.cuda.synchronize()
    _lib.check(_lib.lib().aem_device_status(None), "aem_device_status")
    return idx.cpu().numpy(), val.cpu().numpy()


def _bf16_bits(x):
    f = O.bf16_round(x)
    return (f.view(np.uint32) >> 16).astype(np.uint16), f


@pytest.mark.parametrize("e,k,d,ts", [
    (8, 2, 4096, (1, 7, 128, 512, 513, 3000)),     # d-split kernel, then the large one
    (64, 6, 2048, (1, 100, 600, 16384)),           # the layer bench's gate shape
    (256, 8, 96, (5, 700)),
    (17, 3, 37, (9, 5000)),                        # padded E and D
    (5, 5, 16, (3, 40)),                           # k == E
])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_certified_indices_equal_exact(cuda, e, k, d, ts, dtype):
    from aethermoe_b200 import _lib
    rng = np.random.default_rng(e * 1000 + d)
    t_max = max(ts)
    x = rng.normal(size=(t_max, d)).astype(np.float32)
    w = (rng.normal(size=(d, e)) / np.sqrt(d)).astype(np.float32)
    b = O.zipf_bias(e) if e >= 8 else np.zeros(e, np.float32)
    if e > 5:
        w[:, e - 1] = w[:, 0]  # an exact tie: never certified, always recomputed
        b[e - 1] = b[0]
    if dtype == "bf16":
        x, xf = _bf16_bits(x)
    else:
        xf = x
    gate = _lib.Gate(w, b, 0)
    extra = 1 if k < e else 0
    for t in ts:
        before = gate.fallback_rows()
        ci, cv = _run(cuda, gate, x[:t], k, extra, _lib.GATING_CERTIFIED)
        ei, ev = _run(cuda, gate, x[:t], k, extra, _lib.GATING_EXACT)
        np.testing.assert_array_equal(ci, ei, err_msg=f"T={t}")
        np.testing.assert_allclose(cv, ev, rtol=1e-5, atol=1e-6, err_msg=f"T={t}")
        fell = gate.fallback_rows() - before
        assert 0 <= fell <= t
    last = ci  # the largest call's indices
    if e == 64:
        # without the planted tie the bound decides ordinary rows: only near
        # ties fall back (both kernels: 100 rows d-split, 16384 rows large)
        w2 = (rng.normal(size=(d, e)) / np.sqrt(d)).astype(np.float32)
        gate2 = _lib.Gate(w2, O.zipf_bias(e), 0)
        for t in (100, 16384):
            before = gate2.fallback_rows()
            ci, _ = _run(cuda, gate2, x[:t], k, extra, _lib.GATING_CERTIFIED)
            ei, _ = _run(cuda, gate2, x[:t], k, extra, _lib.GATING_EXACT)
            np.testing.assert_array_equal(ci, ei, err_msg=f"untied T={t}")
            fell = gate2.fallback_rows() - before
            assert fell < 0.1 * t, f"untied T={t}: {fell} rows recomputed"
    # against the oracle as well (every row of the largest call)
    oidx, _ = O.fused_gating(xf[:t_max], w, b, k, extra=extra)
    np.testing.assert_array_equal(last, oidx)


@pytest.mark.parametrize("name", sorted(cases.near_tie_gating_cases()))
def test_certified_recomputes_near_ties(cuda, name):
    """The reference's near-tie fixtures (logits one float32 ulp apart): the
    bound cannot order them, so those rows are recomputed -- and come out
    exactly as EXACT writes them."""
    from aethermoe_b200 import _lib
    h, w, b, k = cases.near_tie_gating_cases()[name]
    h = np.ascontiguousarray(h, dtype=np.float32)
    gate = _lib.Gate(w, b, 0)
    before = gate.fallback_rows()
    ci, cv = _run(cuda, gate, h, k, 0, _lib.GATING_CERTIFIED)
    assert gate.fallback_rows() - before > 0
    ei, ev = _run(cuda, gate, h, k, 0, _lib.GATING_EXACT)
    np.testing.assert_array_equal(ci, ei)
    oidx, _ = O.fused_gating(h, w, b, k)
    np.testing.assert_array_equal(ci, oidx)


@pytest.mark.parametrize("name", sorted(cases.nonfinite_gating_cases()))
def test_certified_nonfinite_rows_are_exact(cuda, golden, name):
    """NaN / +-inf logits are never certified: the recomputation writes the
    reference simulation's selection and values (NaN-equal)."""
    from aethermoe_b200 import _lib
    h, w, b, k = cases.nonfinite_gating_cases()[name]
    h = np.ascontiguousarray(h, dtype=np.float32)
    gate = _lib.Gate(w, b, 0)
    with np.errstate(invalid="ignore"):
        ci, cv = _run(cuda, gate, h, k, 0, _lib.GATING_CERTIFIED)
    np.testing.assert_array_equal(ci, golden["gating"][f"{name}/sim_idx"])
    np.testing.assert_allclose(cv, golden["gating"][f"{name}/sim_val"], rtol=0, atol=1e-6,
                               equal_nan=True)


def test_certified_moe_layer_routes_like_exact(cuda):
    """A MoE layer in CERTIFIED mode routes every unit exactly as in EXACT
    mode (same gating indices, so the same capacity routing) and its output
    agrees within the layer tolerance."""
    import torch
    from aethermoe_b200 import _lib
    from aethermoe_b200.moe import MoELayer
    rng = np.random.default_rng(3)
    d, f, e, k, t = 256, 384, 16, 4, 700
    gw = (rng.normal(size=(d, e)) / np.sqrt(d)).astype(np.float32)
    gb = O.zipf_bias(e)
    qu = torch.randint(-127, 128, (e, d, f), dtype=torch.int8, device=cuda)
    qd = torch.randint(-127, 128, (e, f, d), dtype=torch.int8, device=cuda)
    up = _lib.DeviceQWeight(qu, torch.full((e, f), 1e-3, device=cuda))
    dn = _lib.DeviceQWeight(qd, torch.full((e, d), 1e-3, device=cuda))
    x = torch.randn(t, d, device=cuda).to(torch.bfloat16)
    outs, routes, layers = [], [], []
    for mode in (_lib.GATING_EXACT, _lib.GATING_CERTIFIED):
        # both layers share the packed weights (a layer frees what it was
        # given when it goes), so both stay alive to the end of the test
        layer = MoELayer(gw, gb, up, None, dn, None, k, capacity=int(1.25 * t * k / e),
                         gating_mode=mode)
        layers.append(layer)
        o = torch.empty((t, d), dtype=torch.float32, device=cuda)
        layer.forward(x, out=o)
        torch.cuda.synchronize()
        outs.append(o.cpu().numpy())
        routes.append([a.cpu().numpy() for a in layer.last_routing(t)])
    np.testing.assert_array_equal(routes[0][0], routes[1][0])  # gating indices
    np.testing.assert_array_equal(routes[0][2], routes[1][2])  # effective experts
    np.testing.assert_allclose(outs[1], outs[0], rtol=1e-3, atol=1e-3)
