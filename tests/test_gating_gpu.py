"""Fused gating on the B200 vs the oracle and the reference's test contracts.

Mirrors ``tests/python/test_gating_numerical.py`` and ``test_gating_property.py``
of the reference (same shapes, seeds, distributions and checks) and adds the
strict contract of this build: in EXACT mode indices are bit-identical --
order included -- to ``fused_kernel_simulation`` on every row, and weights
match within 1e-6.  Tolerance for values against the float32 reference tiers
is the reference's 1e-4 (``test_gating_numerical.py:30``).
"""
import numpy as np
import pytest

import aem_oracle as O
import cases

pytestmark = pytest.mark.gpu

TOLERANCE = 1e-4


@pytest.fixture(scope="module")
def shim(cuda):
    from aethermoe_b200.kernels import fused_gating_metal, reference_gating
    return fused_gating_metal, reference_gating


def _sets_equal_per_row(a, b):
    return all(set(x.tolist()) == set(y.tolist()) for x, y in zip(a, b))


@pytest.mark.parametrize("name", sorted(cases.gating_cases()))
def test_exact_matches_reference_simulation(shim, golden, name):
    fg, _ = shim
    h, w, b, k = cases.gating_cases()[name]
    idx, val = fg.fused_gating(h, w, b, k)
    assert idx.dtype == np.int32 and val.dtype == np.float32
    np.testing.assert_array_equal(idx, golden["gating"][f"{name}/sim_idx"])
    np.testing.assert_allclose(val, golden["gating"][f"{name}/sim_val"], rtol=0, atol=1e-6)


@pytest.mark.parametrize("mode", ["exact", "fast"])
@pytest.mark.parametrize("name", sorted(cases.nonfinite_gating_cases()))
def test_nonfinite_logits_match_reference_simulation(cuda, golden, name, mode):
    """NaN / +-inf logits select like np.argmax in fused_kernel_simulation
    (prototype/math_proto.py:38-42): first NaN first, lowest id on ties, a
    winner overwritten by -inf (so -inf ids repeat); values NaN-equal."""
    from aethermoe_b200 import _lib
    from aethermoe_b200.kernels.fused_gating_metal import gating
    h, w, b, k = cases.nonfinite_gating_cases()[name]
    md = _lib.GATING_EXACT if mode == "exact" else _lib.GATING_FAST
    idx, val = gating(h, w, b, k, mode=md)
    np.testing.assert_array_equal(idx, golden["gating"][f"{name}/sim_idx"])
    np.testing.assert_allclose(val, golden["gating"][f"{name}/sim_val"], rtol=0, atol=1e-6,
                               equal_nan=True)
    assert idx.min() >= 0 and idx.max() < w.shape[1]
    # the next choice for capacity rerouting follows the same order
    with np.errstate(invalid="ignore"):
        oidx, oval = O.fused_gating(h, w, b, k, extra=1)
    idx2, val2 = gating(h, w, b, k, mode=md, k_extra=1)
    np.testing.assert_array_equal(idx2, oidx)
    np.testing.assert_allclose(val2, oval, rtol=0, atol=1e-6, equal_nan=True)


def test_exact_c0(shim, golden):
    fg, _ = shim
    h, w, b, k = cases.c0_gating_inputs()
    idx, val = fg.fused_gating(h, w, b, k)
    np.testing.assert_array_equal(idx, golden["gating"]["c0/sim_idx"])
    np.testing.assert_allclose(val, golden["gating"]["c0/sim_val"], atol=1e-6)


@pytest.mark.parametrize("n_tokens,d_model,num_experts,k", [
    (8, 32, 8, 2), (16, 64, 16, 4), (1, 16, 8, 1), (32, 128, 32, 8)])
def test_fused_matches_reference_tier(shim, n_tokens, d_model, num_experts, k):
    fg, rg = shim
    h, w, b = cases._gating_inputs(np.random.default_rng(42), n_tokens, d_model, num_experts)
    ref_idx, ref_val = rg.reference_gating(h, w, b, k)
    idx, val = fg.fused_gating(h, w, b, k)
    assert _sets_equal_per_row(ref_idx, idx)
    np.testing.assert_allclose(np.sort(val, -1), np.sort(ref_val, -1), atol=TOLERANCE)


@pytest.mark.parametrize("n_tokens,d_model,num_experts,k", [(8, 32, 8, 2), (16, 64, 16, 4)])
def test_fused_matches_pytorch(shim, n_tokens, d_model, num_experts, k):
    import torch
    fg, _ = shim
    h, w, b = cases._gating_inputs(np.random.default_rng(7), n_tokens, d_model, num_experts)
    lg = torch.as_tensor(h) @ torch.as_tensor(w) + torch.as_tensor(b)
    pv, pi = torch.topk(lg, k, dim=-1)
    pv = torch.softmax(pv, -1).numpy()
    idx, val = fg.fused_gating(h, w, b, k)
    assert _sets_equal_per_row(idx, pi.numpy())
    np.testing.assert_allclose(np.sort(val, -1), np.sort(pv, -1), atol=TOLERANCE)


def test_rows_sum_to_one(shim):
    fg, _ = shim
    h, w, b = cases._gating_inputs(np.random.default_rng(1), 10, 32, 8)
    _, val = fg.fused_gating(h, w, b, 3)
    np.testing.assert_allclose(val.sum(-1), 1.0, atol=1e-5)


def test_property_invariants(shim):
    """Hypothesis-driven invariants (test_gating_property.py:36-91)."""
    from hypothesis import given, settings, strategies as st
    fg, _ = shim

    @st.composite
    def gating_inputs(draw):
        e = draw(st.integers(1, 32))
        k = draw(st.integers(1, e))
        n = draw(st.integers(1, 64))
        d = draw(st.integers(1, 64))
        seed = draw(st.integers(0, 2 ** 31 - 1))
        h, w, b = cases._gating_inputs(np.random.default_rng(seed), n, d, e)
        return h, w, b, k, e, n

    @given(gating_inputs())
    @settings(max_examples=100, deadline=None)
    def run(inp):
        h, w, b, k, e, n = inp
        idx, val = fg.fused_gating(h, w, b, k)
        assert idx.shape == (n, k) and val.shape == (n, k)
        assert np.allclose(val.sum(-1), 1.0, atol=1e-4)
        assert (idx >= 0).all() and (idx < e).all()
        for row in idx:
            assert len(set(row.tolist())) == len(row)
        assert (val >= 0).all() and (val <= 1.0 + 1e-6).all()
        oidx, oval = O.fused_gating(h, w, b, k)
        np.testing.assert_array_equal(idx, oidx)
        np.testing.assert_allclose(val, oval, atol=1e-6)

    run()


@pytest.mark.parametrize("e", [1, 2, 3, 7, 8, 9, 15, 16, 17, 31, 32])
def test_small_shape_grid(shim, e):
    """Exhaustive-ish small grid (the reference's crash bisector shapes)."""
    fg, _ = shim
    rng = np.random.default_rng(e)
    for n in (1, 2, 7, 64):
        for d in (1, 3, 31, 33, 64):
            for k in sorted({1, max(1, e // 2), e}):
                h, w, b = cases._gating_inputs(rng, n, d, e)
                idx, val = fg.fused_gating(h, w, b, k)
                oidx, oval = O.fused_gating(h, w, b, k)
                np.testing.assert_array_equal(idx, oidx, err_msg=f"n={n} d={d} e={e} k={k}")
                np.testing.assert_allclose(val, oval, atol=1e-6)


@pytest.mark.parametrize("name", sorted(cases.near_tie_gating_cases()))
def test_exact_mode_near_ties(shim, name):
    """Rows with adjacent-float32 logits: EXACT mode rounds every product and
    partial sum like the reference loop, so even these orders match."""
    fg, _ = shim
    h, w, b, k = cases.near_tie_gating_cases()[name]
    idx, _ = fg.fused_gating(h, w, b, k)
    oidx, _ = O.fused_gating(h, w, b, k)
    np.testing.assert_array_equal(idx, oidx)


def test_ties_pick_lowest_ids(shim):
    fg, _ = shim
    for name, want in (("tie_2_5", [2, 5]), ("tie_1_4", [1, 4])):
        h, w, b, k = cases.gating_cases()[name]
        idx, val = fg.fused_gating(h, w, b, k)
        assert idx[0].tolist() == want
        np.testing.assert_allclose(val[0], [0.5, 0.5], atol=1e-7)


def test_k_equals_e_and_single_expert(shim):
    fg, _ = shim
    h, w, b, k = cases.gating_cases()["k_eq_e"]
    idx, val = fg.fused_gating(h, w, b, k)
    for row in idx:
        assert set(row.tolist()) == set(range(8))
    h, w, b, k = cases.gating_cases()["single_expert"]
    idx, val = fg.fused_gating(h, w, b, k)
    assert (idx == 0).all() and np.allclose(val, 1.0, atol=1e-6)


def test_max_experts_and_topk(shim):
    fg, _ = shim
    h, w, b = cases._gating_inputs(np.random.default_rng(21), 40, 96, 256)
    for k in (1, 6, 64):
        idx, val = fg.fused_gating(h, w, b, k)
        oidx, oval = O.fused_gating(h, w, b, k)
        np.testing.assert_array_equal(idx, oidx)
        np.testing.assert_allclose(val, oval, atol=1e-6)


def _bf16_bits(x):
    f = O.bf16_round(x)
    return (f.view(np.uint32) >> 16).astype(np.uint16), f


@pytest.mark.parametrize("e,k", [(8, 2), (64, 6)])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_sweep_bit_exact(shim, e, k, dtype):
    """Gating sweep config: T in {1,16,128,1024,8192}, d=4096, E in {8,64},
    k in {2,6}; x ~ N(0,1) (float32 and bfloat16), W ~ N(0,1/d); duplicated
    weight columns plant exact logit ties.  Indices (k + the reroute choice)
    bit-exact on every row."""
    fg, _ = shim
    d = 4096
    rng = np.random.default_rng(1000 + e)
    w = (rng.normal(size=(d, e)) / np.sqrt(d)).astype(np.float32)
    w[:, e - 1] = w[:, 0]  # exact ties between experts 0 and e-1
    b = np.zeros(e, np.float32)
    x = rng.normal(size=(8192, d)).astype(np.float32)
    x[5] = x[4]  # duplicated token rows
    if dtype == "bf16":
        bits, x = _bf16_bits(x)
        xin = bits
    else:
        xin = x
    logits = O.gating_logits_seq(x, w, b)  # once for all T (rows are independent)
    for t in (1, 16, 128, 1024, 8192):
        idx, val = fg.gating(xin[:t], w, b, k, k_extra=1)
        oidx = O.topk_strict(logits[:t], k + 1).astype(np.int32)
        np.testing.assert_array_equal(idx, oidx, err_msg=f"T={t}")
        oval = O.softmax_selected(np.take_along_axis(logits[:t], oidx[:, :k].astype(np.int64), 1))
        np.testing.assert_allclose(val, oval, atol=1e-6)


def test_fast_mode_matches_on_certified_rows(shim):
    fg, _ = shim
    from aethermoe_b200 import _lib
    rng = np.random.default_rng(77)
    d, e, k = 2048, 64, 6
    x = rng.normal(size=(2048, d)).astype(np.float32)
    w = (rng.normal(size=(d, e)) / np.sqrt(d)).astype(np.float32)
    b = O.zipf_bias(e)
    idx, val = fg.gating(x, w, b, k, mode=_lib.GATING_FAST)
    oidx, oval = O.fused_gating(x, w, b, k)
    cert = O.certified_rows(x, w, b, k)
    assert cert.mean() > 0.8  # the forward-error bound is conservative
    for i in np.flatnonzero(cert):
        assert set(idx[i].tolist()) == set(oidx[i].tolist())
    np.testing.assert_allclose(np.sort(val, 1), np.sort(oval, 1), atol=1e-4)


def test_device_pointer_entry_point(cuda):
    """aem_gating on torch device buffers (bf16 activations), k_extra=1."""
    import torch
    from aethermoe_b200 import _lib
    rng = np.random.default_rng(5)
    n, d, e, k = 300, 512, 16, 4
    x = rng.normal(size=(n, d)).astype(np.float32)
    bits, xf = _bf16_bits(x)
    w = (rng.normal(size=(d, e)) / np.sqrt(d)).astype(np.float32)
    b = (rng.normal(size=e) * 0.1).astype(np.float32)
    gate = _lib.Gate(w, b, 0)
    xt = torch.from_numpy(bits.view(np.int16)).to(cuda).view(torch.bfloat16)
    idx = torch.empty((n, k + 1), dtype=torch.int32, device=cuda)
    val = torch.empty((n, k), dtype=torch.float32, device=cuda)
    st = _lib.lib().aem_gating(gate.handle, xt.data_ptr(), _lib.BF16, n, k, 1, _lib.GATING_EXACT,
                               idx.data_ptr(), val.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(st)
    torch.cuda.synchronize()
    oidx, oval = O.fused_gating(xf, w, b, k, extra=1)
    np.testing.assert_array_equal(idx.cpu().numpy(), oidx)
    np.testing.assert_allclose(val.cpu().numpy(), oval, atol=1e-6)


@pytest.mark.parametrize("e,k,d", [(17, 3, 37), (33, 6, 64), (64, 6, 130), (8, 2, 96), (5, 5, 16)])
def test_many_tokens_kernel_bit_exact(shim, e, k, d):
    """More than 4096 tokens take the large-batch configuration (several
    tokens per lane group); padding of E and D, k == E, and the reroute
    choice included."""
    fg, _ = shim
    h, w, b = cases._gating_inputs(np.random.default_rng(e * 100 + d), 5000, d, e)
    w[:, e - 1] = w[:, 0]
    b[e - 1] = b[0]  # exact tie between the first and the last expert
    extra = 1 if k < e else 0
    idx, val = fg.gating(h, w, b, k, k_extra=extra)
    oidx, oval = O.fused_gating(h, w, b, k, extra=extra)
    np.testing.assert_array_equal(idx, oidx)
    np.testing.assert_allclose(val, oval, atol=1e-6)


@pytest.mark.parametrize("e", [100, 200, 256])
@pytest.mark.parametrize("t", [7, 3000, 9000])
def test_wide_gates_bit_exact(shim, e, t):
    """128- and 256-expert gates across the few-token (<= 4096) and
    many-token configurations, with an exact tie and the reroute choice."""
    fg, _ = shim
    h, w, b = cases._gating_inputs(np.random.default_rng(e + t), t, 72, e)
    w[:, e - 1] = w[:, 3]
    b[e - 1] = b[3]
    idx, val = fg.gating(h, w, b, 4, k_extra=1)
    oidx, oval = O.fused_gating(h, w, b, 4, extra=1)
    np.testing.assert_array_equal(idx, oidx)
    np.testing.assert_allclose(val, oval, atol=1e-6)
