"""Seeded input cases shared by the golden-fixture generator and the tests.

Shapes, seeds and value distributions follow the reference's own tests
(``tests/python/test_math_prototype.py``, ``test_gating_numerical.py``,
``test_gating_property.py``, ``test_quantized_gemm.py``,
``tests/test_orchestration.cpp``) and the CPU-runnable config
(T=256, d=512, E=8, top-2, W_gate ~ N(0, 1/d), expert GEMM d -> 1024 with
weights ~ N(0, 0.02), seed 0).
"""
from __future__ import annotations

import numpy as np


def _gating_inputs(rng, n, d, e, w_scale=0.1, b_scale=0.01):
    h = rng.normal(size=(n, d)).astype(np.float32)
    w = (rng.normal(size=(d, e)) * w_scale).astype(np.float32)
    b = (rng.normal(size=(e,)) * b_scale).astype(np.float32)
    return h, w, b


def gating_cases():
    c = {}
    c["proto_seed0"] = _gating_inputs(np.random.default_rng(0), 5, 16, 8) + (3,)
    for n, d, e, k in [(8, 32, 8, 2), (16, 64, 16, 4), (1, 16, 8, 1), (32, 128, 32, 8)]:
        c[f"numerical_{n}_{d}_{e}_{k}"] = _gating_inputs(np.random.default_rng(42), n, d, e) + (k,)
    for n, d, e, k in [(8, 32, 8, 2), (16, 64, 16, 4)]:
        c[f"torch_{n}_{d}_{e}_{k}"] = _gating_inputs(np.random.default_rng(7), n, d, e) + (k,)
    # exact ties in the bias with zero activations
    for name, d, e, hot, val in [("tie_2_5", 8, 8, (2, 5), 5.0), ("tie_1_4", 8, 6, (1, 4), 3.0)]:
        h = np.zeros((1, d), np.float32)
        w = np.zeros((d, e), np.float32)
        b = np.zeros((e,), np.float32)
        b[list(hot)] = val
        c[name] = (h, w, b, 2)
    rng = np.random.default_rng(3)
    h = rng.normal(size=(4, 16)).astype(np.float32)
    w = rng.normal(size=(16, 8)).astype(np.float32)
    b = rng.normal(size=(8,)).astype(np.float32)
    c["k_eq_e"] = (h, w, b, 8)
    rng = np.random.default_rng(4)
    c["single_expert"] = (rng.normal(size=(5, 16)).astype(np.float32),
                          rng.normal(size=(16, 1)).astype(np.float32),
                          rng.normal(size=(1,)).astype(np.float32), 1)
    c["one_token"] = (np.random.default_rng(5).normal(size=(1, 32)).astype(np.float32),
                      np.random.default_rng(6).normal(size=(32, 8)).astype(np.float32),
                      np.zeros((8,), np.float32), 2)
    c["large_batch"] = _gating_inputs(np.random.default_rng(8), 2048, 64, 16) + (4,)
    # duplicated weight columns: exact logit ties between experts 3/11 and 5/6
    h, w, b = _gating_inputs(np.random.default_rng(9), 64, 48, 16)
    w[:, 11] = w[:, 3]
    w[:, 6] = w[:, 5]
    b[11] = b[3]
    b[6] = b[5]
    c["dup_columns"] = (h, w, b, 4)
    return c


# (n, d, e, k, seed) of _gating_inputs draws holding a row whose k-th and
# (k+1)-th (or two neighbouring) logits are adjacent float32 values: the
# sequential float32 sum and a fused multiply-add sum order them differently,
# so these cases tell the two apart (found by a random sweep of 86895 draws).
NEAR_TIE_GATING = [(38, 44, 19, 12, 1595066796), (46, 58, 20, 17, 2056578468),
                   (48, 32, 23, 18, 115215509), (38, 61, 29, 19, 1082537402),
                   (36, 7, 30, 24, 608740648)]


def near_tie_gating_cases():
    return {f"near_tie_{n}_{d}_{e}_{k}": _gating_inputs(np.random.default_rng(seed), n, d, e) + (k,)
            for n, d, e, k, seed in NEAR_TIE_GATING}


def nonfinite_gating_cases():
    """Rows whose logits hold NaN, +inf or -inf (through the bias or the
    activations).  The reference's selection is np.argmax
    (prototype/math_proto.py:38-42): the first NaN wins, ties go to the lowest
    id, and a winner is overwritten with -inf rather than removed."""
    c = {}
    h, w, b = _gating_inputs(np.random.default_rng(21), 6, 16, 8)
    b[[3, 5]] = np.nan
    c["nan_bias"] = (h, w, b, 3)
    h, w, b = _gating_inputs(np.random.default_rng(22), 4, 16, 8)
    b[:] = -np.inf
    c["neg_inf_all"] = (h, w, b, 3)
    h, w, b = _gating_inputs(np.random.default_rng(23), 4, 16, 8)
    b[:] = -np.inf
    b[4] = 0.5
    c["neg_inf_but_one"] = (h, w, b, 3)
    h, w, b = _gating_inputs(np.random.default_rng(24), 4, 16, 8)
    b[[1, 6]] = np.inf
    c["pos_inf_pair"] = (h, w, b, 3)
    h, w, b = _gating_inputs(np.random.default_rng(25), 5, 16, 8)
    h[1, 7] = np.nan
    h[3, :] = np.nan
    c["nan_rows"] = (h, w, b, 3)
    h, w, b = _gating_inputs(np.random.default_rng(26), 5, 16, 8)
    w[0, :] = np.array([1.0, -1.0, 0.0, 2.0, -0.5, 0.0, 1.0, -3.0], np.float32)
    h[0, 0] = np.inf   # logits +inf, -inf or NaN (inf * 0) by the sign of w[0, e]
    h[2, 0] = -np.inf
    c["inf_activation"] = (h, w, b, 4)
    return c


def c0_inputs():
    """CPU-runnable config: x [256,512], W_gate [512,8] ~ N(0,1/d), bias 0,
    expert weight [512,1024] ~ N(0,0.02); one generator, seed 0."""
    rng = np.random.default_rng(0)
    t, d, e, n = 256, 512, 8, 1024
    x = rng.normal(size=(t, d)).astype(np.float32)
    gw = (rng.normal(size=(d, e)) / np.sqrt(d)).astype(np.float32)
    gb = np.zeros((e,), np.float32)
    we = (rng.normal(size=(d, n)) * 0.02).astype(np.float32)
    return x, gw, gb, we


def c0_gating_inputs():
    x, gw, gb, _ = c0_inputs()
    return x, gw, gb, 2


def c0_quant_inputs():
    x, _, _, we = c0_inputs()
    return we, x


def quant_cases():
    c = {}
    rng = np.random.default_rng(1)
    w = rng.normal(size=(64, 8)).astype(np.float32)
    x = np.random.default_rng(101).normal(size=(4, 64)).astype(np.float32)
    c["proto_64x8"] = (w, x)
    rng = np.random.default_rng(2)
    w = rng.normal(size=(32, 8)).astype(np.float32)
    x = rng.normal(size=(4, 32)).astype(np.float32)
    c["proto_32x8"] = (w, x)
    for n, d, e in [(4, 32, 8), (16, 64, 16), (1, 16, 4)]:
        rng = np.random.default_rng(11)
        x = rng.normal(size=(n, d)).astype(np.float32)
        w = rng.normal(size=(d, e)).astype(np.float32)
        c[f"gemm_{n}_{d}_{e}"] = (w, x)
    w = np.zeros((16, 4), np.float32)
    w[:, 1] = np.random.default_rng(14).normal(size=16)
    x = np.random.default_rng(15).normal(size=(4, 16)).astype(np.float32)
    c["zero_column"] = (w, x)
    return c


def routing_cases():
    """``name -> (primary, secondary, batch_position, capacity, num_experts, num_shards)``."""
    c = {}
    rng = np.random.default_rng(11)
    n = 500
    prim = np.array([0 if i < 400 else 1 + i % 15 for i in range(n)])
    sec = rng.integers(1, 16, size=n)
    c["overflow_400_of_500"] = (prim, sec, np.arange(n), 20, 16, 4)
    rng = np.random.default_rng(10)
    c["unlimited_random"] = (rng.integers(0, 16, 500), rng.integers(0, 16, 500), np.arange(500),
                             None, 16, 4)
    rng = np.random.default_rng(12)
    n = 800
    hot = rng.random(n) < 0.9
    prim = np.where(hot, 0, 1 + np.arange(n) % 31)
    sec = rng.integers(1, 32, size=n)
    c["stress_90pct"] = (prim, sec, np.arange(n), 15, 32, 8)
    for i, (n, e, cap) in enumerate([(1, 3, 0), (17, 3, 2), (1000, 16, 40), (5000, 64, 60),
                                     (4096, 8, 300)]):
        rng = np.random.default_rng(100 + i)
        z = rng.zipf(1.6, size=n) % e
        c[f"perm_{n}_{e}_{cap}"] = (z, rng.integers(0, e, size=n), rng.permutation(n), cap, e, 1)
    return c
