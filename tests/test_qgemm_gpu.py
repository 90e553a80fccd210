"""INT8 quantisation and the tcgen05 INT8-weight GEMM vs the oracle.

Mirrors ``tests/python/test_quantized_gemm.py`` and ``test_math_prototype.py``
of the reference; quantisation must be bit-exact, GEMM outputs within
``|gpu - ref| <= 1e-3 + 1e-3 * |ref|`` of the float64 oracle (the reference's
``FUSED_VS_NAIVE_TOLERANCE = 1e-3`` as rtol and atol).
"""
import numpy as np
import pytest

import aem_oracle as O
import cases

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-3


def _close(got, ref, rtol=RTOL, atol=ATOL):
    err = np.abs(np.asarray(got, np.float64) - ref)
    bound = atol + rtol * np.abs(ref)
    assert np.all(err <= bound), f"max excess {(err - bound).max():.3e}, max err {err.max():.3e}"


@pytest.fixture(scope="module")
def qg(cuda):
    from aethermoe_b200.kernels import quantized_gemm
    return quantized_gemm


@pytest.mark.parametrize("name", sorted(cases.quant_cases()))
def test_quantize_bit_exact(qg, golden, name):
    w, x = cases.quant_cases()[name]
    q, s = qg.quantize_weights(w)
    np.testing.assert_array_equal(q, golden["quant"][f"{name}/q"])
    np.testing.assert_array_equal(s, golden["quant"][f"{name}/scale"])


def test_quantize_c0_and_large(qg, golden):
    import hashlib
    w, x = cases.c0_quant_inputs()
    q, s = qg.quantize_weights(w)
    assert hashlib.sha256(q.tobytes()).hexdigest() == str(golden["quant"]["c0/q_digest"])
    assert hashlib.sha256(s.tobytes()).hexdigest() == str(golden["quant"]["c0/scale_digest"])
    rng = np.random.default_rng(3)
    w = (rng.normal(size=(4096, 1536)) * 0.02).astype(np.float32)
    w[:, 7] = 0.0
    q, s = qg.quantize_weights(w)
    oq, os_ = O.quantize_int8(w)
    np.testing.assert_array_equal(q, oq)
    np.testing.assert_array_equal(s, os_)


@pytest.mark.parametrize("name", sorted(cases.quant_cases()))
def test_fused_matches_reference_perentry(qg, golden, name):
    w, x = cases.quant_cases()[name]
    q, s = O.quantize_int8(w)
    out = qg.fused_quantized_matmul(x, q, s)
    _close(out, golden["quant"][f"{name}/perentry"])


@pytest.mark.parametrize("n_tokens,d_model,num_experts", [(4, 32, 8), (16, 64, 16), (1, 16, 4)])
def test_fused_matches_naive(qg, n_tokens, d_model, num_experts):
    rng = np.random.default_rng(11)
    x = rng.normal(size=(n_tokens, d_model)).astype(np.float32)
    w = rng.normal(size=(d_model, num_experts)).astype(np.float32)
    q, s = qg.quantize_weights(w)
    naive = qg.naive_quantized_matmul(x, q, s)
    fused = qg.fused_quantized_matmul(x, q, s)
    assert np.allclose(naive, fused, atol=1e-3), np.abs(naive - fused).max()


def test_quantized_output_within_bound_of_true_fp32(qg):
    rng = np.random.default_rng(13)
    x = rng.normal(size=(8, 64)).astype(np.float32)
    w = rng.normal(size=(64, 16)).astype(np.float32)
    q, s = qg.quantize_weights(w)
    out = qg.fused_quantized_matmul(x, q, s)
    rel = np.abs(out - x @ w) / (np.abs(x @ w) + 1e-6)
    assert rel.mean() < 0.35


def test_all_zero_weight_column(qg):
    d, e = 16, 4
    w = np.zeros((d, e), np.float32)
    w[:, 1] = np.random.default_rng(14).normal(size=d)
    q, s = qg.quantize_weights(w)
    x = np.random.default_rng(15).normal(size=(4, d)).astype(np.float32)
    out = qg.fused_quantized_matmul(x, q, s)
    assert not np.isnan(out).any()
    assert np.allclose(out[:, 0], 0.0, atol=1e-5)


@pytest.mark.parametrize("m,k,n", [(1, 24, 40), (5, 40, 130), (3, 16, 8), (33, 48, 300),
                                   (7, 272, 129), (130, 64, 256), (257, 128, 384)])
def test_odd_shapes(qg, m, k, n):
    """Tails in every dimension; K % 16 != 0 takes the CUDA-core path."""
    rng = np.random.default_rng(m * 1000 + k + n)
    x = rng.normal(size=(m, k)).astype(np.float32)
    q, s = O.quantize_int8((rng.normal(size=(k, n)) * 0.02).astype(np.float32))
    _close(qg.fused_quantized_matmul(x, q, s), O.qgemm(x, q, s))


@pytest.fixture(scope="module")
def sweep_weight():
    """K=4096, N=14336, W ~ N(0, 0.02) quantised per output channel, and the
    float64 dequantised copy the oracle multiplies with."""
    rng = np.random.default_rng(2024)
    w = (rng.normal(size=(4096, 14336)) * 0.02).astype(np.float32)
    q, s = O.quantize_int8(w)
    return q, s, O.dequantize_int8(q, s).astype(np.float64)


@pytest.mark.parametrize("m", [1, 8, 64, 512, 4096])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_sweep(qg, sweep_weight, m, dtype):
    """INT8 GEMM sweep config: M in {1,8,64,512,4096}, K=4096, N=14336;
    float32 / bfloat16 x ~ N(0,1).  Rows checked against the float64 oracle:
    all for M <= 64, 64 sampled rows above (the same kernel tiles computed them)."""
    q, s, wd = sweep_weight
    rng = np.random.default_rng(m)
    x = rng.normal(size=(m, q.shape[0])).astype(np.float32)
    if dtype == "bf16":
        xf = O.bf16_round(x)
        out = _bf16_gemm(q, s, (xf.view(np.uint32) >> 16).astype(np.uint16))
    else:
        xf = x
        out = qg.fused_quantized_matmul(x, q, s)
    rows = np.arange(m) if m <= 64 else np.unique(np.r_[0, m - 1, rng.integers(0, m, 62)])
    _close(out[rows], xf[rows].astype(np.float64) @ wd)


def _bf16_gemm(q, s, xbits):
    """aem_qgemm on device with bf16 activations (torch buffers)."""
    import torch
    from aethermoe_b200 import _lib
    w = _lib.QWeight(q, s, 0)
    dev = torch.device("cuda", 0)
    xt = torch.from_numpy(xbits.view(np.int16)).to(dev).view(torch.bfloat16)
    out = torch.empty((xbits.shape[0], q.shape[1]), dtype=torch.float32, device=dev)
    _lib.check(_lib.lib().aem_qgemm(w.handle, 0, xt.data_ptr(), _lib.BF16, xbits.shape[0],
                                    out.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_groups_select_their_weights(cuda):
    """A packed weight with G groups; aem_qgemm(group=g) uses group g."""
    import torch
    from aethermoe_b200 import _lib
    rng = np.random.default_rng(9)
    g, kdim, n, m = 5, 256, 384, 37
    q = rng.integers(-127, 128, size=(g, kdim, n), dtype=np.int8)
    s = (rng.random(size=(g, n)) * 1e-3 + 1e-4).astype(np.float32)
    w = _lib.QWeight(q, s, 0)
    x = rng.normal(size=(m, kdim)).astype(np.float32)
    xt = torch.from_numpy(x).to(cuda)
    out = torch.empty((m, n), dtype=torch.float32, device=cuda)
    for grp in (0, 3, 4):
        _lib.check(_lib.lib().aem_qgemm(w.handle, grp, xt.data_ptr(), _lib.F32, m, out.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        _close(out.cpu().numpy(), O.qgemm(x, q[grp], s[grp:grp + 1]))


def _set_form(form):
    """single: single SMs, converted weights in shared memory; pairs: SM
    pairs from 64-row token tiles on; tmem_a: single SMs with the converted
    weights in tensor memory for every tile (the MMA reads A from TMEM; token
    tiles capped at 192 rows; also taken by calls of at most 32 rows);
    auto: the library's own choice."""
    from aethermoe_b200 import _lib
    L = _lib.lib()
    pairs, tmem_a = {"single": (0, 0), "pairs": (1, 0), "tmem_a": (0, 1), "auto": (-1, -1)}[form]
    _lib.check(L.aem_set_gemm_pairs(pairs))
    _lib.check(L.aem_set_gemm_tmem_a(tmem_a))


@pytest.fixture(params=["single", "pairs", "tmem_a"])
def gemm_form(cuda, request):
    """Runs a test with each form of the tensor-core GEMM (see _set_form)."""
    _set_form(request.param)
    yield request.param
    _set_form("auto")


@pytest.fixture(params=["stream", "tmem_a"])
def small_form(cuda, request):
    """Few-row calls: the weight-stream kernel (default) and the tensor-core
    kernel with weights in TMEM."""
    _set_form("auto" if request.param == "stream" else "tmem_a")
    yield request.param
    _set_form("auto")


@pytest.mark.parametrize("m", [1, 8, 64, 512])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_sweep_tmem_a(qg, sweep_weight, m, dtype):
    """The sweep shape (K=4096, N=14336) with the converted weights in TMEM
    for every tile, float32 (hi + lo) and bf16 activations."""
    _set_form("tmem_a")
    try:
        test_sweep(qg, sweep_weight, m, dtype)
    finally:
        _set_form("auto")


@pytest.mark.parametrize("tile", [256, 128, 64])
@pytest.mark.parametrize("mode", ["relu_bf16", "scaled_add"])
def test_grouped_ragged_tiles(cuda, gemm_form, tile, mode):
    """aem_grouped_qgemm over ragged groups (empty, 1 row, 191-193 rows,
    several tiles) at token tiles 256, 128 and 64, on single SMs and on SM
    pairs; a partial output-channel block (N = 300: three 128-channel blocks,
    so the last SM pair has a block past N).
    relu_bf16: the up projection's epilogue; scaled_add: the down
    projection's (gate-weight row scale, float32 red.add into mapped rows)."""
    import torch
    from aethermoe_b200 import _lib
    rng = np.random.default_rng(tile + len(mode))
    sizes = [0, 1, 15, 191, 192, 193, 700, 37]
    G, K, N = len(sizes), 448, 300
    q = rng.integers(-127, 128, size=(G, K, N), dtype=np.int8)
    s = (rng.random(size=(G, N)) * 1e-3 + 1e-4).astype(np.float32)
    w = _lib.QWeight(q, s, 0)
    rows = np.r_[0, np.cumsum(sizes)].astype(np.int32)
    M = int(rows[-1])
    x = O.bf16_round(rng.normal(size=(M, K)).astype(np.float32))
    xbits = (x.view(np.uint32) >> 16).astype(np.uint16)
    xt = torch.from_numpy(xbits.view(np.int16)).to(cuda).view(torch.bfloat16)
    rt = torch.from_numpy(rows).to(cuda)
    ref = np.zeros((M, N))
    for g in range(G):
        a, b = rows[g], rows[g + 1]
        ref[a:b] = x[a:b].astype(np.float64) @ (q[g].astype(np.float64) * s[g].astype(np.float64))
    stream = torch.cuda.current_stream().cuda_stream
    if mode == "relu_bf16":
        out = torch.zeros((M, N), dtype=torch.bfloat16, device=cuda)
        _lib.check(_lib.lib().aem_grouped_qgemm(w.handle, rt.data_ptr(), G, xt.data_ptr(), M,
                                                out.data_ptr(), _lib.BF16, N, 1, 0, None, None,
                                                tile, 1, stream), "aem_grouped_qgemm")
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        want = O.bf16_round(np.maximum(ref, 0.0).astype(np.float32))
        # bf16 output: within one bf16 rounding of the float64 result
        _close(got, np.maximum(ref, 0.0), rtol=2 ** -8 + 1e-3, atol=1e-3)
        assert np.mean(got == want) > 0.99
    else:
        rmap = rng.permutation(M).astype(np.int32)
        rscale = (rng.random(M) + 0.5).astype(np.float32)
        base = rng.normal(size=(M, N)).astype(np.float32)
        out = torch.from_numpy(base.copy()).to(cuda)
        mt = torch.from_numpy(rmap).to(cuda)
        st = torch.from_numpy(rscale).to(cuda)
        _lib.check(_lib.lib().aem_grouped_qgemm(w.handle, rt.data_ptr(), G, xt.data_ptr(), M,
                                                out.data_ptr(), _lib.F32, N, 0, 1, mt.data_ptr(),
                                                st.data_ptr(), tile, 1, stream), "aem_grouped_qgemm")
        torch.cuda.synchronize()
        want = base.astype(np.float64).copy()
        want[rmap] += ref * rscale[:, None].astype(np.float64)
        _close(out.cpu().numpy(), want)


@pytest.mark.parametrize("mode", ["relu_bf16", "scaled_add"])
def test_grouped_decode_sizes(cuda, small_form, mode):
    """At most 4 rows (decode sizes) take the CUDA-core path: groups of 0-2
    rows, a partial output-channel block, K not a multiple of 64."""
    import torch
    from aethermoe_b200 import _lib
    rng = np.random.default_rng(31 + len(mode))
    sizes = [0, 1, 2, 0, 1]
    G, K, N = len(sizes), 200, 300
    q = rng.integers(-127, 128, size=(G, K, N), dtype=np.int8)
    s = (rng.random(size=(G, N)) * 1e-3 + 1e-4).astype(np.float32)
    w = _lib.QWeight(q, s, 0)
    rows = np.r_[0, np.cumsum(sizes)].astype(np.int32)
    M = int(rows[-1])
    x = O.bf16_round(rng.normal(size=(M, K)).astype(np.float32))
    xt = torch.from_numpy((x.view(np.uint32) >> 16).astype(np.uint16).view(np.int16)).to(cuda)
    xt = xt.view(torch.bfloat16)
    rt = torch.from_numpy(rows).to(cuda)
    ref = np.zeros((M, N))
    for g in range(G):
        a, b = rows[g], rows[g + 1]
        ref[a:b] = x[a:b].astype(np.float64) @ (q[g].astype(np.float64) * s[g].astype(np.float64))
    stream = torch.cuda.current_stream().cuda_stream
    if mode == "relu_bf16":
        out = torch.zeros((M, N), dtype=torch.bfloat16, device=cuda)
        _lib.check(_lib.lib().aem_grouped_qgemm(w.handle, rt.data_ptr(), G, xt.data_ptr(), M,
                                                out.data_ptr(), _lib.BF16, N, 1, 0, None, None,
                                                0, 1, stream), "aem_grouped_qgemm")
        torch.cuda.synchronize()
        _close(out.float().cpu().numpy(), np.maximum(ref, 0.0), rtol=2 ** -8 + 1e-3, atol=1e-3)
    else:
        rmap = np.array([5, 2, 7, 2], np.int32)[:M]  # output row 2 receives two rows
        rscale = (rng.random(M) + 0.5).astype(np.float32)
        base = rng.normal(size=(8, N)).astype(np.float32)
        out = torch.from_numpy(base.copy()).to(cuda)
        # device copies held in names: a temporary's memory could be reused by
        # the next argument before the kernel reads it
        mt = torch.from_numpy(rmap).to(cuda)
        st = torch.from_numpy(rscale).to(cuda)
        _lib.check(_lib.lib().aem_grouped_qgemm(
            w.handle, rt.data_ptr(), G, xt.data_ptr(), M, out.data_ptr(), _lib.F32, N, 0, 1,
            mt.data_ptr(), st.data_ptr(), 0, 1, stream), "aem_grouped_qgemm")
        torch.cuda.synchronize()
        want = base.astype(np.float64).copy()
        np.add.at(want, rmap, ref * rscale[:, None].astype(np.float64))
        _close(out.cpu().numpy(), want)
    _lib.check(_lib.lib().aem_device_status(None), "aem_device_status")


@pytest.mark.parametrize("m,k,n", [(1, 4096, 14336), (2, 448, 300), (3, 40, 130), (4, 200, 129)])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_decode_sizes_dense(qg, m, k, n, dtype):
    """aem_qgemm with at most 4 rows: the CUDA-core path with K split across
    CTAs (float32 plain store: rows zeroed, partial sums added)."""
    rng = np.random.default_rng(m * 7 + k + n)
    x = rng.normal(size=(m, k)).astype(np.float32)
    q, s = O.quantize_int8((rng.normal(size=(k, n)) * 0.02).astype(np.float32))
    if dtype == "bf16":
        xf = O.bf16_round(x)
        out = _bf16_gemm(q, s, (xf.view(np.uint32) >> 16).astype(np.uint16))
    else:
        xf = x
        out = qg.fused_quantized_matmul(x, q, s)
    _close(out, xf.astype(np.float64) @ O.dequantize_int8(q, s).astype(np.float64))


@pytest.mark.parametrize("m", [16, 40, 64, 200, 1000])
def test_repeated_launches_stay_consistent(cuda, gemm_form, m):
    """Forty back-to-back launches per token tile (16 .. 256 rows): every
    output equal to the first up to split-K reassociation, and no bounded wait
    ran out.  Guards the ring
    protocol (a parity wait that could read an older phase of a slot showed
    up only in some launches)."""
    import torch
    from aethermoe_b200 import _lib
    rng = np.random.default_rng(m)
    K, N = 4096, 1536
    q = rng.integers(-127, 128, size=(K, N), dtype=np.int8)
    s = (rng.random(size=(1, N)) * 1e-3 + 1e-4).astype(np.float32)
    w = _lib.QWeight(q, s, 0)
    x = O.bf16_round(rng.normal(size=(m, K)).astype(np.float32))
    xt = torch.from_numpy((x.view(np.uint32) >> 16).astype(np.uint16).view(np.int16)).to(cuda)
    xt = xt.view(torch.bfloat16)
    outs = [torch.empty((m, N), dtype=torch.float32, device=cuda) for _ in range(40)]
    stream = torch.cuda.current_stream().cuda_stream
    for o in outs:
        _lib.check(_lib.lib().aem_qgemm(w.handle, 0, xt.data_ptr(), _lib.BF16, m, o.data_ptr(),
                                        stream), "aem_qgemm")
    torch.cuda.synchronize()
    _lib.check(_lib.lib().aem_device_status(None), "aem_device_status")
    first = outs[0].cpu().numpy()
    _close(first, x.astype(np.float64) @ (q.astype(np.float64) * s.astype(np.float64)))
    for o in outs[1:]:
        # split-K adds partial sums with float32 atomics in any order: a few
        # ulp of reassociation; stale operands would be off by O(1)
        np.testing.assert_allclose(o.cpu().numpy(), first, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("m,dtype", [(512, "bf16"), (1000, "f32"), (4096, "bf16")])
def test_pairs_match_single_sms(cuda, m, dtype):
    """The same dense GEMM on single SMs and on SM pairs: both within the
    GEMM tolerance of the float64 oracle and within float32 reassociation of
    each other."""
    import torch
    from aethermoe_b200 import _lib
    rng = np.random.default_rng(m + len(dtype))
    K, N = 2048, 1408  # 11 channel blocks: the last pair holds one real block
    q = rng.integers(-127, 128, size=(K, N), dtype=np.int8)
    s = (rng.random(size=(1, N)) * 1e-3 + 1e-4).astype(np.float32)
    w = _lib.QWeight(q, s, 0)
    x = rng.normal(size=(m, K)).astype(np.float32)
    if dtype == "bf16":
        x = O.bf16_round(x)
        xt = torch.from_numpy((x.view(np.uint32) >> 16).astype(np.uint16).view(np.int16))
        xt, code = xt.to(cuda).view(torch.bfloat16), _lib.BF16
    else:
        xt, code = torch.from_numpy(x).to(cuda), _lib.F32
    stream = torch.cuda.current_stream().cuda_stream
    res = {}
    for mode in (0, 1):
        _lib.check(_lib.lib().aem_set_gemm_pairs(mode))
        o = torch.empty((m, N), dtype=torch.float32, device=cuda)
        _lib.check(_lib.lib().aem_qgemm(w.handle, 0, xt.data_ptr(), code, m, o.data_ptr(),
                                        stream), "aem_qgemm")
        torch.cuda.synchronize()
        res[mode] = o.cpu().numpy()
    _lib.check(_lib.lib().aem_set_gemm_pairs(-1))
    _lib.check(_lib.lib().aem_device_status(None), "aem_device_status")
    ref = x.astype(np.float64) @ (q.astype(np.float64) * s.astype(np.float64))
    _close(res[0], ref)
    _close(res[1], ref)
    np.testing.assert_allclose(res[1], res[0], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("sizes,K,N", [([0, 1, 6, 0, 9], 448, 300), ([16], 200, 130),
                                        ([3, 0, 5], 4096, 1536), ([8, 8], 40, 257)])
@pytest.mark.parametrize("mode", ["relu_bf16", "scaled_add", "f32_store"])
def test_weight_stream_path(cuda, small_form, sizes, K, N, mode):
    """At most 16 rows: the bandwidth-bound weight stream (warp MMAs on
    registers loaded straight from the int8 tiles).  Groups of 0-16 rows, K
    and N that are not multiples of the 64 x 128 tile, float32 activations as
    hi + lo (f32_store; the layer tests cover the hi + lo hidden output)."""
    import torch
    from aethermoe_b200 import _lib
    rng = np.random.default_rng(sum(sizes) + K + N + len(mode))
    G = len(sizes)
    q = rng.integers(-127, 128, size=(G, K, N), dtype=np.int8)
    s = (rng.random(size=(G, N)) * 1e-3 + 1e-4).astype(np.float32)
    w = _lib.QWeight(q, s, 0)
    rows = np.r_[0, np.cumsum(sizes)].astype(np.int32)
    M = int(rows[-1])
    x = rng.normal(size=(M, K)).astype(np.float32)
    ref = np.zeros((M, N))
    for g in range(G):
        a, b = rows[g], rows[g + 1]
        ref[a:b] = x[a:b].astype(np.float64) @ (q[g].astype(np.float64) * s[g].astype(np.float64))
    hi = O.bf16_round(x)
    tobf = lambda a: torch.from_numpy((a.view(np.uint32) >> 16).astype(np.uint16).view(np.int16)).to(cuda).view(torch.bfloat16)  # noqa: E731
    rt = torch.from_numpy(rows).to(cuda)
    stream = torch.cuda.current_stream().cuda_stream
    L = _lib.lib()
    if mode == "f32_store":
        # dense call on each group's rows through aem_qgemm (float32 x split hi + lo)
        for g in range(G):
            a, b = rows[g], rows[g + 1]
            if b == a:
                continue
            xt = torch.from_numpy(x[a:b].copy()).to(cuda)
            out = torch.empty((b - a, N), dtype=torch.float32, device=cuda)
            _lib.check(L.aem_qgemm(w.handle, g, xt.data_ptr(), _lib.F32, b - a, out.data_ptr(),
                                   stream), "aem_qgemm")
            torch.cuda.synchronize()
            _close(out.cpu().numpy(), ref[a:b])
        return
    if mode == "relu_bf16":
        # the MoE layer's up projection: grouped, ReLU, bf16 output
        xt = tobf(hi)
        out = torch.zeros((M, N), dtype=torch.bfloat16, device=cuda)
        _lib.check(L.aem_grouped_qgemm(w.handle, rt.data_ptr(), G, xt.data_ptr(), M,
                                       out.data_ptr(), _lib.BF16, N, 1, 0, None, None, 0, 1,
                                       stream), "aem_grouped_qgemm")
        torch.cuda.synchronize()
        refh = np.zeros((M, N))
        for g in range(G):
            a, b = rows[g], rows[g + 1]
            refh[a:b] = hi[a:b].astype(np.float64) @ (q[g].astype(np.float64) * s[g].astype(np.float64))
        _close(out.float().cpu().numpy(), np.maximum(refh, 0.0), rtol=2 ** -8 + 1e-3, atol=1e-3)
    else:
        rmap = rng.permutation(M).astype(np.int32)
        rscale = (rng.random(M) + 0.5).astype(np.float32)
        base = rng.normal(size=(M, N)).astype(np.float32)
        out = torch.from_numpy(base.copy()).to(cuda)
        mt = torch.from_numpy(rmap).to(cuda)
        st = torch.from_numpy(rscale).to(cuda)
        xt = tobf(hi)
        _lib.check(L.aem_grouped_qgemm(w.handle, rt.data_ptr(), G, xt.data_ptr(), M,
                                       out.data_ptr(), _lib.F32, N, 0, 1, mt.data_ptr(),
                                       st.data_ptr(), 0, 1, stream), "aem_grouped_qgemm")
        torch.cuda.synchronize()
        refh = np.zeros((M, N))
        for g in range(G):
            a, b = rows[g], rows[g + 1]
            refh[a:b] = hi[a:b].astype(np.float64) @ (q[g].astype(np.float64) * s[g].astype(np.float64))
        want = base.astype(np.float64).copy()
        want[rmap] += refh * rscale[:, None].astype(np.float64)
        _close(out.cpu().numpy(), want)
    _lib.check(L.aem_device_status(None), "aem_device_status")
