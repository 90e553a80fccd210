// INT8 weight-only quantisation (bit-exact with the reference's float32
// NumPy), packing of INT8 expert weights into the output-channel-major
// layout the GEMM streams, the float32 -> (bf16 hi, bf16 lo) activation
// split, and the CUDA-core GEMM used when K is not a multiple of 8.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "runtime.h"

namespace aem {

namespace {

// scale[n] = max(max_k |w[k,n]| / 127, 1e-12) and q = clip(rint(w / scale)),
// in IEEE float32 exactly as prototype/math_proto.py:63-65 evaluates it
// (correctly rounded division, round-half-even).  One thread per column;
// consecutive threads read consecutive columns (coalesced rows).
__global__ void quantize_kernel(const float* __restrict__ w, int64_t K, int64_t N,
                                int8_t* __restrict__ q, float* __restrict__ scale) {
    const int64_t n = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (n >= N) return;
    float amax = 0.0f;
    for (int64_t k = 0; k < K; ++k) amax = fmaxf(amax, fabsf(w[k * N + n]));
    float s = __fdiv_rn(amax, 127.0f);
    s = fmaxf(s, 1e-12f);
    scale[n] = s;
    for (int64_t k = 0; k < K; ++k) {
        float r = rintf(__fdiv_rn(w[k * N + n], s));
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        q[k * N + n] = static_cast<int8_t>(static_cast<int>(r));
    }
}

// [G][K][N] (reference layout) -> the tiled layout of QWeight, via 32x32
// shared-memory transposes (padding stays zero from the memset before).
__global__ void transpose_i8_kernel(const int8_t* __restrict__ in, int64_t K, int64_t N,
                                    int64_t NT, int64_t KT, int8_t* __restrict__ out) {
    __shared__ int8_t tile[32][33];
    const int64_t g = blockIdx.z;
    const int64_t k0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * 32;
    const int8_t* src = in + g * K * N;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t k = k0 + i, n = n0 + threadIdx.x;
        if (k < K && n < N) tile[i][threadIdx.x] = src[k * N + n];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t n = n0 + i, k = k0 + threadIdx.x;
        if (k < K && n < N) out[wtile_offset(g, n, k, NT, KT)] = tile[threadIdx.x][i];
    }
}

// x (float32) -> hi = bf16_rn(x), lo = bf16_rn(x - hi); or bf16 copy.
__global__ void split_kernel(const float* __restrict__ x, int64_t count,
                             __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float v = x[i];
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        hi[i] = h;
        if (lo) lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
}

// CUDA-core fallback, used only when K % 8 != 0 (the tensor-core path's
// activation TMA needs 16-byte rows): one thread per output element, activations as the
// bf16 hi (+ lo) pair the tensor-core path consumes.
// out[r, n] = scale[n] * sum_k (hi[r,k] + lo[r,k]) * q[n,k].
__global__ void qgemm_simt_kernel(const __nv_bfloat16* __restrict__ xh,
                                  const __nv_bfloat16* __restrict__ xl,
                                  const int8_t* __restrict__ q, const float* __restrict__ scale,
                                  int64_t M, int64_t K, int64_t N, int64_t NT, int64_t KT,
                                  const int* __restrict__ group_rows, int G, int64_t group_base,
                                  int wmod,
                                  void* __restrict__ out, void* __restrict__ out_lo, int64_t ldo,
                                  bool out_bf16, bool relu,
                                  bool atomic_add, const int* __restrict__ rowmap,
                                  const float* __restrict__ rowscale) {
    const int64_t total = M * N;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / N;
        const int64_t n = i % N;
        int g = 0;
        if (group_rows) {
            if (r < group_rows[0] || r >= group_rows[G]) continue;
            while (g < G - 1 && r >= group_rows[g + 1]) ++g;
        }
        const int64_t wg = group_base + (wmod ? g % wmod : g);
        float acc = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            float xv = __bfloat162float(xh[r * K + k]);
            if (xl) xv += __bfloat162float(xl[r * K + k]);
            acc = fmaf(xv, static_cast<float>(q[wtile_offset(wg, n, k, NT, KT)]), acc);
        }
        float v = acc * scale[wg * N + n];
        if (rowscale) v *= rowscale[r];
        if (relu) v = fmaxf(v, 0.0f);
        const int64_t orow = rowmap ? rowmap[r] : r;
        if (out_bf16) {
            const __nv_bfloat16 hi = __float2bfloat16_rn(v);
            static_cast<__nv_bfloat16*>(out)[orow * ldo + n] = hi;
            if (out_lo)
                static_cast<__nv_bfloat16*>(out_lo)[orow * ldo + n] =
                    __float2bfloat16_rn(v - __bfloat162float(hi));
        } else if (atomic_add) {
            atomicAdd(static_cast<float*>(out) + orow * ldo + n, v);
        } else {
            static_cast<float*>(out)[orow * ldo + n] = v;
        }
    }
}

// Decode-size INT8 GEMM on the CUDA cores (at most MAXM <= 4 rows per weight
// group; dispatched for single-row calls, where it measured ahead of the
// warp-MMA weight stream).  One CTA of 128 threads per (row group, 128-channel block, K range).
// Thread t owns the 16-byte chunk at position t % 4 (16 consecutive K) of
// channel rows t/4 + 32j (j < 4) of every 8 KB weight tile, so each warp load
// reads 512 contiguous bytes and the chunk's 16 activations serve four rows.  int8 ->
// float is exact (2^23 + 128 + b as a float bit pattern, minus 2^23 + 128);
// products are summed by packed float32 FMAs (even and odd K in two lanes);
// the four owners of a row combine by shuffles.  Split-K partial sums (KS > 1)
// are added with float32 atomics into a float32 output.
constexpr int kDecodeThreads = 128;
constexpr int kDecodeStageK = 8;  // 64-wide K blocks of activations staged at once
constexpr int kDecodeXRow = kDecodeStageK * 64 + kDecodeStageK * 8;  // padded row

// Staged activation k (relative to the chunk) -> its padded position: 4 floats
// of padding after every 32, so the four chunk owners' 16-byte loads of one
// quarter warp fall in distinct banks.
__device__ __forceinline__ int xpad(int kk) { return kk + 4 * (kk >> 5); }

template <int MAXM>
__global__ void __launch_bounds__(kDecodeThreads)
    qgemm_decode_kernel(const __nv_bfloat16* __restrict__ xh, const __nv_bfloat16* __restrict__ xl,
                        const int8_t* __restrict__ q, const float* __restrict__ scale, int64_t M,
                        int64_t K, int64_t N, int64_t NT, int64_t KT,
                        const int* __restrict__ group_rows, int64_t group_base, int wmod, int KS,
                        int kper, void* __restrict__ out, void* __restrict__ out_lo, int64_t ldo,
                        int out_bf16, int relu,
                        int atomic_add, const int* __restrict__ rowmap,
                        const float* __restrict__ rowscale, int* __restrict__ err) {
    __shared__ __align__(16) float xs[MAXM][kDecodeXRow];
    int64_t b = blockIdx.x;
    const int ks = static_cast<int>(b % KS);
    b /= KS;
    const int64_t nb = b % NT;
    const int g = static_cast<int>(b / NT);
    const int r0 = group_rows ? group_rows[g] : 0;
    const int r1 = group_rows ? group_rows[g + 1] : static_cast<int>(M);
    const int m = r1 - r0;
    if (m < 0 || m > MAXM || r0 < 0 || r1 > M) {  // group table inconsistent with M
        if (threadIdx.x == 0) atomicOr(err, ERR_GEMM_GROUPS);
        return;
    }
    const int kt0 = ks * kper;
    const int kt1 = static_cast<int>(min(KT, static_cast<int64_t>(kt0 + kper)));
    if (m <= 0 || kt0 >= kt1) return;  // uniform over the CTA
    const int64_t wg = group_base + (wmod ? g % wmod : g);
    const int t = threadIdx.x;
    // this thread streams chunk position t & 3 of rows t/4 + 32j: the K
    // offsets (logical chunk) stored there, the same for every j
    const int c = wtile_chunk(t >> 2, t & 3);
    const int8_t* wtile = q + ((wg * NT + nb) * KT) * kWTileBytes + t * 16;  // + j * 2048
    float2 acc[4][MAXM];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < MAXM; ++i) acc[j][i] = make_float2(0.0f, 0.0f);
    const float2 magic = make_float2(-8388736.0f, -8388736.0f);
    for (int kc = kt0; kc < kt1; kc += kDecodeStageK) {
        const int nkb = min(kDecodeStageK, kt1 - kc);
        __syncthreads();  // the previous chunk's activations are consumed
        for (int i = t; i < MAXM * kDecodeStageK * 64; i += kDecodeThreads) {
            const int mm = i / (kDecodeStageK * 64), kk = i % (kDecodeStageK * 64);
            const int64_t k = static_cast<int64_t>(kc) * 64 + kk;
            float v = 0.0f;
            if (mm < m && kk < nkb * 64 && k < K) {
                const int64_t o = static_cast<int64_t>(r0 + mm) * K + k;
                v = __bfloat162float(xh[o]);
                if (xl) v += __bfloat162float(xl[o]);
            }
            xs[mm][xpad(kk)] = v;
        }
        __syncthreads();
#pragma unroll 4
        for (int kb = 0; kb < nkb; ++kb) {
            const int8_t* src = wtile + static_cast<int64_t>(kc + kb) * kWTileBytes;
            uint4 wv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                             : "=r"(wv[j].x), "=r"(wv[j].y), "=r"(wv[j].z), "=r"(wv[j].w)
                             : "l"(src + 2048 * j));
            }
            float4 xv[MAXM][4];  // this chunk's 16 activations of each row
#pragma unroll
            for (int mm = 0; mm < MAXM; ++mm)
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    xv[mm][e] = *reinterpret_cast<const float4*>(
                        &xs[mm][xpad(kb * 64 + c * 16) + 4 * e]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t words[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint32_t u = words[e] ^ 0x80808080u;
                    const float2 w01 = __fadd2_rn(
                        make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)),
                                    __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441))),
                        magic);
                    const float2 w23 = __fadd2_rn(
                        make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)),
                                    __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443))),
                        magic);
#pragma unroll
                    for (int mm = 0; mm < MAXM; ++mm) {
                        acc[j][mm] = __ffma2_rn(w01, make_float2(xv[mm][e].x, xv[mm][e].y),
                                                acc[j][mm]);
                        acc[j][mm] = __ffma2_rn(w23, make_float2(xv[mm][e].z, xv[mm][e].w),
                                                acc[j][mm]);
                    }
                }
            }
        }
    }
    // the four chunk owners of a row (lanes 4i..4i+3) combine; lane c == 0 stores
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int64_t n = nb * kWTileN + (t >> 2) + 32 * j;
        const float sc = (n < N) ? scale[wg * N + n] : 0.0f;
#pragma unroll
        for (int mm = 0; mm < MAXM; ++mm) {
            float v = acc[j][mm].x + acc[j][mm].y;
            v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
            v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
            if (c != 0 || mm >= m || n >= N) continue;
            const int r = r0 + mm;
            v *= sc;
            if (rowscale) v *= rowscale[r];
            if (relu) v = fmaxf(v, 0.0f);
            const int64_t orow = rowmap ? rowmap[r] : r;
            if (out_bf16) {
                const __nv_bfloat16 hi = __float2bfloat16_rn(v);
                static_cast<__nv_bfloat16*>(out)[orow * ldo + n] = hi;
                if (out_lo)
                    static_cast<__nv_bfloat16*>(out_lo)[orow * ldo + n] =
                        __float2bfloat16_rn(v - __bfloat162float(hi));
            } else if (atomic_add) {
                atomicAdd(static_cast<float*>(out) + orow * ldo + n, v);
            } else {
                static_cast<float*>(out)[orow * ldo + n] = v;
            }
        }
    }
}

}  // namespace

aem_status launch_qgemm_decode(const GemmArgs& a, cudaStream_t s) {
    const QWeight& w = *a.w;
    if (a.M == 0) return AEM_OK;
    AEM_REQUIRE(a.M <= 4, "qgemm decode path: M=%lld > 4", (long long)a.M);
    const int dev = current_device();
    const int sms = sm_count(dev);
    int* err = device_error_word(dev);
    AEM_REQUIRE(err != nullptr, "qgemm: no device error word");
    // at most M row groups hold rows
    const int64_t busy = static_cast<int64_t>(a.group_rows ? std::min<int64_t>(a.G, a.M) : 1) * w.NT;
    // split K across CTAs when partial sums may be added: float32 output
    // without ReLU, and either an accumulating caller or a plain store into
    // rows that are zeroed first (no row map)
    const bool can_split = !a.out_bf16 && !a.relu && (a.atomic_add || a.rowmap == nullptr);
    // one wave: at most as many CTAs as can be resident at once (a second,
    // partial wave of a few CTAs would double the time)
    int per_sm = 8;
    {
        int n = 0;
        auto k1 = qgemm_decode_kernel<1>;
        auto k4 = qgemm_decode_kernel<4>;
        if ((a.M <= 1 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k1, kDecodeThreads, 0)
                      : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k4, kDecodeThreads, 0)) ==
                cudaSuccess &&
            n > 0)
            per_sm = n;
        else
            cudaGetLastError();
    }
    const int64_t slots = static_cast<int64_t>(per_sm) * sms;
    int64_t ks = 1;
    if (can_split) {
        ks = std::max<int64_t>(1, slots / busy);
        ks = std::min<int64_t>(ks, w.KT);
    }
    const int kper = static_cast<int>((w.KT + ks - 1) / ks);
    ks = (w.KT + kper - 1) / kper;
    const bool add = a.atomic_add || ks > 1;
    if (ks > 1 && !a.atomic_add) {
        // a plain store split over K: start the rows at zero, then add
        AEM_TRY_CUDA(cudaMemset2DAsync(a.out, static_cast<size_t>(a.ldo) * 4, 0,
                                       static_cast<size_t>(w.N) * 4, static_cast<size_t>(a.M), s));
    }
    const int64_t grid = static_cast<int64_t>(a.group_rows ? a.G : 1) * w.NT * ks;
    AEM_REQUIRE(grid < (1ll << 31), "qgemm decode path: grid too large");
    const int m_max = static_cast<int>(a.M);
    auto go = [&](auto kern) {
        kern<<<static_cast<unsigned>(grid), kDecodeThreads, 0, s>>>(
            static_cast<const __nv_bfloat16*>(a.x_hi), static_cast<const __nv_bfloat16*>(a.x_lo),
            w.q, w.scale, a.M, w.K, w.N, w.NT, w.KT, a.group_rows, a.group_base, a.wmod,
            static_cast<int>(ks), kper, a.out, a.out_bf16 ? a.out_lo : nullptr, a.ldo,
            a.out_bf16 ? 1 : 0, a.relu ? 1 : 0,
            add ? 1 : 0, a.rowmap, a.rowscale, err);
    };
    if (m_max <= 1) go(qgemm_decode_kernel<1>);
    else if (m_max <= 2) go(qgemm_decode_kernel<2>);
    else go(qgemm_decode_kernel<4>);
    AEM_CHECK_LAUNCH();
    count_launches(1);
    return AEM_OK;
}

aem_status launch_split_bf16(const void* x, aem_dtype xd, int64_t count, void* hi, void* lo,
                             cudaStream_t s) {
    if (count == 0) return AEM_OK;
    if (xd == AEM_BF16) {
        AEM_TRY_CUDA(cudaMemcpyAsync(hi, x, count * 2, cudaMemcpyDeviceToDevice, s));
        return AEM_OK;
    }
    const int64_t blocks = (count + 255) / 256 < 4096 ? (count + 255) / 256 : 4096;
    split_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        static_cast<const float*>(x), count, static_cast<__nv_bfloat16*>(hi),
        static_cast<__nv_bfloat16*>(lo));
    AEM_CHECK_LAUNCH();
    count_launches(1);
    return AEM_OK;
}

aem_status launch_qgemm_simt(const GemmArgs& a, cudaStream_t s) {
    const QWeight& w = *a.w;
    if (a.M == 0) return AEM_OK;
    const int64_t total = a.M * w.N;
    const int64_t blocks = (total + 255) / 256 < 8192 ? (total + 255) / 256 : 8192;
    qgemm_simt_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(a.x_hi), static_cast<const __nv_bfloat16*>(a.x_lo), w.q,
        w.scale, a.M, w.K, w.N, w.NT, w.KT, a.group_rows, a.G, a.group_base, a.wmod, a.out,
        a.out_bf16 ? a.out_lo : nullptr, a.ldo, a.out_bf16, a.relu, a.atomic_add || a.ksplit > 1,
        a.rowmap, a.rowscale);
    AEM_CHECK_LAUNCH();
    count_launches(1);
    return AEM_OK;
}

aem_status pack_qweight_device(const int8_t* q, const float* scale, int64_t G, int64_t K,
                               int64_t N, cudaStream_t s, QWeight* w) {
    w->NT = (N + kWTileN - 1) / kWTileN;
    w->KT = (K + kWTileK - 1) / kWTileK;
    const size_t bytes = static_cast<size_t>(G * w->NT * w->KT * kWTileBytes);
    AEM_TRY_CUDA(cudaMallocAsync(&w->q, bytes, s));
    AEM_TRY_CUDA(cudaMallocAsync(&w->scale, sizeof(float) * G * N, s));
    AEM_TRY_CUDA(cudaMemsetAsync(w->q, 0, bytes, s));
    dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>((K + 31) / 32),
              static_cast<unsigned>(G));
    transpose_i8_kernel<<<grid, dim3(32, 8), 0, s>>>(q, K, N, w->NT, w->KT, w->q);
    AEM_CHECK_LAUNCH();
    count_launches(1);
    AEM_TRY_CUDA(cudaMemcpyAsync(w->scale, scale, sizeof(float) * G * N, cudaMemcpyDeviceToDevice, s));
    return AEM_OK;
}

}  // namespace aem

using aem::set_error;

extern "C" {

aem_status aem_quantize_int8(const float* w, int64_t K, int64_t N, int8_t* q, float* scale,
                             void* stream) {
    AEM_REQUIRE(K >= 1 && N >= 1, "aem_quantize_int8: K=%lld N=%lld must be >= 1", (long long)K,
                (long long)N);
    AEM_REQUIRE(w && q && scale, "aem_quantize_int8: NULL buffer");
    auto s = static_cast<cudaStream_t>(stream);
    aem::quantize_kernel<<<static_cast<unsigned>((N + 127) / 128), 128, 0, s>>>(w, K, N, q, scale);
    AEM_CHECK_LAUNCH();
    aem::count_launches(1);
    return AEM_OK;
}

aem_status aem_quantize_int8_host(aem_context_t ctx, const float* w, int64_t K, int64_t N,
                                  int8_t* q, float* scale) {
    AEM_REQUIRE(ctx != nullptr, "aem_quantize_int8_host: context is NULL");
    AEM_REQUIRE(K >= 1 && N >= 1, "aem_quantize_int8_host: K=%lld N=%lld must be >= 1",
                (long long)K, (long long)N);
    AEM_REQUIRE(w && q && scale, "aem_quantize_int8_host: NULL buffer");
    auto* c = reinterpret_cast<aem::Context*>(ctx);
    AEM_TRY_CUDA(cudaSetDevice(c->device));
    const size_t wb = sizeof(float) * K * N, qb = static_cast<size_t>(K * N),
                 sb = sizeof(float) * N;
    const size_t o1 = aem::align_up(wb, 256), o2 = o1 + aem::align_up(qb, 256);
    AEM_TRY(c->reserve_device(o2 + sb));
    char* d = static_cast<char*>(c->dev);
    AEM_TRY_CUDA(cudaMemcpyAsync(d, w, wb, cudaMemcpyHostToDevice, c->stream));
    AEM_TRY(aem_quantize_int8(reinterpret_cast<float*>(d), K, N, reinterpret_cast<int8_t*>(d + o1),
                              reinterpret_cast<float*>(d + o2), c->stream));
    AEM_TRY_CUDA(cudaMemcpyAsync(q, d + o1, qb, cudaMemcpyDeviceToHost, c->stream));
    AEM_TRY_CUDA(cudaMemcpyAsync(scale, d + o2, sb, cudaMemcpyDeviceToHost, c->stream));
    AEM_TRY_CUDA(cudaStreamSynchronize(c->stream));
    return AEM_OK;
}

aem_status aem_qweight_pack_device(const int8_t* q, const float* scale, int64_t G, int64_t K,
                                   int64_t N, void* stream, aem_qweight_t* out) {
    AEM_REQUIRE(out != nullptr, "aem_qweight_pack: out is NULL");
    *out = nullptr;
    AEM_REQUIRE(q && scale, "aem_qweight_pack: NULL buffer");
    AEM_REQUIRE(G >= 1 && K >= 1 && N >= 1, "aem_qweight_pack: G=%lld K=%lld N=%lld must be >= 1",
                (long long)G, (long long)K, (long long)N);
    AEM_REQUIRE(K <= (1ll << 31) && G * N <= (1ll << 31),
                "aem_qweight_pack: dimensions exceed 2^31");
    auto* w = new aem::QWeight();
    w->device = aem::current_device();
    w->G = G;
    w->K = K;
    w->N = N;
    aem_status st = aem::pack_qweight_device(q, scale, G, K, N, static_cast<cudaStream_t>(stream), w);
    if (st != AEM_OK) {
        cudaFree(w->q);
        cudaFree(w->scale);
        delete w;
        return st;
    }
    *out = reinterpret_cast<aem_qweight_t>(w);
    return AEM_OK;
}

aem_status aem_qweight_pack(const int8_t* q, const float* scale, int64_t G, int64_t K, int64_t N,
                            int device, aem_qweight_t* out) {
    AEM_REQUIRE(out != nullptr, "aem_qweight_pack: out is NULL");
    *out = nullptr;
    AEM_REQUIRE(q && scale, "aem_qweight_pack: NULL buffer");
    AEM_REQUIRE(G >= 1 && K >= 1 && N >= 1, "aem_qweight_pack: G=%lld K=%lld N=%lld must be >= 1",
                (long long)G, (long long)K, (long long)N);
    if (!aem::is_sm100(device)) {
        set_error("aem_qweight_pack: device %d is not an sm_100 (B200) GPU", device);
        return AEM_EUNSUPPORTED;
    }
    AEM_TRY_CUDA(cudaSetDevice(device));
    int8_t* dq = nullptr;
    float* ds = nullptr;
    AEM_TRY_CUDA(cudaMalloc(&dq, static_cast<size_t>(G * K * N)));
    if (cudaMalloc(&ds, sizeof(float) * G * N) != cudaSuccess) {
        cudaFree(dq);
        set_error("aem_qweight_pack: device allocation failed");
        return AEM_ENOMEM;
    }
    aem_status st = AEM_OK;
    if (cudaMemcpy(dq, q, static_cast<size_t>(G * K * N), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(ds, scale, sizeof(float) * G * N, cudaMemcpyHostToDevice) != cudaSuccess) {
        set_error("aem_qweight_pack: copy failed");
        st = AEM_ECUDA;
    }
    if (st == AEM_OK) st = aem_qweight_pack_device(dq, ds, G, K, N, nullptr, out);
    if (st == AEM_OK && cudaDeviceSynchronize() != cudaSuccess) {
        set_error("aem_qweight_pack: %s", cudaGetErrorString(cudaGetLastError()));
        st = AEM_ECUDA;
    }
    cudaFree(dq);
    cudaFree(ds);
    return st;
}

aem_status aem_qweight_free(aem_qweight_t wh) {
    if (!wh) return AEM_OK;
    auto* w = reinterpret_cast<aem::QWeight*>(wh);
    cudaSetDevice(w->device);
    cudaDeviceSynchronize();
    cudaFree(w->q);
    cudaFree(w->scale);
    delete w;
    return AEM_OK;
}

aem_status aem_qweight_shape(aem_qweight_t wh, int64_t* G, int64_t* K, int64_t* N) {
    AEM_REQUIRE(wh != nullptr, "aem_qweight_shape: handle is NULL");
    auto* w = reinterpret_cast<aem::QWeight*>(wh);
    if (G) *G = w->G;
    if (K) *K = w->K;
    if (N) *N = w->N;
    return AEM_OK;
}

}  // extern "C"
