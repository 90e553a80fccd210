// Bandwidth-bound INT8 GEMM for few activation rows (GEMV-style), on the
// tensor cores' warp-level MMA.
//
// With at most 16 rows per weight group the work per weight byte is a few
// multiply-adds, so the kernel is a weight stream: every warp loads its int8
// rows straight from global memory into registers (16-byte non-caching loads,
// the next tiles' while the current one is multiplied), converts them exactly
// to bf16 in registers and multiplies them with mma.sync.m16n8k16 (bf16 in,
// float32 accumulate).  No shared memory holds weights and no barrier paces
// the stream; shared memory holds the CTA's activation rows, restaged every
// 768 K of its range.  Three register buffers keep two tiles in flight
// while a third is converted and multiplied (the loop is unrolled by three,
// so no buffer is copied), and the K split makes one wave of CTAs (four per
// SM at this register use).  Many small CTAs (four warps): converting int8
// costs about two instructions per weight byte, so the kernel needs issue
// slots and warps to hide latency as much as bytes in flight.  Measured on
// B200 against this form, a bulk-copy shared-memory ring, a per-thread
// cp.async pipeline, an fp16 conversion with four tiles in flight and the
// tcgen05 kernel were all slower at 1-16 rows (fewer warps per SM, more
// instructions, or the tcgen05 issue chain); the tcgen05 kernel wins from
// 17 rows on.
//
// K permutation: a dot product does not depend on the order of K, so the MMA
// fragment's K positions are mapped to memory such that thread (g, t) of a warp
// (g = lane / 4, t = lane % 4) finds its A operand for the four 16-wide K steps
// of a 64-wide tile in ONE 16-byte chunk of a packed weight row (chunk t: K
// offsets 16t .. 16t+15, K step j using 16t + 4j .. 16t + 4j + 3), and its B
// operand (activations of token g) in the same 16 consecutive K of the token's
// row: fragment positions {2t, 2t+1, 2t+8, 2t+9} of K step j hold memory K
// {16t+4j, +1, +2, +3} in both operands.
//
// CTA: 4 warps over one 128-channel weight-tile row (32 channels per warp = two
// 16-row MMA tiles), a K range, one weight group.  Partial sums over K ranges
// are added with float32 atomics into the zeroed output.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "runtime.h"

namespace aem {

namespace {

constexpr int kGvWarps = 4;
constexpr int kGvThreads = kGvWarps * 32;
constexpr int kGvMaxRows = 16;  // above: the tensor-core kernel (measured faster from 17 rows)
constexpr int kGvMaxGroups = 256;

// 4 signed bytes (one 32-bit word, bytes b0 b1 b2 b3) -> two bf16x2 words
// (b0, b1) and (b2, b3), exact: each byte becomes the float 2^23 + (b + 128)
// by byte permutation, minus (2^23 + 128); the bf16 is the float's upper half.
__device__ __forceinline__ uint2 gv_i8x4_to_bf16x4(uint32_t v) {
    const uint32_t u = v ^ 0x80808080u;
    const float2 m = make_float2(-8388736.0f, -8388736.0f);
    const float2 f01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)),
                                              __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441))),
                                  m);
    const float2 f23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)),
                                              __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443))),
                                  m);
    uint2 o;
    o.x = __byte_perm(__float_as_uint(f01.x), __float_as_uint(f01.y), 0x7632);
    o.y = __byte_perm(__float_as_uint(f23.x), __float_as_uint(f23.y), 0x7632);
    return o;
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ld_stream16(const int8_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

struct GvParams {
    const __nv_bfloat16* xh;  // [M][K]
    const __nv_bfloat16* xl;  // [M][K] or nullptr (float32 activations split hi + lo)
    const float* xf;          // [M][K] float32 pre-activations (instead of xh / xl) or nullptr
    int has_lo;               // a lo plane: xl given, or xf staged as a pair
    const int8_t* wq;         // tiled int8 weights
    const float* scale;
    int64_t M, K, N, NT, KT;
    const int* group_rows;    // nullptr: one group of M rows
    int G;                    // groups in group_rows (blockIdx.z picks the z-th with rows)
    int64_t group_base;
    int wmod;
    int ks;                   // K ranges
    int kper;                 // 64-wide K tiles per range
    void* out;
    void* out_lo;
    int64_t ldo;
    int out_bf16, relu, atomic_add;
    const int* rowmap;
    const float* rowscale;
    int* err;
};

// NT8: 8-row MMA tiles of activation rows (rows per group <= 8 * NT8).
template <int NT8>
__global__ void __launch_bounds__(kGvThreads)
    qgemv_kernel(const GvParams p) {
    extern __shared__ __align__(16) unsigned char gsm[];
    const int nb = blockIdx.x;  // 128-channel tile row
    const int ks = blockIdx.y;
    // grouped: the grid covers min(G, M) group slots; slot z takes the z-th
    // group that has rows (most groups are empty at decode sizes)
    int g = 0;
    if (p.group_rows) {
        __shared__ int s_rows[kGvMaxGroups + 1];
        __shared__ int s_pick;
        for (int i = threadIdx.x; i <= p.G; i += kGvThreads) s_rows[i] = p.group_rows[i];
        __syncthreads();
        if (threadIdx.x < 32) {
            const int lane0 = threadIdx.x;
            int base = 0, pick = -1;
            bool bad = false;
            for (int c0 = 0; c0 < p.G; c0 += 32) {
                const int gg = c0 + lane0;
                const int mm = gg < p.G ? s_rows[gg + 1] - s_rows[gg] : 0;
                if (mm < 0 || mm > NT8 * 8) bad = true;
                const unsigned bal = __ballot_sync(0xFFFFFFFFu, mm > 0);
                const int before = base + __popc(bal & ((1u << lane0) - 1u));
                if (mm > 0 && before == static_cast<int>(blockIdx.z)) pick = gg;
                base += __popc(bal);
            }
            // one lane at most found the slot's group
            const unsigned has = __ballot_sync(0xFFFFFFFFu, pick >= 0);
            if (lane0 == 0) s_pick = has ? -2 : -1;
            __syncwarp();
            if (pick >= 0) s_pick = pick;
            if (__any_sync(0xFFFFFFFFu, bad) && lane0 == 0 && blockIdx.x == 0 && blockIdx.y == 0 &&
                blockIdx.z == 0)
                atomicOr(p.err, ERR_GEMM_GROUPS);
        }
        __syncthreads();
        g = s_pick;
        if (g < 0) return;  // fewer groups with rows than slots (uniform over the CTA)
    }
    const int r0 = p.group_rows ? p.group_rows[g] : 0;
    const int r1 = p.group_rows ? p.group_rows[g + 1] : static_cast<int>(p.M);
    const int m = r1 - r0;
    if (m < 0 || m > NT8 * 8 || r0 < 0 || r1 > p.M) {
        if (threadIdx.x == 0) atomicOr(p.err, ERR_GEMM_GROUPS);
        return;
    }
    const int kt0 = ks * p.kper;
    const int kt1 = static_cast<int>(min(p.KT, static_cast<int64_t>(kt0 + p.kper)));
    if (m == 0 || kt0 >= kt1) return;  // uniform over the CTA
    const int64_t wg = p.group_base + (p.wmod ? g % p.wmod : g);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int gq = lane >> 2;  // fragment row group
    const int t = lane & 3;    // fragment column pair
    // this thread's four weight rows in the 128-row tile: 32*warp + {g, g+8, g+16, g+24}
    int offs[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = 32 * warp + gq + 8 * i;
        offs[i] = row * 64 + wtile_chunk(row, t) * 16;
    }
    const int8_t* wtile0 = p.wq + ((wg * p.NT + nb) * p.KT) * kWTileBytes;

    float acc[2][NT8][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int n = 0; n < NT8; ++n)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[a][n][c] = 0.0f;

    constexpr int SUB = 12;  // 64-wide K tiles of activations staged at once (a multiple of 3)
    constexpr int XS = SUB * 64 * 2 + 16;   // padded activation row, bytes
    unsigned char* xs = gsm;                 // [NT8*8][XS] bf16 (hi)
    unsigned char* xls = gsm + NT8 * 8 * XS; // [NT8*8][XS] bf16 (lo), float32 activations only

    // two weight tiles in flight during each tile's compute: tile kt0 + r lives in
    // wa, wb or wc by r mod 3
    uint4 wa[4], wb[4], wc[4];
    auto fetch = [&](uint4 (&w)[4], int kt) {
        if (kt < kt1) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                w[i] = ld_stream16(wtile0 + static_cast<int64_t>(kt) * kWTileBytes + offs[i]);
        }
    };
    fetch(wa, kt0);
    fetch(wb, kt0 + 1);
    auto compute = [&](const uint4 (&w)[4], int kt, int sb) {
        // A fragments: rows i = 0..3 (m-tile i/2, half i%2), K steps j = 0..3
        uint2 a[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            a[i][0] = gv_i8x4_to_bf16x4(w[i].x);
            a[i][1] = gv_i8x4_to_bf16x4(w[i].y);
            a[i][2] = gv_i8x4_to_bf16x4(w[i].z);
            a[i][3] = gv_i8x4_to_bf16x4(w[i].w);
        }
        const int kk = (kt - sb) * 64 + 16 * t;
#pragma unroll
        for (int n = 0; n < NT8; ++n) {
            const unsigned char* xr = xs + (n * 8 + gq) * XS + kk * 2;
            const uint4 b01 = *reinterpret_cast<const uint4*>(xr);       // K steps 0, 1
            const uint4 b23 = *reinterpret_cast<const uint4*>(xr + 16);  // K steps 2, 3
            const uint32_t bw[8] = {b01.x, b01.y, b01.z, b01.w, b23.x, b23.y, b23.z, b23.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                mma_bf16_16816(acc[0][n], a[0][j].x, a[1][j].x, a[0][j].y, a[1][j].y,
                               bw[2 * j], bw[2 * j + 1]);
                mma_bf16_16816(acc[1][n], a[2][j].x, a[3][j].x, a[2][j].y, a[3][j].y,
                               bw[2 * j], bw[2 * j + 1]);
            }
            if (p.has_lo) {
                const unsigned char* xq = xls + (n * 8 + gq) * XS + kk * 2;
                const uint4 l01 = *reinterpret_cast<const uint4*>(xq);
                const uint4 l23 = *reinterpret_cast<const uint4*>(xq + 16);
                const uint32_t lw[8] = {l01.x, l01.y, l01.z, l01.w, l23.x, l23.y, l23.z, l23.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    mma_bf16_16816(acc[0][n], a[0][j].x, a[1][j].x, a[0][j].y, a[1][j].y,
                                   lw[2 * j], lw[2 * j + 1]);
                    mma_bf16_16816(acc[1][n], a[2][j].x, a[3][j].x, a[2][j].y, a[3][j].y,
                                   lw[2 * j], lw[2 * j + 1]);
                }
            }
        }
    };
    for (int sb = kt0; sb < kt1; sb += SUB) {
        const int se = min(kt1, sb + SUB);
        // ---- the token rows' activations of tiles [sb, se) (rows past m, K past K: zero)
        const int R = (se - sb) * 64;
        const int64_t kbase = static_cast<int64_t>(sb) * 64;
        __syncthreads();  // the previous sub-range's rows are consumed
        for (int i = threadIdx.x; i < NT8 * 8 * (R / 8); i += kGvThreads) {
            const int row = i / (R / 8), c8 = i % (R / 8);
            uint4 hv = make_uint4(0, 0, 0, 0), lv = make_uint4(0, 0, 0, 0);
            const int64_t k = kbase + c8 * 8;
            if (row < m) {
                const int64_t o = static_cast<int64_t>(r0 + row) * p.K + k;
                if (p.xf) {
                    // float32 pre-activation: ReLU, then bf16 (and the pair's low half)
                    __nv_bfloat16 h[8], l[8];
                    const bool fv = k + 8 <= p.K && (reinterpret_cast<uintptr_t>(p.xf + o) & 15) == 0;
                    float f[8];
                    if (fv) {
                        const float4 f0 = *reinterpret_cast<const float4*>(p.xf + o);
                        const float4 f1 = *reinterpret_cast<const float4*>(p.xf + o + 4);
                        f[0] = f0.x; f[1] = f0.y; f[2] = f0.z; f[3] = f0.w;
                        f[4] = f1.x; f[5] = f1.y; f[6] = f1.z; f[7] = f1.w;
                    } else {
                        for (int e = 0; e < 8; ++e) f[e] = k + e < p.K ? p.xf[o + e] : 0.0f;
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float v = fmaxf(f[e], 0.0f);
                        h[e] = __float2bfloat16_rn(v);
                        l[e] = __float2bfloat16_rn(v - __bfloat162float(h[e]));
                    }
                    hv = *reinterpret_cast<uint4*>(h);
                    lv = *reinterpret_cast<uint4*>(l);
                } else if (k + 8 <= p.K && (reinterpret_cast<uintptr_t>(p.xh + o) & 15) == 0 &&
                           (!p.xl || (reinterpret_cast<uintptr_t>(p.xl + o) & 15) == 0)) {
                    hv = *reinterpret_cast<const uint4*>(p.xh + o);
                    if (p.xl) lv = *reinterpret_cast<const uint4*>(p.xl + o);
                } else {
                    __nv_bfloat16 h[8], l[8];
                    for (int e = 0; e < 8; ++e) {
                        const bool in = k + e < p.K;
                        h[e] = in ? p.xh[o + e] : __float2bfloat16_rn(0.0f);
                        l[e] = (in && p.xl) ? p.xl[o + e] : __float2bfloat16_rn(0.0f);
                    }
                    hv = *reinterpret_cast<uint4*>(h);
                    lv = *reinterpret_cast<uint4*>(l);
                }
            }
            *reinterpret_cast<uint4*>(xs + row * XS + c8 * 16) = hv;
            if (p.has_lo) *reinterpret_cast<uint4*>(xls + row * XS + c8 * 16) = lv;
        }
        __syncthreads();

        // sub-ranges start a multiple of 3 tiles after kt0 (SUB is)
        for (int kt = sb; kt < se; kt += 3) {
            fetch(wc, kt + 2);
            compute(wa, kt, sb);
            if (kt + 1 < se) {
                fetch(wa, kt + 3);
                compute(wb, kt + 1, sb);
            }
            if (kt + 2 < se) {
                fetch(wb, kt + 4);
                compute(wc, kt + 2, sb);
            }
        }
    }

    // ---- epilogue: accumulator (m-tile a, n-tile n) element c holds
    // channel 32*warp + 16a + g (+8 for c >= 2), token 8n + 2t + (c & 1)
#pragma unroll
    for (int am = 0; am < 2; ++am) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int64_t ch = static_cast<int64_t>(nb) * kWTileN + 32 * warp + 16 * am + gq + 8 * half;
            if (ch >= p.N) continue;
            const float sc = p.scale[wg * p.N + ch];
#pragma unroll
            for (int n = 0; n < NT8; ++n) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int tok = 8 * n + 2 * t + c;
                    if (tok >= m) continue;
                    const int r = r0 + tok;
                    float v = acc[am][n][2 * half + c] * sc;
                    if (p.rowscale) v *= p.rowscale[r];
                    if (p.relu) v = fmaxf(v, 0.0f);
                    const int64_t orow = p.rowmap ? p.rowmap[r] : r;
                    if (p.out_bf16) {
                        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
                        static_cast<__nv_bfloat16*>(p.out)[orow * p.ldo + ch] = hi;
                        if (p.out_lo)
                            static_cast<__nv_bfloat16*>(p.out_lo)[orow * p.ldo + ch] =
                                __float2bfloat16_rn(v - __bfloat162float(hi));
                    } else if (p.atomic_add) {
                        atomicAdd(static_cast<float*>(p.out) + orow * p.ldo + ch, v);
                    } else {
                        static_cast<float*>(p.out)[orow * p.ldo + ch] = v;
                    }
                }
            }
        }
    }
}

template <int NT8>
aem_status launch_gv(const GvParams& p, int64_t groups, cudaStream_t s) {
    constexpr int SUB = 12;
    const size_t smem = static_cast<size_t>((p.has_lo ? 2 : 1) * NT8 * 8) * (SUB * 64 * 2 + 16);
    auto kern = qgemv_kernel<NT8>;
    if (smem > 48 * 1024)
        AEM_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem)));
    const dim3 grid(static_cast<unsigned>(p.NT), static_cast<unsigned>(p.ks),
                    static_cast<unsigned>(groups));
    kern<<<grid, kGvThreads, smem, s>>>(p);
    AEM_CHECK_LAUNCH();
    count_launches(1);
    return AEM_OK;
}

}  // namespace

int gemv_max_rows() { return kGvMaxRows; }

aem_status launch_qgemm_gemv(const GemmArgs& a, cudaStream_t s) {
    const QWeight& w = *a.w;
    if (a.M == 0) return AEM_OK;
    AEM_REQUIRE(a.M <= kGvMaxRows || a.group_rows, "qgemv: %lld rows in one group > %d",
                (long long)a.M, kGvMaxRows);
    const int dev = current_device();
    const int sms = sm_count(dev);
    int* err = device_error_word(dev);
    AEM_REQUIRE(err != nullptr, "qgemv: no device error word");
    // rows of the largest group: at most M (the group sizes live on the device)
    const int64_t mrows = std::min<int64_t>(a.M, kGvMaxRows);
    const int nt8 = mrows <= 8 ? 1 : 2;
    AEM_REQUIRE(a.G >= 1 && a.G <= kGvMaxGroups, "qgemv: G=%d outside [1, %d]", a.G, kGvMaxGroups);
    // group slots: at most min(G, M) groups have rows (each slot finds its group)
    const int64_t groups = a.group_rows ? std::min<int64_t>(a.G, a.M) : 1;
    const int64_t busy = groups * w.NT;  // CTAs with rows per K range
    // K ranges: enough CTAs for ~4 per SM, ranges of at most 1024 K (shared
    // memory for the activation rows); split only where partial sums may add
    const bool can_split = !a.out_bf16 && !a.relu && (a.atomic_add || a.rowmap == nullptr);
    int64_t ks = 1;
    if (can_split) {
        // one wave: as many CTAs as fit resident (4 per SM at this register use)
        ks = std::max<int64_t>(1, (4 * static_cast<int64_t>(sms)) / busy);
        ks = std::min<int64_t>(ks, w.KT);
    }
    const int kper = static_cast<int>((w.KT + ks - 1) / ks);
    ks = (w.KT + kper - 1) / kper;
    const bool add = a.atomic_add || ks > 1;
    if (ks > 1 && !a.atomic_add)
        AEM_TRY_CUDA(cudaMemset2DAsync(a.out, static_cast<size_t>(a.ldo) * 4, 0,
                                       static_cast<size_t>(w.N) * 4, static_cast<size_t>(a.M), s));
    GvParams p;
    p.xh = static_cast<const __nv_bfloat16*>(a.x_hi);
    p.xl = a.x_f32_relu ? nullptr : static_cast<const __nv_bfloat16*>(a.x_lo);
    p.xf = a.x_f32_relu;
    p.has_lo = (a.x_f32_relu ? a.x_f32_lo : a.x_lo != nullptr) ? 1 : 0;
    p.wq = w.q;
    p.scale = w.scale;
    p.M = a.M;
    p.K = w.K;
    p.N = w.N;
    p.NT = w.NT;
    p.KT = w.KT;
    p.group_rows = a.group_rows;
    p.G = a.group_rows ? a.G : 1;
    p.group_base = a.group_base;
    p.wmod = a.wmod;
    p.ks = static_cast<int>(ks);
    p.kper = kper;
    p.out = a.out;
    p.out_lo = a.out_bf16 ? a.out_lo : nullptr;
    p.ldo = a.ldo;
    p.out_bf16 = a.out_bf16 ? 1 : 0;
    p.relu = a.relu ? 1 : 0;
    p.atomic_add = add ? 1 : 0;
    p.rowmap = a.rowmap;
    p.rowscale = a.rowscale;
    p.err = err;
    if (nt8 == 1) return launch_gv<1>(p, groups, s);
    return launch_gv<2>(p, groups, s);
}

}  // namespace aem
