// Fused MoE gating on sm_100a: logits = hidden @ W + b, top-k by repeated
// strict-greater max extraction (ties -> lowest expert id), softmax over the
// k selected logits -- the semantics of fused_gating
// (src/kernels/fused_gating_metal.py:236-307, :361-435) and of its NumPy
// specification fused_kernel_simulation (prototype/math_proto.py:19-50).
//
// Design (B200): lanes own experts, not slices of d.  A warp is split into
// lane groups of GROUP lanes (8, 16 or 32); a group owns kTPG tokens (4, or 8
// for many tokens) and lane
// `le` of the group owns experts le, le+GROUP, ...  Every (token, expert)
// logit is therefore one sequential dot product inside one thread -- no
// cross-lane reduction -- which makes the EXACT mode possible: float32
// products summed in float32 in increasing d order (bit-identical to the
// reference loop), computed two tokens at a time with the sm_100 packed
// fp32x2 multiply/add so the exact arithmetic runs at FMA rate.
// The CTA stages a 64-wide (or narrower for large E) chunk of d of the
// packed weight ([d/4][Epad][4], contiguous per chunk) and of its tokens'
// activations in shared memory; every weight chunk is reused by all tokens
// of the CTA.  The top-k is a register/shuffle argmax inside the lane group.
#include <cuda_bf16.h>

#include <algorithm>
#include <cfloat>

#include "common.cuh"
#include "runtime.h"

namespace aem {

namespace {

constexpr int kWarps = 8;

template <typename XT>
__device__ __forceinline__ float load_x(const XT* p);
template <>
__device__ __forceinline__ float load_x<float>(const float* p) {
    return *p;
}
template <>
__device__ __forceinline__ float load_x<__nv_bfloat16>(const __nv_bfloat16* p) {
    return __bfloat162float(*p);
}

constexpr int kStages = 3;  // depth of the cp.async ring

__device__ __forceinline__ void cp_async_16(void* dst, const void* src, int src_bytes) {
    // copies src_bytes (0..16) and zero-fills the rest of the 16 bytes
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dev::smem_u32(dst)),
                 "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int NPENDING>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(NPENDING) : "memory");
}

// Compile-time shape of one kernel configuration.
template <int GROUP, int NSLOT, int TPG, int WARPS, typename XT, int DKO = 0>
struct GatingCfg {
    static constexpr int kThreads = WARPS * 32;
    static constexpr int GPW = 32 / GROUP;
    static constexpr int TOK = WARPS * GPW * TPG;  // tokens per CTA
    static constexpr int EPAD = GROUP * NSLOT;
    static constexpr int DK_E = DKO ? DKO : (EPAD <= 64 ? 64 : (EPAD <= 128 ? 32 : 16));
    static constexpr int DK = (TOK * (DK_E + 4) * 4 > 36 * 1024) ? DK_E / 2 : DK_E;
    static constexpr int DK4 = DK / 4;
    // float32 activations of a chunk, token pairs interleaved: pair p's row
    // holds, for every 4 consecutive d, (t0 d0, t1 d0, t0 d1, t1 d1, t0 d2,
    // t1 d2, t0 d3, t1 d3) with t0 = 2p, t1 = 2p+1 -- two 16-byte loads
    // give both tokens' activations for the 4 d of one weight float4; rows
    // padded against bank conflicts
    static constexpr int XS = 2 * DK + 4;
    static constexpr int XB = static_cast<int>(sizeof(XT));
    static constexpr int XPC = 16 / XB;     // activation elements per 16-byte piece
    static constexpr int XCH = DK / XPC;    // pieces per token row of a chunk
    static constexpr int WST = DK4 * EPAD;  // float4 per weight stage
    static constexpr int XST = TOK * XCH;   // 16-byte pieces per activation stage
    static constexpr size_t SMEM =
        16 * static_cast<size_t>(kStages) * (WST + XST) + 4 * static_cast<size_t>(TOK / 2) * XS;
    static_assert(DK % XPC == 0, "activation chunk must be whole 16-byte pieces");
    static_assert(TPG % 2 == 0, "tokens are processed in pairs");
};

// Packed fused multiply-add of two float32 lanes, each rounded once.
__device__ __forceinline__ float2 fma_rn2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// Selection key of a logit in np.argmax order: every NaN ranks above every
// number (np.argmax returns the first NaN), -0.0 ranks equal to +0.0, and
// otherwise the float order; the low word (0xFFFFFFFF - expert) makes the
// lowest expert id win between equal keys.  Keys of real experts are > 0.
__device__ __forceinline__ uint64_t select_key(float v, int e) {
    uint32_t u = __float_as_uint(__fadd_rn(v, 0.0f));  // -0.0 + 0.0 = +0.0
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);     // monotone map of the float order
    if (v != v) u = 0xFFFFFFFFu;                         // NaN above +inf
    return (static_cast<uint64_t>(u) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(e));
}

// Top-k of one token's logits held by a group of GROUP lanes (lane le owns
// experts le + GROUP*s; v = logit + bias): ksel rounds of np.argmax over the
// row (prototype/math_proto.py:38-42; for finite logits the strict-greater
// scan of fused_gating_metal.py:284-293, lowest id on ties), every lane
// learns each winner, lane 0 writes the index and exp(value - first value).
// Like the reference, a winner is not removed but overwritten with -inf, so a
// row with fewer than ksel logits above -inf selects its lowest -inf id
// again, and the value recorded is the row's current one (NaN for a NaN, -inf
// for a repeat).  The first k are normalised by their float32 sum in
// selection order.
template <int GROUP, int NSLOT>
__device__ __forceinline__ void topk_select(float (&v)[NSLOT], int le, unsigned gmask, int64_t tg,
                                            int64_t N, int E, int k, int ksel,
                                            int32_t* __restrict__ idx_out,
                                            float* __restrict__ val_out) {
    float m = 0.0f, sum = 0.0f;
    for (int kk = 0; kk < ksel; ++kk) {
        uint64_t bkey = 0;  // below every real expert's key
        float best = 0.0f;
#pragma unroll
        for (int s = 0; s < NSLOT; ++s) {
            const int e = le + GROUP * s;
            const uint64_t key = select_key(v[s], e);
            if (e < E && key > bkey) {
                bkey = key;
                best = v[s];
            }
        }
#pragma unroll
        for (int off = GROUP / 2; off >= 1; off >>= 1) {
            const uint64_t ok = __shfl_xor_sync(gmask, bkey, off, GROUP);
            const float ob = __shfl_xor_sync(gmask, best, off, GROUP);
            if (ok > bkey) {
                bkey = ok;
                best = ob;
            }
        }
        const int beste = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(bkey));
        // overwrite the winner in its owner lane (np.argmax's `local[best] = -inf`)
#pragma unroll
        for (int s = 0; s < NSLOT; ++s)
            if (le + GROUP * s == beste) v[s] = -INFINITY;
        if (kk == 0) m = best;
        const float ev = kk < k ? expf(best - m) : 0.0f;
        if (kk < k) sum = __fadd_rn(sum, ev);
        if (le == 0 && tg < N) {
            idx_out[tg * ksel + kk] = beste;
            if (kk < k) val_out[tg * k + kk] = ev;
        }
    }
    __syncwarp(gmask);
    if (tg < N)
        for (int kk = le; kk < k; kk += GROUP)
            val_out[tg * k + kk] = __fdiv_rn(val_out[tg * k + kk], sum);
    __syncwarp(gmask);
}

// ---------------------------------------------------------------------------
// CERTIFIED mode.  Fast logits F (fused multiply-adds, any order of d split
// into 64-wide blocks) come with a bound B such that the EXACT logit (float32
// products summed in increasing d order, then + bias) lies in [F - B, F + B].
// With P_i the partial sums and a_j >= sum over block j of |x_d w_d|:
//   * the EXACT sum's rounding is at most u * (sum_i |P_i| + sum |p_i|),
//   * a chain of fused multiply-adds' rounding is at most u * sum_i |acc_i|,
//   * inside a block every partial sum is within a_j of the block's end, so
//     sum_i |P_i| over the block <= 64 * (|P at the block end| + a_j),
//   * parts of d summed separately and then added carry their start offsets
//     (sum over a part of |P_i| <= part length * |P at the part start| + the
//     part's own bound) and one rounding per addition,
// so with Q = sum over blocks of (64 |P_end| + 65 a_j) (plus the parts'
// offsets) and Qc = sum over parts of (|P_start| + |S_part|),
//   |F - EXACT| <= u (2 Q + Qc + 2|F| + 2|b|) (1 + O(D u)),
// and B = 4 u (Q + Qc + |F| + |b|) leaves a margin for the second-order terms
// and the float32 rounding of the bound itself.  a_j is the Cauchy-Schwarz
// bound |x_block| |w_block| (norms precomputed for the weights, per token and
// block for the activations).  u = 2^-24.
constexpr float kCertU4 = 4.0f * 5.9604645e-8f;

// Certification of one token's selection from fast logits F and bounds B
// held by a group of GROUP lanes (lane le owns experts le + GROUP*s): true
// when every logit is finite, the top ksel (by F, ties to the lowest id) have
// pairwise ordered intervals (each one's lower end above the next one's upper
// end) and the last one's lower end is above every unselected expert's upper
// end -- then the EXACT logits select the same experts in the same order.
template <int GROUP, int NSLOT>
__device__ __forceinline__ bool certify_row(const float (&F)[NSLOT], const float (&B)[NSLOT],
                                            int le, unsigned gmask, int E, int ksel) {
    bool fin = true;
#pragma unroll
    for (int s = 0; s < NSLOT; ++s) {
        const int e = le + GROUP * s;
        if (e < E && !(isfinite(F[s]) && isfinite(B[s]))) fin = false;
    }
    if (!__all_sync(gmask, fin)) return false;
    bool sel[NSLOT];
#pragma unroll
    for (int s = 0; s < NSLOT; ++s) sel[s] = false;
    bool ok = true;
    float prev_lo = 0.0f;
    for (int kk = 0; kk < ksel; ++kk) {
        uint64_t bkey = 0;
        float bf = 0.0f, bb = 0.0f;
#pragma unroll
        for (int s = 0; s < NSLOT; ++s) {
            const int e = le + GROUP * s;
            const uint64_t key = select_key(F[s], e);
            if (e < E && !sel[s] && key > bkey) {
                bkey = key;
                bf = F[s];
                bb = B[s];
            }
        }
#pragma unroll
        for (int off = GROUP / 2; off >= 1; off >>= 1) {
            const uint64_t ok2 = __shfl_xor_sync(gmask, bkey, off, GROUP);
            const float of = __shfl_xor_sync(gmask, bf, off, GROUP);
            const float ob = __shfl_xor_sync(gmask, bb, off, GROUP);
            if (ok2 > bkey) {
                bkey = ok2;
                bf = of;
                bb = ob;
            }
        }
        const int beste = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(bkey));
#pragma unroll
        for (int s = 0; s < NSLOT; ++s)
            if (le + GROUP * s == beste) sel[s] = true;
        if (kk > 0 && !(prev_lo > bf + bb)) ok = false;
        prev_lo = bf - bb;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int s = 0; s < NSLOT; ++s) {
        const int e = le + GROUP * s;
        if (e < E && !sel[s]) mx = fmaxf(mx, F[s] + B[s]);
    }
#pragma unroll
    for (int off = GROUP / 2; off >= 1; off >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(gmask, mx, off, GROUP));
    if (ksel < E && !(prev_lo > mx)) ok = false;
    return ok;
}

// Appends row tg to the uncertified list (rows[0] = count).
__device__ __forceinline__ void cert_defer(int* rows, int64_t tg) {
    const int i = atomicAdd(rows, 1);
    rows[1 + i] = static_cast<int>(tg);
}

template <int GROUP, int NSLOT, int kTPG, int WARPS, typename XT, bool EXACT, int DKO = 0,
          bool CERT = false>
__global__ void __launch_bounds__(WARPS * 32)
    gating_kernel(const XT* __restrict__ x, const float4* __restrict__ wpk,
                  const float* __restrict__ bias, int64_t N, int D, int E, int k, int ksel,
                  int32_t* __restrict__ idx_out, float* __restrict__ val_out,
                  const float* __restrict__ wsq16, int* __restrict__ cert_rows,
                  const int* __restrict__ rowlist, unsigned long long* __restrict__ rows_total,
                  float one, float neg0) {
    using C = GatingCfg<GROUP, NSLOT, kTPG, WARPS, XT, DKO>;
    // 1.0 and -0.0 arrive as launch arguments, so the compiler cannot fold
    // the EXACT mode's fused multiply-adds below back into a plain multiply
    // and add (which it may then contract into one fused multiply-add)
    const float2 one2 = make_float2(one, one);
    const float2 nz2 = make_float2(neg0, neg0);
    constexpr int kThreads = C::kThreads;
    constexpr int GPW = C::GPW;
    constexpr int TOK = C::TOK;
    constexpr int EPAD = C::EPAD;
    constexpr int DK = C::DK;
    constexpr int DK4 = C::DK4;
    constexpr int XS = C::XS;
    constexpr int XB = C::XB;
    constexpr int XPC = C::XPC;
    constexpr int XCH = C::XCH;
    constexpr int WST = C::WST;
    constexpr int XST = C::XST;

    // Shared memory: a kStages-deep ring of weight chunks and raw activation
    // chunks filled by cp.async (16-byte asynchronous copies, zero-filled past
    // the end of the data), and the current chunk's activations as float32.
    extern __shared__ __align__(16) unsigned char gsm[];
    float4* wring = reinterpret_cast<float4*>(gsm);
    uint4* xring = reinterpret_cast<uint4*>(gsm + sizeof(float4) * kStages * WST);
    float* xs = reinterpret_cast<float*>(xring + kStages * XST);
    float* xn = xs + (TOK / 2) * XS;  // CERTIFIED: |x| of the chunk, per token

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int grp = lane / GROUP;
    const int le = lane % GROUP;
    const int64_t tok0 = static_cast<int64_t>(blockIdx.x) * TOK;
    const int tbase = (warp * GPW + grp) * kTPG;  // first local token of this lane group
    // With a row list (rowlist[0] = count, then row ids: the rows a certified
    // launch deferred) token tl of the grid is row rowlist[1 + tl]; the grid
    // is sized for every row and the CTAs past the count leave at once.
    __shared__ int64_t s_row[TOK];
    if (rowlist) {
        const int64_t n_eff = min(N, static_cast<int64_t>(rowlist[0]));
        if (blockIdx.x == 0 && tid == 0 && rows_total && n_eff > 0)
            atomicAdd(rows_total, static_cast<unsigned long long>(n_eff));
        if (tok0 >= n_eff) return;  // uniform over the CTA
        for (int i = tid; i < TOK; i += kThreads)
            s_row[i] = tok0 + i < n_eff ? static_cast<int64_t>(rowlist[1 + tok0 + i]) : N;
        __syncthreads();
    }
    auto row_of = [&](int tl) -> int64_t { return rowlist ? s_row[tl] : tok0 + tl; };

    float2 acc[kTPG / 2][NSLOT];  // (token 2p, token 2p+1) of this lane group
    float2 qb[kTPG / 2][NSLOT];   // CERTIFIED: the bound's sum Q (see certify_row)
#pragma unroll
    for (int i = 0; i < kTPG / 2; ++i)
#pragma unroll
        for (int s = 0; s < NSLOT; ++s) {
            acc[i][s] = make_float2(0.0f, 0.0f);
            qb[i][s] = make_float2(0.0f, 0.0f);
        }

    // activation rows can be copied in 16-byte pieces when every row start is aligned
    const bool xvec = (static_cast<int64_t>(D) * XB) % 16 == 0 &&
                      (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const int nchunks = (D + DK - 1) / DK;
    // Issues chunk c's copies (if it exists) and always commits a group, so
    // that "all but the newest kStages-1 groups complete" means chunk c landed.
    auto issue = [&](int c) {
        if (c < nchunks) {
            const int st = c % kStages;
            const float4* wsrc = wpk + static_cast<int64_t>(c) * WST;  // Dpad: whole chunks of <= 256
            float4* wdst = wring + st * WST;
            for (int i = tid; i < WST; i += kThreads) cp_async_16(wdst + i, wsrc + i, 16);
            if (xvec) {
                const int d0 = c * DK;
                uint4* xdst = xring + st * XST;
                for (int i = tid; i < XST; i += kThreads) {
                    const int t = i / XCH;
                    const int d = d0 + (i % XCH) * XPC;
                    const int64_t tg = row_of(t);
                    const bool in = tg < N && d < D;
                    const XT* src = in ? x + tg * static_cast<int64_t>(D) + d : x;
                    cp_async_16(xdst + i, src, in ? min(16, (D - d) * XB) : 0);
                }
            }
        }
        cp_async_commit();
    };
    for (int c = 0; c < kStages - 1; ++c) issue(c);
    for (int c = 0; c < nchunks; ++c) {
        issue(c + kStages - 1);
        cp_async_wait<kStages - 1>();
        __syncthreads();  // chunk c is in its stage, from every thread's copies
        const int st = c % kStages;
        const float4* ws = wring + st * WST;
        // the chunk's activations as float32 rows (padded against bank conflicts)
        auto xpos = [&](int i) {  // element (token i / DK, d i % DK) in the pair layout
            const int t = i / DK, dd = i % DK;
            return (t >> 1) * XS + (dd >> 2) * 8 + (dd & 3) * 2 + (t & 1);
        };
        if (xvec) {
            const XT* xr = reinterpret_cast<const XT*>(xring + st * XST);
            for (int i = tid; i < TOK * DK; i += kThreads) xs[xpos(i)] = load_x<XT>(xr + i);
        } else {
            const int d0 = c * DK;
            for (int i = tid; i < TOK * DK; i += kThreads) {
                const int64_t tg = row_of(i / DK);
                const int d = d0 + i % DK;
                xs[xpos(i)] =
                    (tg < N && d < D) ? load_x<XT>(x + tg * static_cast<int64_t>(D) + d) : 0.0f;
            }
        }
        __syncthreads();
#pragma unroll 4
        for (int q = 0; q < DK4; ++q) {
            // xa[p] = (t0 d0, t1 d0, t0 d1, t1 d1), xb[p] = (t0 d2, t1 d2, t0 d3, t1 d3)
            float4 xa[kTPG / 2], xb[kTPG / 2];
#pragma unroll
            for (int p = 0; p < kTPG / 2; ++p) {
                const float* row = &xs[(tbase / 2 + p) * XS + 8 * q];
                xa[p] = *reinterpret_cast<const float4*>(row);
                xb[p] = *reinterpret_cast<const float4*>(row + 4);
            }
#pragma unroll
            for (int s = 0; s < NSLOT; ++s) {
                const float4 wv = ws[q * EPAD + le + GROUP * s];
#pragma unroll
                for (int p = 0; p < kTPG / 2; ++p) {
                    float2 a = acc[p][s];
                    if constexpr (EXACT) {
                        // float32 product, then float32 add, d in increasing order,
                        // for the lane group's two tokens at once: the product as
                        // x*w + (-0.0) and the sum as p*1.0 + acc, packed fp32x2
                        // fused multiply-adds that each round exactly once like the
                        // plain multiply and add (x*w + -0 and p*1 are exact; a
                        // -0 product stays -0).  A packed multiply followed by a
                        // packed add was measured to round like one fused
                        // multiply-add, which reorders experts whose logits are
                        // 1 ulp apart; this form halves the scalar instruction count.
                        a = fma_rn2(fma_rn2(make_float2(xa[p].x, xa[p].y),
                                            make_float2(wv.x, wv.x), nz2), one2, a);
                        a = fma_rn2(fma_rn2(make_float2(xa[p].z, xa[p].w),
                                            make_float2(wv.y, wv.y), nz2), one2, a);
                        a = fma_rn2(fma_rn2(make_float2(xb[p].x, xb[p].y),
                                            make_float2(wv.z, wv.z), nz2), one2, a);
                        a = fma_rn2(fma_rn2(make_float2(xb[p].z, xb[p].w),
                                            make_float2(wv.w, wv.w), nz2), one2, a);
                    } else {
                        a.x = fmaf(xa[p].x, wv.x, a.x);
                        a.y = fmaf(xa[p].y, wv.x, a.y);
                        a.x = fmaf(xa[p].z, wv.y, a.x);
                        a.y = fmaf(xa[p].w, wv.y, a.y);
                        a.x = fmaf(xb[p].x, wv.z, a.x);
                        a.y = fmaf(xb[p].y, wv.z, a.y);
                        a.x = fmaf(xb[p].z, wv.w, a.x);
                        a.y = fmaf(xb[p].w, wv.w, a.y);
                    }
                    acc[p][s] = a;
                }
            }
        }
        if constexpr (CERT) {
            // |x| over this chunk, per token (warps over tokens, lanes over d)
            for (int t = warp; t < TOK; t += WARPS) {
                float ss = 0.0f;
                for (int dd = lane; dd < DK; dd += 32) {
                    const float v = xs[(t >> 1) * XS + (dd >> 2) * 8 + (dd & 3) * 2 + (t & 1)];
                    ss = fmaf(v, v, ss);
                }
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
                if (lane == 0) xn[t] = sqrtf(ss);
            }
        }
        __syncthreads();  // the stage and xs are rewritten next
        if constexpr (CERT) {
            // Q += DK |P at the chunk's end| + (DK + 1) |x_chunk| |w_chunk|
            float wn[NSLOT];
#pragma unroll
            for (int s = 0; s < NSLOT; ++s) {
                const int e = le + GROUP * s;
                float sq = 0.0f;
                for (int b = 0; b < DK / 16; ++b) sq += __ldg(wsq16 + (c * (DK / 16) + b) * EPAD + e);
                wn[s] = sqrtf(sq);
            }
#pragma unroll
            for (int p = 0; p < kTPG / 2; ++p) {
                const float x0 = xn[tbase + 2 * p], x1 = xn[tbase + 2 * p + 1];
#pragma unroll
                for (int s = 0; s < NSLOT; ++s) {
                    qb[p][s].x += static_cast<float>(DK) * fabsf(acc[p][s].x) +
                                  static_cast<float>(DK + 1) * x0 * wn[s];
                    qb[p][s].y += static_cast<float>(DK) * fabsf(acc[p][s].y) +
                                  static_cast<float>(DK + 1) * x1 * wn[s];
                }
            }
        }
    }
    cp_async_wait<0>();

    // ---- bias, top-k selection, softmax (per lane group, per token)
    float bv[NSLOT];
#pragma unroll
    for (int s = 0; s < NSLOT; ++s) {
        const int e = le + GROUP * s;
        bv[s] = e < E ? __ldg(bias + e) : 0.0f;
    }
    const unsigned gmask =
        GROUP == 32 ? 0xFFFFFFFFu : (((1u << GROUP) - 1u) << (grp * GROUP));
#pragma unroll
    for (int i = 0; i < kTPG; ++i) {
        const int tl = tbase + i;
        const int64_t tg = row_of(tl);
        float v[NSLOT];
#pragma unroll
        for (int s = 0; s < NSLOT; ++s) {
            const int e = le + GROUP * s;
            const float lg = (i & 1) ? acc[i >> 1][s].y : acc[i >> 1][s].x;
            v[s] = e < E ? __fadd_rn(lg, bv[s]) : -FLT_MAX;
        }
        if constexpr (CERT) {
            float bnd[NSLOT];
#pragma unroll
            for (int s = 0; s < NSLOT; ++s) {
                const float q = (i & 1) ? qb[i >> 1][s].y : qb[i >> 1][s].x;
                bnd[s] = kCertU4 * (q + fabsf(v[s]) + fabsf(bv[s]));
            }
            if (!certify_row<GROUP, NSLOT>(v, bnd, le, gmask, E, ksel)) {
                if (le == 0 && tg < N) cert_defer(cert_rows, tg);
                continue;
            }
        }
        topk_select<GROUP, NSLOT>(v, le, gmask, tg, N, E, k, ksel, idx_out, val_out);
    }
}

// ---------------------------------------------------------------------------
// Small batches (decode sizes): experts split over the CTAs of a cluster.
//
// With few tokens the work is a handful of long sequential dot products, so
// the time is one float32 add chain of D steps, as long as the operands keep
// flowing.  The kernel spreads the gate's experts over the CL CTAs of a
// thread-block cluster (EB experts each) and the tokens over clusters (TT per
// CTA); every consumer thread owns ONE (token, expert) logit and walks d in
// increasing order (EXACT: float32 product, float32 add).  A producer warp
// streams chunks of d (up to 512 wide) -- the CTA's expert block of the weights (one
// contiguous bulk copy in the expert-block layout) and its tokens' activation
// rows (one bulk copy per row) -- through a ring of mbarrier-tracked stages,
// so no CTA-wide barrier interrupts the chains.  At the end every thread
// stores its logit + bias into the leader CTA's shared memory (DSMEM), the
// cluster synchronises, and the leader selects the top-k of each token with
// the same selection as the large-batch kernel.  Every mbarrier wait is
// bounded (globaltimer); a timeout sets an error bit and the roles run out,
// so the cluster barrier is always reached by every thread.
constexpr int kSmallStages = 4;
constexpr int kSmallCons = 128;   // consumer threads (warps 0-3); warp 4 produces
constexpr int kSmallThreads = kSmallCons + 32;

template <int EPAD, typename XT>
struct SmallCfg {
    static constexpr int EB = EPAD / 8 > 8 ? EPAD / 8 : 8;  // experts per CTA
    static constexpr int CL = EPAD / EB;                   // CTAs per cluster (<= 8)
    static constexpr int TT = kSmallCons / EB;             // tokens per CTA
    // d per stage: 16 KB of weights per stage (512 d for up to 64 experts),
    // so four stages keep about 4 us of the add chain's operands in flight
    // with few, large bulk copies
    static constexpr int DK = 4096 / EB > 512 ? 512 : 4096 / EB;
    static constexpr int XB = static_cast<int>(sizeof(XT));
    static constexpr int XROW = DK * XB + 16;              // padded activation row, bytes
    static constexpr int WST = DK / 4 * EB * 16;           // weight stage, bytes
    static constexpr int XST = TT * XROW;                  // activation stage, bytes
    static constexpr int LG = TT * EPAD * 4;               // gathered logits, bytes
    static constexpr int SMEM = kSmallStages * (WST + XST) + LG + 2 * kSmallStages * 8 + 16;
    static_assert(CL >= 1 && CL <= 8 && EB * CL == EPAD && TT * EB == kSmallCons, "shape");
    static_assert((DK * XB) % 16 == 0 && XROW % 16 == 0 && WST % 16 == 0, "16-byte copies");
    static_assert(DK % 64 == 0 && SMEM <= 227 * 1024, "chunk and shared memory");
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Stores v at the same shared-memory offset as `local` in CTA `rank` of the cluster.
__device__ __forceinline__ void st_cluster_f32(const float* local, uint32_t rank, float v) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                 : "=r"(remote)
                 : "r"(dev::smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// Raw activations of 4 consecutive d as loaded from shared memory (float32:
// 16 bytes; bf16: 8 bytes in .x/.y), widened to float32 only when used, so
// that a block of loads can be issued ahead of the add chain.
template <typename XT>
__device__ __forceinline__ uint4 load_x4_raw(const unsigned char* p);
template <>
__device__ __forceinline__ uint4 load_x4_raw<float>(const unsigned char* p) {
    return *reinterpret_cast<const uint4*>(p);
}
template <>
__device__ __forceinline__ uint4 load_x4_raw<__nv_bfloat16>(const unsigned char* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    return make_uint4(u.x, u.y, 0u, 0u);
}
template <typename XT>
__device__ __forceinline__ float4 widen_x4(uint4 r);
template <>
__device__ __forceinline__ float4 widen_x4<float>(uint4 r) {
    return make_float4(__uint_as_float(r.x), __uint_as_float(r.y), __uint_as_float(r.z),
                       __uint_as_float(r.w));
}
template <>
__device__ __forceinline__ float4 widen_x4<__nv_bfloat16>(uint4 r) {
    return make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u),
                       __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xFFFF0000u));
}

// Marks a prefetched operand block as needed at this point of the program:
// the block's loads must be issued before it, so they overlap the add chain
// placed in front of it instead of sitting next to their uses.
__device__ __forceinline__ void pin4(const float4& w, const uint4& x) {
    asm volatile("" ::"f"(w.x), "f"(w.y), "f"(w.z), "f"(w.w), "r"(x.x), "r"(x.y), "r"(x.z),
                 "r"(x.w));
}

// One chain step over 4 consecutive d: float32 product, float32 add, in order.
template <bool EXACT>
__device__ __forceinline__ float chain4(float acc, float4 x, float4 w) {
    if constexpr (EXACT) {
        acc = __fadd_rn(acc, __fmul_rn(x.x, w.x));
        acc = __fadd_rn(acc, __fmul_rn(x.y, w.y));
        acc = __fadd_rn(acc, __fmul_rn(x.z, w.z));
        acc = __fadd_rn(acc, __fmul_rn(x.w, w.w));
    } else {
        acc = fmaf(x.x, w.x, acc);
        acc = fmaf(x.y, w.y, acc);
        acc = fmaf(x.z, w.z, acc);
        acc = fmaf(x.w, w.w, acc);
    }
    return acc;
}

template <int EPAD, typename XT, bool EXACT>
__global__ void __launch_bounds__(kSmallThreads, 1)
    gating_small_kernel(const XT* __restrict__ x, const float4* __restrict__ wblk,
                        const float* __restrict__ bias, int64_t N, int D, int64_t Dpad, int E,
                        int k, int ksel, int32_t* __restrict__ idx_out,
                        float* __restrict__ val_out, int* __restrict__ err) {
    using C = SmallCfg<EPAD, XT>;
    constexpr int EB = C::EB;
    constexpr int TT = C::TT;
    extern __shared__ __align__(128) unsigned char ssm[];
    unsigned char* wring = ssm;
    unsigned char* xring = wring + kSmallStages * C::WST;
    float* lg = reinterpret_cast<float*>(xring + kSmallStages * C::XST);
    uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(lg) + C::LG);
    uint64_t* empty = full + kSmallStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kSmallStages);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int cb = blockIdx.y;  // expert block = rank in the (1, CL, 1) cluster
    const int64_t tok0 = static_cast<int64_t>(blockIdx.x) * TT;
    const int rows = static_cast<int>(min(static_cast<int64_t>(TT), N - tok0));
    const int nch = (D + C::DK - 1) / C::DK;
    if (tid == 0) {
        for (int st = 0; st < kSmallStages; ++st) {
            dev::mbar_init(&full[st], 1);
            dev::mbar_init(&empty[st], kSmallCons / 32);
        }
        *abort_flag = 0;
        dev::fence_barrier_init();
    }
    __syncthreads();

    float acc = 0.0f;
    const int tl = tid / EB;  // consumer: local token
    const int el = tid % EB;  //           expert within the block
    if (warp == kSmallCons / 32) {
        // ---- producer: one lane issues the bulk copies of every chunk
        if (lane == 0) {
            const float4* wsrc = wblk + static_cast<int64_t>(cb) * (Dpad / 4) * EB;
            for (int c = 0; c < nch; ++c) {
                const int st = c % kSmallStages;
                const uint32_t ph = (c / kSmallStages) & 1;
                if (!dev::mbar_wait_bounded(&empty[st], ph ^ 1, abort_flag, err, ERR_GEMM_TIMEOUT))
                    break;
                const int dd = min(C::DK, D - c * C::DK);
                const uint32_t xb = static_cast<uint32_t>(dd * C::XB);
                // the packed gate is Dpad wide (a multiple of 256, not of the
                // chunk): the last chunk's weight copy stops at Dpad
                const int wd = static_cast<int>(
                    min(static_cast<int64_t>(C::DK), Dpad - static_cast<int64_t>(c) * C::DK));
                const uint32_t wb = static_cast<uint32_t>(wd / 4 * EB * 16);
                dev::mbar_arrive_expect_tx(&full[st], wb + rows * xb);
                dev::bulk_load(wring + st * C::WST, wsrc + static_cast<int64_t>(c) * (C::DK / 4) * EB,
                               wb, &full[st]);
                for (int r = 0; r < rows; ++r)
                    dev::bulk_load(xring + st * C::XST + r * C::XROW,
                                   x + (tok0 + r) * static_cast<int64_t>(D) + c * C::DK, xb,
                                   &full[st]);
            }
        }
    } else {
        // ---- consumers: one sequential chain each
        for (int c = 0; c < nch; ++c) {
            const int st = c % kSmallStages;
            const uint32_t ph = (c / kSmallStages) & 1;
            if (!dev::mbar_wait_bounded(&full[st], ph, abort_flag, err, ERR_GEMM_TIMEOUT)) break;
            const int n4 = min(C::DK, D - c * C::DK) >> 2;
            const float4* ws = reinterpret_cast<const float4*>(wring + st * C::WST) + el;
            const unsigned char* xs = xring + st * C::XST + tl * C::XROW;
            if (n4 == C::DK / 4) {
                // A whole chunk: operands of the next 32 d are loaded into
                // registers while the chain runs over the current 32 (one warp
                // per scheduler, so the loads must be issued well ahead).
                constexpr int QB = 8;
                float4 wa[QB], wb[QB];
                uint4 xa[QB], xb[QB];
#pragma unroll
                for (int i = 0; i < QB; ++i) {
                    wa[i] = ws[i * EB];
                    xa[i] = load_x4_raw<XT>(xs + i * 4 * C::XB);
                }
#pragma unroll
                for (int b = 0; b < C::DK / 4 / QB; b += 2) {
#pragma unroll
                    for (int i = 0; i < QB; ++i) {
                        wb[i] = ws[((b + 1) * QB + i) * EB];
                        xb[i] = load_x4_raw<XT>(xs + ((b + 1) * QB + i) * 4 * C::XB);
                    }
#pragma unroll
                    for (int i = 0; i < QB; ++i) acc = chain4<EXACT>(acc, widen_x4<XT>(xa[i]), wa[i]);
#pragma unroll
                    for (int i = 0; i < QB; ++i) pin4(wb[i], xb[i]);
                    if (b + 2 < C::DK / 4 / QB) {
#pragma unroll
                        for (int i = 0; i < QB; ++i) {
                            wa[i] = ws[((b + 2) * QB + i) * EB];
                            xa[i] = load_x4_raw<XT>(xs + ((b + 2) * QB + i) * 4 * C::XB);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < QB; ++i) acc = chain4<EXACT>(acc, widen_x4<XT>(xb[i]), wb[i]);
                    if (b + 2 < C::DK / 4 / QB) {
#pragma unroll
                        for (int i = 0; i < QB; ++i) pin4(wa[i], xa[i]);
                    }
                }
            } else {
#pragma unroll 4
                for (int q = 0; q < n4; ++q)
                    acc = chain4<EXACT>(acc, widen_x4<XT>(load_x4_raw<XT>(xs + q * 4 * C::XB)),
                                        ws[q * EB]);
            }
            __syncwarp();
            if (lane == 0) dev::mbar_arrive(&empty[st]);
        }
        const int e = cb * EB + el;
        const float v = __fadd_rn(acc, __ldg(bias + e));  // bias padded to EPAD with zeros
        if constexpr (C::CL == 1)
            lg[tl * EPAD + e] = v;
        else
            st_cluster_f32(&lg[tl * EPAD + e], 0, v);
    }
    __syncwarp();
    if constexpr (C::CL == 1)
        __syncthreads();
    else
        cluster_sync_all();  // every CTA's logits are in the leader's shared memory
    if (cb != 0 || warp >= kSmallCons / 32) return;

    // ---- leader: top-k of each token (lane groups own experts)
    constexpr int GROUP = EPAD >= 32 ? 32 : EPAD;
    constexpr int NSLOT = EPAD / GROUP;
    constexpr int GPW = 32 / GROUP;
    const int grp = lane / GROUP;
    const int le = lane % GROUP;
    const unsigned gmask = GROUP == 32 ? 0xFFFFFFFFu : (((1u << GROUP) - 1u) << (grp * GROUP));
    for (int t = warp * GPW + grp; t < rows; t += (kSmallCons / 32) * GPW) {
        float v[NSLOT];
#pragma unroll
        for (int s2 = 0; s2 < NSLOT; ++s2) v[s2] = lg[t * EPAD + le + GROUP * s2];
        topk_select<GROUP, NSLOT>(v, le, gmask, tok0 + t, N, E, k, ksel, idx_out, val_out);
    }
}

template <int EPAD, typename XT, bool EXACT>
cudaError_t launch_small_e(const Gate& g, const void* x, int64_t N, int k, int ksel, int32_t* idx,
                           float* val, int* err, cudaStream_t s) {
    using C = SmallCfg<EPAD, XT>;
    auto kern = gating_small_kernel<EPAD, XT, EXACT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((N + C::TT - 1) / C::TT), C::CL, 1);
    cfg.blockDim = dim3(kSmallThreads, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = C::CL;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<const XT*>(x),
                              reinterpret_cast<const float4*>(g.wblk),
                              static_cast<const float*>(g.bias), N, static_cast<int>(g.D), g.Dpad,
                              static_cast<int>(g.E), k, ksel, idx, val, err);
}

template <typename XT, bool EXACT>
cudaError_t launch_small(const Gate& g, const void* x, int64_t N, int k, int ksel, int32_t* idx,
                         float* val, int* err, cudaStream_t s) {
    switch (g.Epad) {
        case 8: return launch_small_e<8, XT, EXACT>(g, x, N, k, ksel, idx, val, err, s);
        case 16: return launch_small_e<16, XT, EXACT>(g, x, N, k, ksel, idx, val, err, s);
        case 32: return launch_small_e<32, XT, EXACT>(g, x, N, k, ksel, idx, val, err, s);
        case 64: return launch_small_e<64, XT, EXACT>(g, x, N, k, ksel, idx, val, err, s);
        case 128: return launch_small_e<128, XT, EXACT>(g, x, N, k, ksel, idx, val, err, s);
        default: return launch_small_e<256, XT, EXACT>(g, x, N, k, ksel, idx, val, err, s);
    }
}

// CERTIFIED mode for few tokens: d split over threads.  A CTA takes kCertTT
// tokens and all experts; thread (e, p) of the 256 sums expert e's products
// over part p of d (P = 256 / EPAD contiguous parts, whole 64-wide blocks)
// with fused multiply-adds for the CTA's tokens, keeping per block the
// bound's sum Q (64 |P_end| + 65 |x_block| |w_block|); one thread per
// (token, expert) then adds the parts in order, carrying their start offsets
// into Q (part length * |P_start|) and the additions' own rounding into Qc,
// and a warp per token certifies and selects.  The activation rows and
// their per-block norms live in shared memory; the weights are read from the
// packed [Dpad/4][Epad][4] layout (L2-resident, shared by the CTA's tokens).
constexpr int kCertTT = 4;
constexpr int kCertThreads = 256;

__host__ __device__ constexpr size_t cert_small_smem(int64_t Dpad, int EPAD) {
    return sizeof(float) * (static_cast<size_t>(kCertTT) * Dpad +      // activations
                            static_cast<size_t>(kCertTT) * (Dpad / 64) +  // block norms
                            2 * static_cast<size_t>(kCertTT) * kCertThreads +  // part sums, Q
                            2 * static_cast<size_t>(kCertTT) * EPAD);      // logits, bounds
}

template <int EPAD, typename XT>
__global__ void __launch_bounds__(kCertThreads)
    gating_cert_small_kernel(const XT* __restrict__ x, const float4* __restrict__ wpk,
                             const float* __restrict__ bias, const float* __restrict__ wn64,
                             int64_t N, int D, int64_t Dpad, int E, int k, int ksel,
                             int32_t* __restrict__ idx_out, float* __restrict__ val_out,
                             int* __restrict__ cert_rows) {
    constexpr int P = kCertThreads / EPAD;  // parts of d
    constexpr int TT = kCertTT;
    extern __shared__ __align__(16) float csm[];
    float* xs = csm;                                   // [TT][Dpad]
    float* xnb = xs + TT * Dpad;                       // [TT][Dpad/64]
    float* ps = xnb + TT * (Dpad / 64);                // [TT][P][EPAD] part sums
    float* pq = ps + TT * kCertThreads;                // [TT][P][EPAD] part Q
    float* fl = pq + TT * kCertThreads;                // [TT][EPAD] fast logits
    float* fb = fl + TT * EPAD;                        // [TT][EPAD] bounds
    const int tid = threadIdx.x;
    const int64_t tok0 = static_cast<int64_t>(blockIdx.x) * TT;
    const int nblk = static_cast<int>(Dpad / 64);
    // activation rows as float32, zero past D and past N (16-byte loads when
    // the rows allow them)
    constexpr int VEC = 16 / static_cast<int>(sizeof(XT));
    const bool vec = (static_cast<int64_t>(D) * static_cast<int>(sizeof(XT))) % 16 == 0 &&
                     (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const int dp = static_cast<int>(Dpad);
#pragma unroll 1
    for (int t = 0; t < TT; ++t) {
        float* dst = xs + t * dp;
        if (tok0 + t >= N) {
            for (int d = tid; d < dp; d += kCertThreads) dst[d] = 0.0f;
            continue;
        }
        const XT* row = x + (tok0 + t) * static_cast<int64_t>(D);
        const int d0 = vec ? D / VEC * VEC : 0;
        for (int d = d0 + tid; d < dp; d += kCertThreads)
            dst[d] = d < D ? load_x<XT>(row + d) : 0.0f;
    }
    if (vec) {
        // the 16-byte pieces of all the CTA's rows in flight together
        for (int j = tid; j < D / VEC; j += kCertThreads) {
            uint4 v[TT];
#pragma unroll
            for (int t = 0; t < TT; ++t)
                v[t] = tok0 + t < N ? *reinterpret_cast<const uint4*>(
                                          x + (tok0 + t) * static_cast<int64_t>(D) + j * VEC)
                                    : make_uint4(0, 0, 0, 0);
            asm volatile("" ::: "memory");
#pragma unroll
            for (int t = 0; t < TT; ++t) {
                const XT* e8 = reinterpret_cast<const XT*>(&v[t]);
#pragma unroll
                for (int q = 0; q < VEC; q += 4)
                    *reinterpret_cast<float4*>(xs + t * dp + j * VEC + q) =
                        make_float4(load_x<XT>(e8 + q), load_x<XT>(e8 + q + 1),
                                    load_x<XT>(e8 + q + 2), load_x<XT>(e8 + q + 3));
            }
        }
    }
    __syncthreads();
    {
        // a warp per block: two elements per lane, then a shuffle sum
        const int w = tid >> 5, ln = tid & 31;
        for (int i = w; i < TT * nblk; i += kCertThreads / 32) {
            const float* v = xs + (i / nblk) * dp + (i % nblk) * 64;
            float ss = v[ln] * v[ln];
            ss = fmaf(v[ln + 32], v[ln + 32], ss);
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
            if (ln == 0) xnb[i] = sqrtf(ss);
        }
    }
    __syncthreads();
    // ---- part p of d for expert e, all TT tokens
    const int e = tid % EPAD;
    const int p = tid / EPAD;
    const int bpp = (nblk + P - 1) / P;  // blocks per part
    const int b0 = p * bpp, b1 = min(nblk, b0 + bpp);
    float acc[TT], q[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        acc[t] = 0.0f;
        q[t] = 0.0f;
    }
    // two blocks per round: their 32 weight vectors and 2 norms in flight
    // together (the barrier keeps the compiler from moving loads to their uses)
    for (int b = b0; b < b1; b += 2) {
        const bool two = b + 1 < b1;
        float4 wv[32];
#pragma unroll
        for (int j = 0; j < 16; ++j) wv[j] = __ldg(wpk + static_cast<int64_t>(b * 16 + j) * EPAD + e);
#pragma unroll
        for (int j = 0; j < 16; ++j)
            wv[16 + j] = two ? __ldg(wpk + static_cast<int64_t>((b + 1) * 16 + j) * EPAD + e)
                             : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        const float wn0 = __ldg(wn64 + static_cast<int64_t>(b) * EPAD + e);
        const float wn1 = two ? __ldg(wn64 + static_cast<int64_t>(b + 1) * EPAD + e) : 0.0f;
        asm volatile("" ::: "memory");
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (h == 1 && !two) break;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int d4 = (b + h) * 16 + j;
#pragma unroll
                for (int t = 0; t < TT; ++t) {
                    const float4 xv = *reinterpret_cast<const float4*>(xs + t * dp + 4 * d4);
                    acc[t] = fmaf(xv.x, wv[16 * h + j].x, acc[t]);
                    acc[t] = fmaf(xv.y, wv[16 * h + j].y, acc[t]);
                    acc[t] = fmaf(xv.z, wv[16 * h + j].z, acc[t]);
                    acc[t] = fmaf(xv.w, wv[16 * h + j].w, acc[t]);
                }
            }
            const float wn = h ? wn1 : wn0;
#pragma unroll
            for (int t = 0; t < TT; ++t)
                q[t] += 64.0f * fabsf(acc[t]) + 65.0f * xnb[t * nblk + b + h] * wn;
        }
    }
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        ps[t * kCertThreads + tid] = acc[t];
        pq[t * kCertThreads + tid] = q[t];
    }
    __syncthreads();
    // ---- parts in order: logit, Q with the parts' offsets, Qc
    for (int i = tid; i < TT * EPAD; i += kCertThreads) {
        const int t = i / EPAD, ee = i % EPAD;
        float run = 0.0f, Q = 0.0f, Qc = 0.0f;
        for (int pp = 0; pp < P; ++pp) {
            const float sp = ps[t * kCertThreads + pp * EPAD + ee];
            Q += pq[t * kCertThreads + pp * EPAD + ee] + 64.0f * bpp * fabsf(run);
            Qc += fabsf(run) + fabsf(sp);
            run += sp;
        }
        const float b = ee < E ? __ldg(bias + ee) : 0.0f;
        const float f = ee < E ? __fadd_rn(run, b) : -FLT_MAX;
        fl[i] = f;
        fb[i] = kCertU4 * (Q + Qc + fabsf(f) + fabsf(b));
    }
    __syncthreads();
    // ---- a warp per token: certify, then select from the fast logits or defer
    constexpr int GROUP = EPAD < 32 ? EPAD : 32;
    constexpr int NSLOT = EPAD / GROUP;
    const int warp = tid >> 5, lane = tid & 31;
    if (warp < TT && lane < GROUP) {
        const int t = warp;
        const int64_t tg = tok0 + t;
        const unsigned gmask = GROUP == 32 ? 0xFFFFFFFFu : ((1u << GROUP) - 1u);
        float v[NSLOT], bnd[NSLOT];
#pragma unroll
        for (int s2 = 0; s2 < NSLOT; ++s2) {
            v[s2] = fl[t * EPAD + lane + GROUP * s2];
            bnd[s2] = fb[t * EPAD + lane + GROUP * s2];
        }
        if (tg < N) {
            if (certify_row<GROUP, NSLOT>(v, bnd, lane, gmask, E, ksel))
                topk_select<GROUP, NSLOT>(v, lane, gmask, tg, N, E, k, ksel, idx_out, val_out);
            else if (lane == 0)
                cert_defer(cert_rows, tg);
        }
    }
}

// Squared norms of the packed weights per 16-wide block of d: out[b][e] =
// sum over d in [16b, 16b+16) of w[d][e]^2, [Dpad/16][Epad].
__global__ void gate_norms_kernel(const float4* __restrict__ wpk, int64_t Dpad, int64_t Epad,
                                  float* __restrict__ out, float* __restrict__ out64) {
    const int64_t total = (Dpad / 16) * Epad;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = i / Epad, e = i % Epad;
        float ss = 0.0f;
        for (int j = 0; j < 4; ++j) {
            const float4 w = wpk[(b * 4 + j) * Epad + e];
            ss = fmaf(w.x, w.x, ss);
            ss = fmaf(w.y, w.y, ss);
            ss = fmaf(w.z, w.z, ss);
            ss = fmaf(w.w, w.w, ss);
        }
        out[i] = ss;
    }
    // norms per 64-wide block: out64[c][e] = sqrt(sum of the four 16-blocks)
    const int64_t total64 = (Dpad / 64) * Epad;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total64;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t c = i / Epad, e = i % Epad;
        float ss = 0.0f;
        for (int j = 0; j < 16; ++j) {
            const float4 w = wpk[(c * 16 + j) * Epad + e];
            ss = fmaf(w.x, w.x, ss);
            ss = fmaf(w.y, w.y, ss);
            ss = fmaf(w.z, w.z, ss);
            ss = fmaf(w.w, w.w, ss);
        }
        out64[i] = sqrtf(ss);
    }
}

// [Dpad/4][Epad][4] -> [Epad/eb][Dpad/4][eb][4]
__global__ void block_gate_kernel(const float4* __restrict__ wt, int64_t D4, int64_t Epad, int eb,
                                  float4* __restrict__ out) {
    const int64_t total = D4 * Epad;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t el = i % eb;
        const int64_t d4 = (i / eb) % D4;
        const int64_t b = i / (eb * D4);
        out[i] = wt[d4 * Epad + b * eb + el];
    }
}

template <int GROUP, int NSLOT, int TPG, typename XT, bool EXACT, int WARPS = kWarps, int DKO = 0,
          bool CERT = false>
cudaError_t launch_one(const Gate& g, const void* x, int64_t N, int k, int ksel, int32_t* idx,
                       float* val, cudaStream_t s, const int* rowlist = nullptr,
                       unsigned long long* rows_total = nullptr) {
    using C = GatingCfg<GROUP, NSLOT, TPG, WARPS, XT, DKO>;
    const int64_t blocks = (N + C::TOK - 1) / C::TOK;
    auto kern = gating_kernel<GROUP, NSLOT, TPG, WARPS, XT, EXACT, DKO, CERT>;
    const size_t smem = C::SMEM + (CERT ? 4 * C::TOK : 0);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(
            kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    kern<<<static_cast<unsigned>(blocks), WARPS * 32, smem, s>>>(
        static_cast<const XT*>(x), reinterpret_cast<const float4*>(g.wt), g.bias, N,
        static_cast<int>(g.D), static_cast<int>(g.E), k, ksel, idx, val, g.wsq16, g.cert_rows,
        rowlist, rows_total, 1.0f, -0.0f);
    return cudaGetLastError();
}

template <typename XT, bool EXACT, bool CERT = false>
cudaError_t dispatch_e(const Gate& g, const void* x, int64_t N, int k, int ksel, int32_t* idx,
                       float* val, cudaStream_t s) {
    // Few tokens through a narrow gate: few CTAs, each walking all of D, so
    // the time is the number of chunk rounds; 256-wide chunks (a 2-8 KB
    // weight stage) take a quarter of the rounds (154 -> 65 us at D=4096,
    // E=8).  Wider gates keep 64-wide chunks: a 64 KB stage lands slower
    // than the barriers it saves (78 -> 94 us at E=64).
    if (N <= 1024) {
        switch (g.Epad) {
            case 8: return launch_one<8, 1, 2, XT, EXACT, 4, 256, CERT>(g, x, N, k, ksel, idx, val, s);
            case 16: return launch_one<16, 1, 2, XT, EXACT, 4, 256, CERT>(g, x, N, k, ksel, idx, val, s);
            default: break;
        }
    }
    // Many tokens: 8 tokens per lane group halves the weight loads per
    // multiply-add; fewer: 4, for more CTAs.
    if (N >= 12288) {
        // 7 warps: 56 tokens per CTA, so 16384 tokens make 293 CTAs -- two
        // per SM on all 148 SMs instead of two on 108 and one on 40
        switch (g.Epad) {
            case 8: return launch_one<8, 1, 8, XT, EXACT, 7, 0, CERT>(g, x, N, k, ksel, idx, val, s);
            case 16: return launch_one<16, 1, 8, XT, EXACT, 7, 0, CERT>(g, x, N, k, ksel, idx, val, s);
            case 32: return launch_one<32, 1, 8, XT, EXACT, 7, 0, CERT>(g, x, N, k, ksel, idx, val, s);
            case 64: return launch_one<32, 2, 8, XT, EXACT, 7, 0, CERT>(g, x, N, k, ksel, idx, val, s);
            default: break;
        }
    }
    if (N <= 4096) {
        // Few tokens: 2 tokens per lane group and 4 warps per CTA, so that
        // even T = 2048 spreads over 256 CTAs; the weights' chunks then come
        // from L2 once per 8 tokens.
        switch (g.Epad) {
            case 32: return launch_one<32, 1, 2, XT, EXACT, 4, 0, CERT>(g, x, N, k, ksel, idx, val, s);
            case 64: return launch_one<32, 2, 2, XT, EXACT, 4, 0, CERT>(g, x, N, k, ksel, idx, val, s);
            case 128: return launch_one<32, 4, 2, XT, EXACT, 4, 0, CERT>(g, x, N, k, ksel, idx, val, s);
            case 256: return launch_one<32, 8, 2, XT, EXACT, 4, 0, CERT>(g, x, N, k, ksel, idx, val, s);
            default: break;
        }
    }
    switch (g.Epad) {
        case 8: return launch_one<8, 1, 4, XT, EXACT, kWarps, 0, CERT>(g, x, N, k, ksel, idx, val, s);
        case 16: return launch_one<16, 1, 4, XT, EXACT, kWarps, 0, CERT>(g, x, N, k, ksel, idx, val, s);
        case 32: return launch_one<32, 1, 4, XT, EXACT, kWarps, 0, CERT>(g, x, N, k, ksel, idx, val, s);
        case 64: return launch_one<32, 2, 4, XT, EXACT, kWarps, 0, CERT>(g, x, N, k, ksel, idx, val, s);
        case 128: return launch_one<32, 4, 4, XT, EXACT, kWarps, 0, CERT>(g, x, N, k, ksel, idx, val, s);
        default: return launch_one<32, 8, 4, XT, EXACT, kWarps, 0, CERT>(g, x, N, k, ksel, idx, val, s);
    }
}

// Packs W [D, E] (device, row-major) into [Dpad/4][Epad][4].
__global__ void pack_gate_kernel(const float* __restrict__ w, const float* __restrict__ b, int64_t D,
                                 int64_t E, int64_t Dpad, int64_t Epad, float* __restrict__ out,
                                 float* __restrict__ bout) {
    const int64_t total = Dpad * Epad;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t c = i & 3;
        const int64_t e = (i >> 2) % Epad;
        const int64_t d4 = (i >> 2) / Epad;
        const int64_t d = d4 * 4 + c;
        out[i] = (d < D && e < E) ? w[d * E + e] : 0.0f;
    }
    for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < Epad;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x)
        bout[e] = (e < E && b) ? b[e] : 0.0f;
}

template <int EPAD, typename XT>
cudaError_t launch_cert_e(const Gate& g, const void* x, int64_t N, int k, int ksel, int32_t* idx,
                          float* val, bool small, cudaStream_t s) {
    if (small) {
        const size_t smem = cert_small_smem(g.Dpad, EPAD);
        auto kern = gating_cert_small_kernel<EPAD, XT>;
        // the largest shared-memory size this instantiation was opened to, per device
        static size_t opened[64] = {};
        if (g.device < 0 || g.device >= 64 || opened[g.device] < smem) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem));
            if (e != cudaSuccess) return e;
            if (g.device >= 0 && g.device < 64) opened[g.device] = smem;
        }
        kern<<<static_cast<unsigned>((N + kCertTT - 1) / kCertTT), kCertThreads, smem, s>>>(
            static_cast<const XT*>(x), reinterpret_cast<const float4*>(g.wt), g.bias, g.wn64, N,
            static_cast<int>(g.D), g.Dpad, static_cast<int>(g.E), k, ksel, idx, val, g.cert_rows);
    } else {
        const cudaError_t e = dispatch_e<XT, false, true>(g, x, N, k, ksel, idx, val, s);
        if (e != cudaSuccess) return e;
    }
    const cudaError_t e1 = cudaGetLastError();
    if (e1 != cudaSuccess) return e1;
    // The rows the first pass could not certify, with the EXACT arithmetic:
    // the EXACT kernel in a few-tokens-per-CTA form over the row list, so
    // the (few) deferred rows spread over many CTAs.
    constexpr int GR = EPAD < 32 ? EPAD : 32;
    return launch_one<GR, EPAD / GR, 2, XT, true, 4, 0, false>(g, x, N, k, ksel, idx, val, s,
                                                              g.cert_rows, g.cert_total);
}

template <typename XT>
cudaError_t launch_cert(const Gate& g, const void* x, int64_t N, int k, int ksel, int32_t* idx,
                        float* val, bool small, cudaStream_t s) {
    switch (g.Epad) {
        case 8: return launch_cert_e<8, XT>(g, x, N, k, ksel, idx, val, small, s);
        case 16: return launch_cert_e<16, XT>(g, x, N, k, ksel, idx, val, small, s);
        case 32: return launch_cert_e<32, XT>(g, x, N, k, ksel, idx, val, small, s);
        case 64: return launch_cert_e<64, XT>(g, x, N, k, ksel, idx, val, small, s);
        case 128: return launch_cert_e<128, XT>(g, x, N, k, ksel, idx, val, small, s);
        default: return launch_cert_e<256, XT>(g, x, N, k, ksel, idx, val, small, s);
    }
}

}  // namespace

int gate_small_eb(int64_t Epad) { return Epad / 8 > 8 ? static_cast<int>(Epad / 8) : 8; }

// Up to this many tokens the small-batch kernel runs (measured crossover).
constexpr int64_t kSmallBatchMax = 512;
// Certified mode: the d-split kernel up to this many tokens and this much
// shared memory (activation rows of 4 tokens: d up to about 12K).
constexpr int64_t kCertSmallMax = 512;
constexpr int64_t kCertSmallSmemMax = 200 * 1024;

int gate_epad(int64_t E) {
    if (E <= 8) return 8;
    if (E <= 16) return 16;
    if (E <= 32) return 32;
    if (E <= 64) return 64;
    if (E <= 128) return 128;
    return 256;
}

aem_status launch_gating(const Gate& g, const void* x, aem_dtype xd, int64_t N, int k, int ksel,
                         aem_gating_mode mode, int32_t* idx, float* val, cudaStream_t s) {
    if (N == 0) return AEM_OK;
    cudaError_t e;
    if (mode == AEM_GATING_CERTIFIED) {
        // the uncertified-row list: room for every row, emptied per call
        if (g.cert_cap < N) {
            if (g.cert_rows) {
                cudaDeviceSynchronize();
                cudaFree(g.cert_rows);
                g.cert_rows = nullptr;
                g.cert_cap = 0;
            }
            AEM_TRY_CUDA(cudaMalloc(&g.cert_rows, sizeof(int) * (N + 1)));
            g.cert_cap = N;
        }
        AEM_TRY_CUDA(cudaMemsetAsync(g.cert_rows, 0, sizeof(int), s));
        // few tokens: d split over threads (activation rows in shared memory)
        const bool small = N <= kCertSmallMax && cert_small_smem(g.Dpad, static_cast<int>(g.Epad)) <=
                                                     static_cast<size_t>(kCertSmallSmemMax);
        e = xd == AEM_F32 ? launch_cert<float>(g, x, N, k, ksel, idx, val, small, s)
                          : launch_cert<__nv_bfloat16>(g, x, N, k, ksel, idx, val, small, s);
        if (e != cudaSuccess) {
            set_error("certified gating launch failed: %s", cudaGetErrorString(e));
            return AEM_ECUDA;
        }
        count_launches(2);
        return AEM_OK;
    }
    const bool exact = mode == AEM_GATING_EXACT;
    const int xbytes = xd == AEM_F32 ? 4 : 2;
    // the small-batch kernel copies whole 16-byte pieces of activation rows
    const bool small = N <= kSmallBatchMax && g.wblk != nullptr &&
                       (g.D * xbytes) % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    if (small) {
        int* err = device_error_word(g.device);
        if (!err) {
            set_error("gating: no device error word");
            return AEM_ENOMEM;
        }
        if (xd == AEM_F32)
            e = exact ? launch_small<float, true>(g, x, N, k, ksel, idx, val, err, s)
                      : launch_small<float, false>(g, x, N, k, ksel, idx, val, err, s);
        else
            e = exact ? launch_small<__nv_bfloat16, true>(g, x, N, k, ksel, idx, val, err, s)
                      : launch_small<__nv_bfloat16, false>(g, x, N, k, ksel, idx, val, err, s);
    } else if (xd == AEM_F32)
        e = exact ? dispatch_e<float, true>(g, x, N, k, ksel, idx, val, s)
                  : dispatch_e<float, false>(g, x, N, k, ksel, idx, val, s);
    else
        e = exact ? dispatch_e<__nv_bfloat16, true>(g, x, N, k, ksel, idx, val, s)
                  : dispatch_e<__nv_bfloat16, false>(g, x, N, k, ksel, idx, val, s);
    if (e != cudaSuccess) {
        set_error("gating kernel launch failed: %s", cudaGetErrorString(e));
        return AEM_ECUDA;
    }
    count_launches(1);
    return AEM_OK;
}

}  // namespace aem

using aem::set_error;

namespace {
aem_status check_gating_args(const aem::Gate* g, const void* x, aem_dtype xd, int64_t N, int k,
                             int k_extra, const void* idx, const void* val) {
    AEM_REQUIRE(g != nullptr, "gating: gate handle is NULL");
    AEM_REQUIRE(xd == AEM_F32 || xd == AEM_BF16, "gating: hidden dtype must be F32 or BF16");
    AEM_REQUIRE(N >= 0, "gating: N=%lld must be >= 0", (long long)N);
    AEM_REQUIRE(k >= 1, "gating: k=%d must be >= 1", k);
    AEM_REQUIRE(k <= AEM_MAX_TOPK && k <= g->E,
                "k=%d invalid for num_experts=%lld (MAX_TOPK=%d)", k, (long long)g->E,
                AEM_MAX_TOPK);
    AEM_REQUIRE(k_extra == 0 || k_extra == 1, "gating: k_extra=%d must be 0 or 1", k_extra);
    AEM_REQUIRE(k + k_extra <= g->E,
                "gating: k + k_extra = %d exceeds num_experts=%lld", k + k_extra, (long long)g->E);
    AEM_REQUIRE(N == 0 || (x && idx && val), "gating: NULL buffer");
    return AEM_OK;
}
}  // namespace

extern "C" {

aem_status aem_gate_pack(const float* gate_weight, const float* gate_bias, int64_t D, int64_t E,
                         int device, aem_gate_t* out) {
    AEM_REQUIRE(out != nullptr, "aem_gate_pack: out is NULL");
    *out = nullptr;
    AEM_REQUIRE(gate_weight != nullptr, "aem_gate_pack: gate_weight is NULL");
    AEM_REQUIRE(D >= 1 && E >= 1, "aem_gate_pack: D=%lld E=%lld must be >= 1", (long long)D,
                (long long)E);
    AEM_REQUIRE(E <= AEM_MAX_EXPERTS,
                "num_experts=%lld exceeds this kernel's MAX_EXPERTS=%d", (long long)E,
                AEM_MAX_EXPERTS);
    AEM_REQUIRE(D <= (1ll << 30), "aem_gate_pack: D too large");
    if (!aem::is_sm100(device)) {
        set_error("aem_gate_pack: device %d is not an sm_100 (B200) GPU", device);
        return AEM_EUNSUPPORTED;
    }
    AEM_TRY_CUDA(cudaSetDevice(device));
    auto* g = new aem::Gate();
    g->device = device;
    g->D = D;
    g->E = E;
    g->Epad = aem::gate_epad(E);
    g->Dpad = (D + 255) / 256 * 256;  // a whole number of the widest chunk (256)
    float* tmp_w = nullptr;
    float* tmp_b = nullptr;
    aem_status st = AEM_OK;
    do {
        if (cudaMalloc(&g->wt, sizeof(float) * g->Dpad * g->Epad) != cudaSuccess ||
            cudaMalloc(&g->bias, sizeof(float) * g->Epad) != cudaSuccess ||
            cudaMalloc(&tmp_w, sizeof(float) * D * E) != cudaSuccess ||
            cudaMalloc(&tmp_b, sizeof(float) * E) != cudaSuccess) {
            set_error("aem_gate_pack: device allocation failed");
            st = AEM_ENOMEM;
            break;
        }
        if (cudaMemcpy(tmp_w, gate_weight, sizeof(float) * D * E, cudaMemcpyHostToDevice) !=
                cudaSuccess ||
            (gate_bias && cudaMemcpy(tmp_b, gate_bias, sizeof(float) * E,
                                     cudaMemcpyHostToDevice) != cudaSuccess)) {
            set_error("aem_gate_pack: copy failed");
            st = AEM_ECUDA;
            break;
        }
        aem::pack_gate_kernel<<<256, 256>>>(tmp_w, gate_bias ? tmp_b : nullptr, D, E, g->Dpad,
                                             g->Epad, g->wt, g->bias);
        g->eb = aem::gate_small_eb(g->Epad);
        if (cudaMalloc(&g->wblk, sizeof(float) * g->Dpad * g->Epad) != cudaSuccess) {
            set_error("aem_gate_pack: device allocation failed");
            st = AEM_ENOMEM;
            break;
        }
        aem::block_gate_kernel<<<256, 256>>>(reinterpret_cast<const float4*>(g->wt), g->Dpad / 4,
                                              g->Epad, g->eb, reinterpret_cast<float4*>(g->wblk));
        if (cudaMalloc(&g->wsq16, sizeof(float) * (g->Dpad / 16) * g->Epad) != cudaSuccess ||
            cudaMalloc(&g->wn64, sizeof(float) * (g->Dpad / 64) * g->Epad) != cudaSuccess ||
            cudaMalloc(&g->cert_total, sizeof(unsigned long long)) != cudaSuccess ||
            cudaMemset(g->cert_total, 0, sizeof(unsigned long long)) != cudaSuccess) {
            set_error("aem_gate_pack: device allocation failed");
            st = AEM_ENOMEM;
            break;
        }
        aem::gate_norms_kernel<<<256, 256>>>(reinterpret_cast<const float4*>(g->wt), g->Dpad,
                                              g->Epad, g->wsq16, g->wn64);
        if (cudaDeviceSynchronize() != cudaSuccess) {
            set_error("aem_gate_pack: pack kernel failed: %s",
                      cudaGetErrorString(cudaGetLastError()));
            st = AEM_ECUDA;
            break;
        }
    } while (0);
    cudaFree(tmp_w);
    cudaFree(tmp_b);
    if (st != AEM_OK) {
        cudaFree(g->wt);
        cudaFree(g->bias);
        cudaFree(g->wblk);
        cudaFree(g->wsq16);
        cudaFree(g->wn64);
        cudaFree(g->cert_total);
        delete g;
        return st;
    }
    *out = reinterpret_cast<aem_gate_t>(g);
    return AEM_OK;
}

aem_status aem_gate_free(aem_gate_t gate) {
    if (!gate) return AEM_OK;
    auto* g = reinterpret_cast<aem::Gate*>(gate);
    cudaSetDevice(g->device);
    cudaFree(g->wt);
    cudaFree(g->bias);
    cudaFree(g->wblk);
    cudaFree(g->wsq16);
    cudaFree(g->wn64);
    cudaFree(g->cert_rows);
    cudaFree(g->cert_total);
    delete g;
    return AEM_OK;
}

aem_status aem_gate_fallback_rows(aem_gate_t gate, int64_t* rows) {
    AEM_REQUIRE(gate != nullptr && rows != nullptr, "aem_gate_fallback_rows: NULL argument");
    auto* g = reinterpret_cast<aem::Gate*>(gate);
    AEM_TRY_CUDA(cudaSetDevice(g->device));
    AEM_TRY_CUDA(cudaDeviceSynchronize());
    unsigned long long v = 0;
    AEM_TRY_CUDA(cudaMemcpy(&v, g->cert_total, sizeof(v), cudaMemcpyDeviceToHost));
    *rows = static_cast<int64_t>(v);
    return AEM_OK;
}

aem_status aem_gating(aem_gate_t gate, const void* hidden, aem_dtype hidden_dtype, int64_t N,
                      int k, int k_extra, aem_gating_mode mode, int32_t* out_idx, float* out_val,
                      void* stream) {
    auto* g = reinterpret_cast<aem::Gate*>(gate);
    AEM_TRY(check_gating_args(g, hidden, hidden_dtype, N, k, k_extra, out_idx, out_val));
    return aem::launch_gating(*g, hidden, hidden_dtype, N, k, k + k_extra, mode, out_idx, out_val,
                              static_cast<cudaStream_t>(stream));
}

aem_status aem_gating_host(aem_context_t ctx, aem_gate_t gate, const void* hidden,
                           aem_dtype hidden_dtype, int64_t N, int k, int k_extra,
                           aem_gating_mode mode, int32_t* out_idx, float* out_val) {
    AEM_REQUIRE(ctx != nullptr, "aem_gating_host: context is NULL");
    auto* c = reinterpret_cast<aem::Context*>(ctx);
    auto* g = reinterpret_cast<aem::Gate*>(gate);
    AEM_TRY(check_gating_args(g, hidden, hidden_dtype, N, k, k_extra, out_idx, out_val));
    if (N == 0) return AEM_OK;
    AEM_TRY_CUDA(cudaSetDevice(c->device));
    const int ksel = k + k_extra;
    const size_t xb = static_cast<size_t>(N) * g->D * (hidden_dtype == AEM_F32 ? 4 : 2);
    const size_t ib = static_cast<size_t>(N) * ksel * 4;
    const size_t vb = static_cast<size_t>(N) * k * 4;
    const size_t o1 = aem::align_up(xb, 256), o2 = o1 + aem::align_up(ib, 256);
    AEM_TRY(c->reserve_device(o2 + vb));
    char* d = static_cast<char*>(c->dev);
    AEM_TRY_CUDA(cudaMemcpyAsync(d, hidden, xb, cudaMemcpyHostToDevice, c->stream));
    AEM_TRY(aem::launch_gating(*g, d, hidden_dtype, N, k, ksel, mode,
                               reinterpret_cast<int32_t*>(d + o1), reinterpret_cast<float*>(d + o2),
                               c->stream));
    AEM_TRY_CUDA(cudaMemcpyAsync(out_idx, d + o1, ib, cudaMemcpyDeviceToHost, c->stream));
    AEM_TRY_CUDA(cudaMemcpyAsync(out_val, d + o2, vb, cudaMemcpyDeviceToHost, c->stream));
    AEM_TRY_CUDA(cudaStreamSynchronize(c->stream));
    return AEM_OK;
}

}  // extern "C"
