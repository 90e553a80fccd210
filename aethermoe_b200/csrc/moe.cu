// Single-GPU MoE layer and the INT8 GEMM entry points.
//
// The reference never composes its pieces (gating, capacity routing, expert
// GEMM).  This layer composes them the way a Mixtral-style MoE block runs:
//   1. fused gating            -> idx [T, k(+1)], val [T, k]
//   2. capacity routing         -> effective expert per (token, slot) unit,
//                                  slot-major batch_position u = j*T + t
//   3. expert-grouped layout    -> rows grouped by effective expert
//   4. gather                   -> X [U, d] in grouped order: bf16, or for
//                                  float32 x the bf16 pair hi + lo (x = hi + lo
//                                  to about 16 significant bits)
//   5. grouped up GEMM + ReLU   -> H [U, ffn]: bf16, or the bf16 pair hi + lo
//   6. grouped down GEMM + combine -> out[t] += val[t, j] * y  (float32 red.add
//                                  from the GEMM epilogue; bf16 output converted after)
// A split operand costs a second MMA per K step (hi and lo against the same
// exact bf16 copy of the int8 weights), so float32 callers get the
// float32-activation contract of fused_quantized_matmul
// (src/kernels/quantized_gemm.py:184-226) at the price of twice the MMAs.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "moe.h"
#include "route.h"
#include "runtime.h"

namespace aem {

namespace {

// X[dest] = bf16(x[src[dest]]) (and, for float32 x with lo != nullptr,
// lo[dest] = bf16(x - X[dest])): one warp per row, 16-byte vectors when aligned.
template <typename XT>
__global__ void gather_rows_kernel(const XT* __restrict__ x, const int32_t* __restrict__ src,
                                   int64_t rows, int64_t d, __nv_bfloat16* __restrict__ out,
                                   __nv_bfloat16* __restrict__ lo, float4* __restrict__ z1,
                                   int64_t n1, float4* __restrict__ z2, int64_t n2) {
    // zeroing of the step's accumulation buffers rides along (n1, n2 float4s)
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n1 + n2;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        if (i < n1)
            z1[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        else
            z2[i - n1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const int lane = threadIdx.x & 31;
    for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
         r < rows; r += warps) {
        const int64_t s = src[r];
        const XT* in = x + s * d;
        __nv_bfloat16* o = out + r * d;
        if constexpr (sizeof(XT) == 2) {
            if ((d & 7) == 0) {
                const uint4* vi = reinterpret_cast<const uint4*>(in);
                uint4* vo = reinterpret_cast<uint4*>(o);
                for (int64_t i = lane; i < d / 8; i += 32) vo[i] = vi[i];
            } else {
                for (int64_t i = lane; i < d; i += 32) o[i] = in[i];
            }
        } else {
            __nv_bfloat16* ol = lo ? lo + r * d : nullptr;
            if ((d & 3) == 0) {
                const float4* vi = reinterpret_cast<const float4*>(in);
                uint2* vo = reinterpret_cast<uint2*>(o);
                for (int64_t i = lane; i < d / 4; i += 32) {
                    const float4 f = vi[i];
                    __nv_bfloat162 a = __floats2bfloat162_rn(f.x, f.y);
                    __nv_bfloat162 b = __floats2bfloat162_rn(f.z, f.w);
                    uint2 u;
                    u.x = *reinterpret_cast<uint32_t*>(&a);
                    u.y = *reinterpret_cast<uint32_t*>(&b);
                    vo[i] = u;
                    if (ol) {
                        const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
                        __nv_bfloat162 la = __floats2bfloat162_rn(f.x - fa.x, f.y - fa.y);
                        __nv_bfloat162 lb = __floats2bfloat162_rn(f.z - fb.x, f.w - fb.y);
                        u.x = *reinterpret_cast<uint32_t*>(&la);
                        u.y = *reinterpret_cast<uint32_t*>(&lb);
                        reinterpret_cast<uint2*>(ol)[i] = u;
                    }
                }
            } else {
                for (int64_t i = lane; i < d; i += 32) {
                    const __nv_bfloat16 h = __float2bfloat16_rn(in[i]);
                    o[i] = h;
                    if (ol) ol[i] = __float2bfloat16_rn(in[i] - __bfloat162float(h));
                }
            }
        }
    }
}

// out[t] = sum_{j<k} y[t*k + j] (float32, j in increasing order).
template <typename OT>
__global__ void combine_kernel(const float* __restrict__ y, int64_t T, int k, int64_t d,
                               OT* __restrict__ out) {
    const int64_t total = T * d;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / d, c = i % d;
        const float* yr = y + t * k * d + c;
        float acc = 0.0f;
        for (int j = 0; j < k; ++j) acc += yr[static_cast<int64_t>(j) * d];
        if constexpr (sizeof(OT) == 2)
            out[i] = __float2bfloat16_rn(acc);
        else
            out[i] = acc;
    }
}

// Vectorised combine when d % 4 == 0.
template <typename OT>
__global__ void combine4_kernel(const float4* __restrict__ y, int64_t T, int k, int64_t d4,
                                OT* __restrict__ out) {
    const int64_t total = T * d4;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / d4, c = i % d4;
        const float4* yr = y + t * k * d4 + c;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < k; ++j) {
            const float4 v = yr[static_cast<int64_t>(j) * d4];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        if constexpr (sizeof(OT) == 2) {
            __nv_bfloat162 a = __floats2bfloat162_rn(acc.x, acc.y);
            __nv_bfloat162 b = __floats2bfloat162_rn(acc.z, acc.w);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t*>(&a);
            u.y = *reinterpret_cast<uint32_t*>(&b);
            reinterpret_cast<uint2*>(out)[i] = u;
        } else {
            reinterpret_cast<float4*>(out)[i] = acc;
        }
    }
}

// k == 1 with bf16 output (the layer's float32 output rows -> bf16): a
// straight conversion, 8 values per thread and iteration, no row arithmetic.
__global__ void f32_to_bf16_kernel(const float4* __restrict__ y, int64_t n8,
                                   uint4* __restrict__ out) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 a = y[2 * i];
        const float4 b = y[2 * i + 1];
        __nv_bfloat162 h[4] = {__floats2bfloat162_rn(a.x, a.y), __floats2bfloat162_rn(a.z, a.w),
                               __floats2bfloat162_rn(b.x, b.y), __floats2bfloat162_rn(b.z, b.w)};
        out[i] = *reinterpret_cast<const uint4*>(h);
    }
}

unsigned grid_for(int64_t work, int per_block) {
    const int64_t b = (work + per_block - 1) / per_block;
    return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(b, 148 * 16)));
}

}  // namespace

aem_status gather_rows(const void* x, aem_dtype xd, const int32_t* src, int64_t rows, int64_t d,
                       void* out, cudaStream_t s, void* out_lo, float* zero1, int64_t zero1_n,
                       float* zero2, int64_t zero2_n) {
    if (rows == 0 && zero1_n == 0 && zero2_n == 0) return AEM_OK;
    AEM_REQUIRE(zero1_n % 4 == 0 && zero2_n % 4 == 0 &&
                    (reinterpret_cast<uintptr_t>(zero1) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(zero2) & 15) == 0,
                "gather_rows: zeroed ranges must be whole, aligned float4s");
    const int64_t z4 = (zero1_n + zero2_n) / 4;
    const unsigned g = std::max(grid_for(rows, 8), grid_for(z4, 256 * 4));
    if (xd == AEM_BF16)
        gather_rows_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(x), src, rows, d, static_cast<__nv_bfloat16*>(out),
            nullptr, reinterpret_cast<float4*>(zero1), zero1_n / 4,
            reinterpret_cast<float4*>(zero2), zero2_n / 4);
    else
        gather_rows_kernel<float><<<g, 256, 0, s>>>(
            static_cast<const float*>(x), src, rows, d, static_cast<__nv_bfloat16*>(out),
            static_cast<__nv_bfloat16*>(out_lo), reinterpret_cast<float4*>(zero1), zero1_n / 4,
            reinterpret_cast<float4*>(zero2), zero2_n / 4);
    AEM_CHECK_LAUNCH();
    count_launches(1);
    return AEM_OK;
}

aem_status combine_rows(const float* y, int64_t T, int k, int64_t d, void* out, aem_dtype od,
                        cudaStream_t s) {
    if (T == 0) return AEM_OK;
    if (k == 1 && od == AEM_BF16 && (T * d) % 8 == 0 &&
        ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
        f32_to_bf16_kernel<<<grid_for(T * d / 8, 256), 256, 0, s>>>(
            reinterpret_cast<const float4*>(y), T * d / 8, static_cast<uint4*>(out));
    } else if ((d & 3) == 0) {
        const unsigned g = grid_for(T * d / 4, 256);
        if (od == AEM_BF16)
            combine4_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(
                reinterpret_cast<const float4*>(y), T, k, d / 4, static_cast<__nv_bfloat16*>(out));
        else
            combine4_kernel<float><<<g, 256, 0, s>>>(reinterpret_cast<const float4*>(y), T, k,
                                                     d / 4, static_cast<float*>(out));
    } else {
        const unsigned g = grid_for(T * d, 256);
        if (od == AEM_BF16)
            combine_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(y, T, k, d,
                                                            static_cast<__nv_bfloat16*>(out));
        else
            combine_kernel<float><<<g, 256, 0, s>>>(y, T, k, d, static_cast<float*>(out));
    }
    AEM_CHECK_LAUNCH();
    count_launches(1);
    return AEM_OK;
}

// ------------------------------------------------------------------ Moe
aem_status Moe::reserve_split(int64_t T) {
    if (T <= split_cap && split_buf) return AEM_OK;
    if (split_buf) {
        cudaDeviceSynchronize();
        cudaFree(split_buf);
        split_buf = nullptr;
        split_cap = 0;
    }
    const int64_t U = T * cfg.top_k;
    const size_t ox = align_up(2 * static_cast<size_t>(U) * cfg.d_model, 256);
    AEM_TRY_CUDA(cudaMalloc(&split_buf, ox + 2 * static_cast<size_t>(U) * cfg.d_ffn));
    xperm_lo = split_buf;
    h_lo = static_cast<char*>(split_buf) + ox;
    split_cap = T;
    return AEM_OK;
}

aem_status Moe::reserve(int64_t T, bool expert_buffers) {
    if (T <= T_cap && buf) return AEM_OK;
    if (buf) {
        cudaDeviceSynchronize();
        cudaFree(buf);
        buf = nullptr;
    }
    const int64_t U = T * cfg.top_k;
    const int ksel = cfg.top_k < cfg.num_experts ? cfg.top_k + 1 : cfg.top_k;
    const int64_t d = cfg.d_model, f = cfg.d_ffn;
    size_t off = 0;
    auto slot = [&](size_t bytes) {
        const size_t o = off;
        off += align_up(bytes, 256);
        return o;
    };
    const size_t o_idx = slot(sizeof(int32_t) * T * ksel);
    const size_t o_val = slot(sizeof(float) * T * cfg.top_k);
    const size_t o_ws = slot(moe_route_workspace(T, cfg.top_k, cfg.num_experts));
    const size_t o_eff = slot(sizeof(uint32_t) * U);
    const size_t o_starts = slot(sizeof(int) * (cfg.num_experts + 1));
    const size_t o_src = slot(sizeof(int32_t) * U);
    const size_t o_map = slot(sizeof(int32_t) * U);
    const size_t o_rs = slot(sizeof(float) * U);
    const int64_t Ux = expert_buffers ? U : 0;
    const size_t o_x = slot(2 * Ux * d);
    const size_t o_h = slot(2 * Ux * f);
    const size_t o_y = slot(sizeof(float) * Ux * d);
    AEM_TRY_CUDA(cudaMalloc(&buf, off));
    char* b = static_cast<char*>(buf);
    idx = reinterpret_cast<int32_t*>(b + o_idx);
    val = reinterpret_cast<float*>(b + o_val);
    route_ws = b + o_ws;
    eff = reinterpret_cast<uint32_t*>(b + o_eff);
    starts = reinterpret_cast<int*>(b + o_starts);
    src_token = reinterpret_cast<int32_t*>(b + o_src);
    rowmap = reinterpret_cast<int32_t*>(b + o_map);
    rowscale = reinterpret_cast<float*>(b + o_rs);
    xperm = expert_buffers ? b + o_x : nullptr;
    h = expert_buffers ? b + o_h : nullptr;
    y = expert_buffers ? reinterpret_cast<float*>(b + o_y) : nullptr;
    T_cap = T;
    return AEM_OK;
}

aem_status Moe::forward(const void* x, aem_dtype xd, int64_t T, void* out, aem_dtype od,
                        cudaStream_t s) {
    last_T = T;
    if (T == 0) return AEM_OK;
    AEM_TRY(reserve(T));
    StepTimer timer(AEM_METRIC_MOE_STEP, s);
    const int k = cfg.top_k, E = cfg.num_experts;
    const int ksel = k < E ? k + 1 : k;
    const int64_t U = T * k, d = cfg.d_model, f = cfg.d_ffn;
    prof.begin(AEM_PHASE_GATING, s);
    AEM_TRY(launch_gating(*gate, x, xd, T, k, ksel, cfg.gating_mode, idx, val, s));
    prof.end(AEM_PHASE_GATING, s);
    prof.begin(AEM_PHASE_ROUTE, s);
    MoeRouteArgs ra;
    ra.idx = idx;
    ra.T = T;
    ra.ldi = ksel;
    ra.k = k;
    ra.E = E;
    ra.capacity = cfg.capacity;
    ra.val = val;
    ra.workspace = route_ws;
    ra.eff_out = eff;
    ra.starts_out = starts;
    ra.src_token = src_token;
    ra.rowmap = rowmap;
    ra.rowscale = rowscale;
    AEM_TRY(route_moe(ra, s));
    // operand precision: float32 x enters the up GEMM as a bf16 pair; the
    // hidden activation is a pair when hidden_dtype says so (by default when x
    // is float32)
    const bool split_x = xd == AEM_F32;
    const bool split_h = hidden_dtype < 0 ? split_x : hidden_dtype == AEM_F32;
    if (split_x || split_h) AEM_TRY(reserve_split(T));
    // the step's accumulation buffers (float32 output rows; at decode sizes
    // the up projection's pre-activations) are zeroed by the gather's launch
    const bool decode = U <= gemv_max_rows();
    if (decode && !h32) AEM_TRY_CUDA(cudaMalloc(&h32, sizeof(float) * gemv_max_rows() * f));
    float* acc = od == AEM_F32 ? static_cast<float*>(out) : y;
    const bool z_acc = (T * d) % 4 == 0 && (reinterpret_cast<uintptr_t>(acc) & 15) == 0;
    const bool z_h = decode && (U * f) % 4 == 0;
    AEM_TRY(gather_rows(x, xd, src_token, U, d, xperm, s, split_x ? xperm_lo : nullptr,
                        z_h ? h32 : nullptr, z_h ? U * f : 0, z_acc ? acc : nullptr,
                        z_acc ? T * d : 0));
    prof.end(AEM_PHASE_ROUTE, s);
    AEM_TRY(expert_ffn(T, U, out, od, s, split_x, split_h, z_acc, z_h));
    prof.step();
    return AEM_OK;
}

aem_status Moe::expert_ffn(int64_t T, int64_t U, void* out, aem_dtype od, cudaStream_t s,
                           bool split_x, bool split_h, bool acc_zeroed, bool h32_zeroed) {
    const int k = cfg.top_k, E = cfg.num_experts;
    const int64_t d = cfg.d_model, f = cfg.d_ffn;
    // Decode steps (few units): the up projection splits K over the SMs, which
    // its ReLU / bf16 epilogue would forbid, by summing float32 partial
    // products into h32; the down projection's weight-stream kernel applies
    // ReLU and the bf16 rounding (pair) of H as it stages those rows.
    const bool decode = U <= gemv_max_rows();
    if (decode && !h32) AEM_TRY_CUDA(cudaMalloc(&h32, sizeof(float) * gemv_max_rows() * f));
    GemmArgs up_a;
    up_a.w = up;
    up_a.group_base = 0;
    up_a.G = up->G < E ? static_cast<int>(up->G) : E;
    up_a.group_rows = starts;
    up_a.M = U;
    up_a.max_rows = U;
    up_a.x_hi = xperm;
    up_a.x_lo = split_x ? xperm_lo : nullptr;
    up_a.out = h;
    up_a.out_lo = split_h ? h_lo : nullptr;
    up_a.out_bf16 = true;
    up_a.ldo = f;
    up_a.relu = true;
    if (decode) {
        up_a.out = h32;
        up_a.out_lo = nullptr;
        up_a.out_bf16 = false;
        up_a.relu = false;
        up_a.atomic_add = true;
    }
    prof.begin(AEM_PHASE_UP, s);
    if (decode && !h32_zeroed) AEM_TRY_CUDA(cudaMemsetAsync(h32, 0, sizeof(float) * U * f, s));
    AEM_TRY(launch_qgemm(up_a, s));
    prof.end(AEM_PHASE_UP, s);

    // Down projection with the combine fused into its epilogue: every grouped
    // row's output, scaled by its gate weight, is red.add-ed into its token's
    // float32 output row (k contributions per token, from different tiles).
    float* acc = od == AEM_F32 ? static_cast<float*>(out) : y;
    GemmArgs dn;
    dn.w = down;
    dn.G = up_a.G;
    dn.group_rows = starts;
    dn.M = U;
    dn.max_rows = U;
    dn.x_hi = h;
    dn.x_lo = split_h ? h_lo : nullptr;
    dn.out = acc;
    dn.ldo = d;
    dn.rowmap = src_token;
    dn.rowscale = rowscale;
    dn.atomic_add = true;
    if (decode) {
        dn.x_hi = nullptr;
        dn.x_lo = nullptr;
        dn.x_f32_relu = h32;
        dn.x_f32_lo = split_h;
    }
    // Few tiles per SM (decode sizes): stream-K, every SM streams the same
    // number of weight tiles (the output rows start at zero and take red.add).
    const int64_t groups_used = std::min<int64_t>(E, U);
    const int64_t nch = (d + 127) / 128;
    const int64_t tiles = std::max<int64_t>(1, groups_used) * nch *
                          ((U / std::max<int64_t>(1, groups_used) + 255) / 256);
    const int sms = sm_count(gate->device);
    dn.stream_k = tiles < 8 * static_cast<int64_t>(sms);
    prof.begin(AEM_PHASE_DOWN, s);
    if (!acc_zeroed) AEM_TRY_CUDA(cudaMemsetAsync(acc, 0, sizeof(float) * T * d, s));
    AEM_TRY(launch_qgemm(dn, s));
    prof.end(AEM_PHASE_DOWN, s);
    if (od != AEM_F32) {
        prof.begin(AEM_PHASE_COMBINE, s);
        AEM_TRY(combine_rows(acc, T, 1, d, out, od, s));  // float32 -> bf16
        prof.end(AEM_PHASE_COMBINE, s);
    }
    (void)k;
    return AEM_OK;
}

}  // namespace aem

using aem::set_error;

extern "C" {

aem_status aem_moe_create(const aem_moe_config* cfg, aem_gate_t gate, aem_qweight_t up,
                          aem_qweight_t down, aem_moe_t* out) {
    AEM_REQUIRE(out != nullptr, "aem_moe_create: out is NULL");
    *out = nullptr;
    AEM_REQUIRE(cfg && gate && up && down, "aem_moe_create: NULL argument");
    auto* g = reinterpret_cast<aem::Gate*>(gate);
    auto* u = reinterpret_cast<aem::QWeight*>(up);
    auto* dn = reinterpret_cast<aem::QWeight*>(down);
    AEM_REQUIRE(cfg->top_k >= 1 && cfg->top_k <= AEM_MAX_TOPK && cfg->top_k <= cfg->num_experts,
                "aem_moe_create: top_k=%d invalid for num_experts=%d", cfg->top_k,
                cfg->num_experts);
    AEM_REQUIRE(g->E == cfg->num_experts && g->D == cfg->d_model,
                "aem_moe_create: gate is [%lld, %lld], config wants [%lld, %d]", (long long)g->D,
                (long long)g->E, (long long)cfg->d_model, cfg->num_experts);
    AEM_REQUIRE(u->G == cfg->num_experts && u->K == cfg->d_model && u->N == cfg->d_ffn,
                "aem_moe_create: up weight shape mismatch");
    AEM_REQUIRE(dn->G == cfg->num_experts && dn->K == cfg->d_ffn && dn->N == cfg->d_model,
                "aem_moe_create: down weight shape mismatch");
    AEM_REQUIRE(cfg->gating_mode == AEM_GATING_EXACT || cfg->gating_mode == AEM_GATING_FAST ||
                    cfg->gating_mode == AEM_GATING_CERTIFIED,
                "aem_moe_create: bad gating mode");
    auto* m = new aem::Moe();
    m->cfg = *cfg;
    m->gate = g;
    m->up = u;
    m->down = dn;
    *out = reinterpret_cast<aem_moe_t>(m);
    return AEM_OK;
}

aem_status aem_moe_free(aem_moe_t moe) {
    if (!moe) return AEM_OK;
    auto* m = reinterpret_cast<aem::Moe*>(moe);
    cudaSetDevice(m->gate->device);
    cudaDeviceSynchronize();
    cudaFree(m->buf);
    cudaFree(m->split_buf);
    cudaFree(m->h32);
    aem::seam_free(m);
    delete m;
    return AEM_OK;
}

aem_status aem_moe_forward(aem_moe_t moe, const void* x, aem_dtype x_dtype, int64_t T, void* out,
                           aem_dtype out_dtype, void* stream) {
    AEM_REQUIRE(moe != nullptr, "aem_moe_forward: NULL layer");
    AEM_REQUIRE(T >= 0 && T < (1ll << 28), "aem_moe_forward: T=%lld out of range", (long long)T);
    AEM_REQUIRE(T == 0 || (x && out), "aem_moe_forward: NULL buffer");
    AEM_REQUIRE(x_dtype == AEM_F32 || x_dtype == AEM_BF16, "aem_moe_forward: bad x dtype");
    AEM_REQUIRE(out_dtype == AEM_F32 || out_dtype == AEM_BF16, "aem_moe_forward: bad out dtype");
    auto* m = reinterpret_cast<aem::Moe*>(moe);
    return m->forward(x, x_dtype, T, out, out_dtype, static_cast<cudaStream_t>(stream));
}

aem_status aem_moe_forward_host(aem_context_t ctx, aem_moe_t moe, const void* x, aem_dtype x_dtype,
                                int64_t T, void* out, aem_dtype out_dtype) {
    AEM_REQUIRE(ctx != nullptr && moe != nullptr, "aem_moe_forward_host: NULL argument");
    auto* c = reinterpret_cast<aem::Context*>(ctx);
    auto* m = reinterpret_cast<aem::Moe*>(moe);
    AEM_REQUIRE(T >= 0 && T < (1ll << 28), "aem_moe_forward_host: T out of range");
    if (T == 0) return AEM_OK;
    AEM_REQUIRE(x && out, "aem_moe_forward_host: NULL buffer");
    AEM_TRY_CUDA(cudaSetDevice(c->device));
    const size_t xb = static_cast<size_t>(T) * m->cfg.d_model * (x_dtype == AEM_F32 ? 4 : 2);
    const size_t ob = static_cast<size_t>(T) * m->cfg.d_model * (out_dtype == AEM_F32 ? 4 : 2);
    const size_t o1 = aem::align_up(xb, 256);
    AEM_TRY(c->reserve_device(o1 + ob));
    char* d = static_cast<char*>(c->dev);
    AEM_TRY_CUDA(cudaMemcpyAsync(d, x, xb, cudaMemcpyHostToDevice, c->stream));
    AEM_TRY(m->forward(d, x_dtype, T, d + o1, out_dtype, c->stream));
    AEM_TRY_CUDA(cudaMemcpyAsync(out, d + o1, ob, cudaMemcpyDeviceToHost, c->stream));
    return aem::check_device_errors(c->stream, "aem_moe_forward_host");
}

aem_status aem_moe_set_hidden_dtype(aem_moe_t moe, int hidden_dtype) {
    AEM_REQUIRE(moe != nullptr, "aem_moe_set_hidden_dtype: NULL layer");
    AEM_REQUIRE(hidden_dtype == -1 || hidden_dtype == AEM_F32 || hidden_dtype == AEM_BF16,
                "aem_moe_set_hidden_dtype: %d is not -1, AEM_F32 or AEM_BF16", hidden_dtype);
    reinterpret_cast<aem::Moe*>(moe)->hidden_dtype = hidden_dtype;
    return AEM_OK;
}

aem_status aem_moe_profile(aem_moe_t moe, int enable) {
    AEM_REQUIRE(moe != nullptr, "aem_moe_profile: NULL layer");
    reinterpret_cast<aem::Moe*>(moe)->prof.enable(enable != 0);
    return AEM_OK;
}

aem_status aem_moe_profile_read(aem_moe_t moe, double* ms, int64_t* steps) {
    AEM_REQUIRE(moe != nullptr, "aem_moe_profile_read: NULL layer");
    return reinterpret_cast<aem::Moe*>(moe)->prof.read(ms, steps);
}

aem_status aem_moe_last_routing(aem_moe_t moe, int32_t* idx, float* val, uint32_t* effective,
                                void* stream) {
    AEM_REQUIRE(moe != nullptr, "aem_moe_last_routing: NULL layer");
    auto* m = reinterpret_cast<aem::Moe*>(moe);
    auto s = static_cast<cudaStream_t>(stream);
    const int64_t T = m->last_T;
    if (T == 0) return AEM_OK;
    const int k = m->cfg.top_k;
    const int ksel = k < m->cfg.num_experts ? k + 1 : k;
    if (idx)
        AEM_TRY_CUDA(cudaMemcpyAsync(idx, m->idx, sizeof(int32_t) * T * ksel,
                                     cudaMemcpyDeviceToDevice, s));
    if (val)
        AEM_TRY_CUDA(cudaMemcpyAsync(val, m->val, sizeof(float) * T * k, cudaMemcpyDeviceToDevice, s));
    if (effective)
        AEM_TRY_CUDA(cudaMemcpyAsync(effective, m->eff, sizeof(uint32_t) * T * k,
                                     cudaMemcpyDeviceToDevice, s));
    return AEM_OK;
}

// ------------------------------------------------------------------ INT8 GEMM entry points
aem_status aem_qgemm(aem_qweight_t wh, int64_t group, const void* x, aem_dtype x_dtype, int64_t M,
                     float* out, void* stream) {
    AEM_REQUIRE(wh != nullptr, "aem_qgemm: weight handle is NULL");
    auto* w = reinterpret_cast<aem::QWeight*>(wh);
    AEM_REQUIRE(group >= 0 && group < w->G, "aem_qgemm: group %lld out of range [0, %lld)",
                (long long)group, (long long)w->G);
    AEM_REQUIRE(M >= 0, "aem_qgemm: M must be >= 0");
    AEM_REQUIRE(x_dtype == AEM_F32 || x_dtype == AEM_BF16, "aem_qgemm: bad x dtype");
    if (M == 0) return AEM_OK;
    AEM_REQUIRE(x && out, "aem_qgemm: NULL buffer");
    auto s = static_cast<cudaStream_t>(stream);
    // float32 activations become a bf16 hi + lo pair in a stream-ordered
    // buffer; bf16 activations are used in place.
    const size_t half = aem::align_up(static_cast<size_t>(M) * w->K * 2, 256);
    void* tmp = nullptr;
    const void* hi = x;
    const void* lo = nullptr;
    aem_status st = AEM_OK;
    if (x_dtype == AEM_F32) {
        AEM_TRY_CUDA(cudaMallocAsync(&tmp, 2 * half, s));
        hi = tmp;
        lo = static_cast<char*>(tmp) + half;
        st = aem::launch_split_bf16(x, x_dtype, M * w->K, tmp, static_cast<char*>(tmp) + half, s);
    }
    if (st == AEM_OK) {
        aem::GemmArgs a;
        a.w = w;
        a.group_base = group;
        a.G = 1;
        a.M = M;
        a.x_hi = hi;
        a.x_lo = lo;
        a.out = out;
        a.ldo = w->N;
        // Tensor-core sizes with few tiles per SM: stream-K -- every SM
        // streams the same number of weight tiles (whole tiles leave some SMs
        // a tile more than others), partial sums added into the zeroed
        // output.  With many tiles per SM the imbalance is small and the
        // zeroing and read-modify-write of a large output cost more
        // (measured: M=512 99 us with, 118 without; M=4096 478 with, 430 without).
        const int sms = aem::sm_count(aem::current_device());
        const int64_t tiles = (w->N + 127) / 128 * ((M + 127) / 128);
        if (M > 4 && w->K % 8 == 0 && tiles < 8 * static_cast<int64_t>(sms)) {
            if (cudaMemsetAsync(out, 0, sizeof(float) * M * w->N, s) != cudaSuccess) {
                set_error("aem_qgemm: memset failed");
                st = AEM_ECUDA;
            }
            a.atomic_add = true;
            a.stream_k = true;
        }
        if (st == AEM_OK) st = aem::launch_qgemm(a, s);
    }
    if (tmp) cudaFreeAsync(tmp, s);
    return st;
}

aem_status aem_qgemm_host(aem_context_t ctx, aem_qweight_t wh, int64_t group, const void* x,
                          aem_dtype x_dtype, int64_t M, float* out) {
    AEM_REQUIRE(ctx != nullptr && wh != nullptr, "aem_qgemm_host: NULL argument");
    auto* c = reinterpret_cast<aem::Context*>(ctx);
    auto* w = reinterpret_cast<aem::QWeight*>(wh);
    AEM_REQUIRE(M >= 0, "aem_qgemm_host: M must be >= 0");
    if (M == 0) return AEM_OK;
    AEM_REQUIRE(x && out, "aem_qgemm_host: NULL buffer");
    AEM_TRY_CUDA(cudaSetDevice(c->device));
    const size_t xb = static_cast<size_t>(M) * w->K * (x_dtype == AEM_F32 ? 4 : 2);
    const size_t ob = sizeof(float) * M * w->N;
    const size_t o1 = aem::align_up(xb, 256);
    AEM_TRY(c->reserve_device(o1 + ob));
    char* d = static_cast<char*>(c->dev);
    AEM_TRY_CUDA(cudaMemcpyAsync(d, x, xb, cudaMemcpyHostToDevice, c->stream));
    AEM_TRY(aem_qgemm(wh, group, d, x_dtype, M, reinterpret_cast<float*>(d + o1), c->stream));
    AEM_TRY_CUDA(cudaMemcpyAsync(out, d + o1, ob, cudaMemcpyDeviceToHost, c->stream));
    return aem::check_device_errors(c->stream, "aem_qgemm_host");
}

}  // extern "C"

extern "C" aem_status aem_grouped_qgemm(aem_qweight_t wh, const int32_t* group_rows, int G,
                                        const void* x, int64_t M, void* out, aem_dtype out_dtype,
                                        int64_t ldo, int relu, int accumulate,
                                        const int32_t* rowmap, const float* rowscale,
                                        int token_tile, int ksplit, void* stream) {
    AEM_REQUIRE(wh != nullptr, "aem_grouped_qgemm: weight handle is NULL");
    auto* w = reinterpret_cast<aem::QWeight*>(wh);
    AEM_REQUIRE(G >= 1 && G <= 256 && G <= w->G, "aem_grouped_qgemm: G=%d outside [1, min(256, %lld)]",
                G, (long long)w->G);
    AEM_REQUIRE(M >= 0 && ldo >= w->N, "aem_grouped_qgemm: bad M or ldo");
    AEM_REQUIRE(out_dtype == AEM_F32 || out_dtype == AEM_BF16, "aem_grouped_qgemm: bad out dtype");
    AEM_REQUIRE(!accumulate || out_dtype == AEM_F32, "aem_grouped_qgemm: accumulate needs float32 out");
    AEM_REQUIRE(ksplit <= 1 || accumulate, "aem_grouped_qgemm: ksplit > 1 needs accumulate");
    AEM_REQUIRE(token_tile == 0 || token_tile == 16 || token_tile == 32 || token_tile == 64 ||
                    token_tile == 128 || token_tile == 256,
                "aem_grouped_qgemm: token_tile=%d not in {0,16,32,64,128,256}", token_tile);
    AEM_REQUIRE(!(relu && accumulate), "aem_grouped_qgemm: ReLU of a partial sum is undefined");
    if (M == 0) return AEM_OK;
    AEM_REQUIRE(group_rows && x && out, "aem_grouped_qgemm: NULL buffer");
    aem::GemmArgs a;
    a.w = w;
    a.G = G;
    a.group_rows = group_rows;
    a.M = M;
    a.max_rows = M;
    a.x_hi = x;
    a.out = out;
    a.out_bf16 = out_dtype == AEM_BF16;
    a.ldo = ldo;
    a.relu = relu != 0;
    a.atomic_add = accumulate != 0;
    a.ksplit = ksplit < 1 ? 1 : ksplit;
    a.rowmap = rowmap;
    a.rowscale = rowscale;
    a.token_tile = token_tile;
    return aem::launch_qgemm(a, static_cast<cudaStream_t>(stream));
}
