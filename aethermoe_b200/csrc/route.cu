// Capacity-ceiling routing on the GPU -- Router::assign_effective_experts
// (src/orchestration/router.hpp:249-266): within each primary-expert group,
// ranked by batch_position, the first `capacity` units keep their primary and
// the rest take their own secondary (one hop, router.hpp:21-27).
//
// The rank of a unit inside its expert group is a stable counting sort over
// units in batch_position order:
//   count   -- per chunk of kChunk consecutive positions, a histogram over experts
//   scan    -- per expert, exclusive prefix over chunks (+ expert totals/starts)
//   assign  -- per chunk, stable local ranks from warp match masks + a
//              cross-warp prefix in shared memory; rank = chunk offset + local
// All integer; bit-exact with the reference by construction.  The same three
// kernels, keyed by the effective expert, produce the MoE permutation that
// groups units by expert for the grouped GEMM.
#include <algorithm>

#include "common.cuh"
#include "route.h"
#include "runtime.h"

namespace aem {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
// Positions per thread of the chunk kernels: the stand-alone capacity rule
// uses 2048-position chunks (its scratch sizes are part of the ABI), the MoE
// routing 512-position ones (4x the CTAs for the same batch).
constexpr int kPerThreadApi = 8;
constexpr int kPerThreadMoe = 2;
constexpr int kChunk = kThreads * kPerThreadApi;
constexpr int kChunkMoe = kThreads * kPerThreadMoe;
constexpr int kScanThreads = 1024;

// MoE units, slot-major: u = j*T + t, primary = idx[t][j], secondary = idx[t][k]
// (the (k+1)-th choice; the primary when the gating produced only k).
__global__ void build_units_kernel(const int32_t* __restrict__ idx, int64_t T, int ldi, int k,
                                   int E, uint32_t* __restrict__ prim, uint32_t* __restrict__ sec,
                                   int* err) {
    const int64_t n = T * k;
    for (int64_t u = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; u < n;
         u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t j = u / T, t = u % T;
        const int32_t p = idx[t * ldi + j];
        const int32_t s = ldi > k ? idx[t * ldi + k] : p;
        if (p < 0 || p >= E || s < 0 || s >= E) atomicOr(err, ERR_ROUTE_EXPERT);
        prim[u] = static_cast<uint32_t>(p);
        sec[u] = static_cast<uint32_t>(s);
    }
}

// inv[pos[i]] = i with a permutation check; then gathers primary/secondary
// into position order.
__global__ void invert_positions_kernel(const uint32_t* __restrict__ pos, int64_t n,
                                        int32_t* __restrict__ inv, int32_t* __restrict__ seen,
                                        int* err) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint32_t p = pos[i];
        if (p >= n) {
            atomicOr(err, ERR_ROUTE_POSITION);
            continue;
        }
        if (atomicExch(&seen[p], 1) != 0) {
            atomicOr(err, ERR_ROUTE_POSITION);
            continue;
        }
        inv[p] = static_cast<int32_t>(i);
    }
}

__global__ void gather_by_position_kernel(const uint32_t* __restrict__ primary,
                                          const uint32_t* __restrict__ secondary,
                                          const int32_t* __restrict__ inv, int64_t n, int E,
                                          uint32_t* __restrict__ prim_s,
                                          uint32_t* __restrict__ sec_s, int* err) {
    for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < n;
         p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int32_t i = inv[p];
        if (i < 0 || i >= n) {  // only after a failed permutation check
            prim_s[p] = 0;
            sec_s[p] = 0;
            continue;
        }
        const uint32_t a = primary[i], b = secondary[i];
        if (a >= static_cast<uint32_t>(E) || b >= static_cast<uint32_t>(E)) {
            atomicOr(err, ERR_ROUTE_EXPERT);
            prim_s[p] = 0;
            sec_s[p] = 0;
            continue;
        }
        prim_s[p] = a;
        sec_s[p] = b;
    }
}

// Histogram of keys per chunk: cnt[c][e].
// Enumeration of the n = k*T units for grouping: identity when half_T == 0;
// otherwise every unit of the first half_T tokens (slot-major among them)
// comes first, then those of the other tokens, so each expert's group lists
// the first half's units first.  Units are u = j*T + t.
__device__ __forceinline__ int64_t unit_at(int64_t p, int64_t T, int64_t half_T, int k) {
    if (half_T <= 0 || half_T >= T) return p;
    const int64_t n_a = static_cast<int64_t>(k) * half_T;
    if (p < n_a) return (p / half_T) * T + p % half_T;
    const int64_t q = p - n_a, tb = T - half_T;
    return (q / tb) * T + half_T + q % tb;
}

template <int PT>
__global__ void __launch_bounds__(kThreads)
    chunk_count_kernel(const uint32_t* __restrict__ key, int64_t n, int E, int* __restrict__ cnt,
                       int64_t T = 0, int64_t half_T = 0, int k = 1) {
    constexpr int CH = kThreads * PT;
    __shared__ int h[AEM_MAX_EXPERTS];
    for (int e = threadIdx.x; e < E; e += kThreads) h[e] = 0;
    __syncthreads();
    const int64_t base = static_cast<int64_t>(blockIdx.x) * CH;
    for (int i = threadIdx.x; i < CH; i += kThreads) {
        const int64_t p = base + i;
        if (p < n) {
            const uint32_t e = key[unit_at(p, T, half_T, k)];
            if (e < static_cast<uint32_t>(E)) atomicAdd(&h[e], 1);
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += kThreads) cnt[static_cast<int64_t>(blockIdx.x) * E + e] = h[e];
}

// In place: cnt[c][e] -> exclusive prefix over c, and starts[0..E]
// (exclusive prefix of the expert totals over e) when starts is given.  One
// CTA: thread (group g, expert e) takes a contiguous range of chunks, so a
// warp's loads are consecutive experts of one chunk (coalesced) and each
// thread's loads are independent (batched); pass 1 sums the group's range,
// a prefix over the groups runs in shared memory, pass 2 writes the range's
// exclusive prefixes.
__global__ void __launch_bounds__(kScanThreads)
    chunk_scan_kernel(int* __restrict__ cnt, int nchunks, int E, int* __restrict__ starts) {
    __shared__ int gsum[kScanThreads];  // [group][expert]
    __shared__ int tot[AEM_MAX_EXPERTS];
    const int ng = kScanThreads / E;    // groups of chunks (E <= 256: at least 4)
    const int tid = threadIdx.x;
    const int g = tid / E, e = tid % E;
    const bool act = g < ng;
    const int per = (nchunks + ng - 1) / ng;
    const int c0 = g * per, c1 = min(nchunks, c0 + per);
    int sum = 0;
    if (act) {
#pragma unroll 8
        for (int c = c0; c < c1; ++c) sum += cnt[static_cast<int64_t>(c) * E + e];
        gsum[g * E + e] = sum;
    }
    __syncthreads();
    if (tid < E) {
        int run = 0;
        for (int q = 0; q < ng; ++q) {
            const int v = gsum[q * E + tid];
            gsum[q * E + tid] = run;
            run += v;
        }
        tot[tid] = run;
    }
    __syncthreads();
    if (act) {
        int run = gsum[g * E + e];
        for (int c = c0; c < c1; ++c) {
            const int64_t i = static_cast<int64_t>(c) * E + e;
            const int v = cnt[i];
            cnt[i] = run;
            run += v;
        }
    }
    if (starts && tid == 0) {
        int run = 0;
        for (int x = 0; x < E; ++x) {
            starts[x] = run;
            run += tot[x];
        }
        starts[E] = run;
    }
}

template <int PT, typename Emit>
__device__ __forceinline__ void chunk_ranks(const uint32_t* __restrict__ key, int64_t n, int E,
                                            const int* __restrict__ off, Emit emit,
                                            int64_t T = 0, int64_t half_T = 0, int k = 1) {
    constexpr int CH = kThreads * PT;
    __shared__ int run[AEM_MAX_EXPERTS];
    __shared__ int hw[kWarps][AEM_MAX_EXPERTS];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const unsigned lt = (1u << lane) - 1u;
    for (int e = tid; e < E; e += kThreads) run[e] = off[static_cast<int64_t>(blockIdx.x) * E + e];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * CH;
    for (int r = 0; r < PT; ++r) {
        for (int i = tid; i < kWarps * E; i += kThreads) hw[i / E][i % E] = 0;
        __syncthreads();
        const int64_t p = base + static_cast<int64_t>(r) * kThreads + tid;
        const bool valid = p < n;
        const int64_t u = valid ? unit_at(p, T, half_T, k) : 0;
        uint32_t e = valid ? key[u] : 0xFFFFFFFFu;
        if (e >= static_cast<uint32_t>(E)) e = 0xFFFFFFFFu;
        const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
        const int in_warp = __popc(peers & lt);
        if (e != 0xFFFFFFFFu && in_warp == 0) hw[warp][e] = __popc(peers);
        __syncthreads();
        for (int x = tid; x < E; x += kThreads) {
            int acc = run[x];
            for (int w = 0; w < kWarps; ++w) {
                const int v = hw[w][x];
                hw[w][x] = acc;
                acc += v;
            }
            run[x] = acc;
        }
        __syncthreads();
        if (e != 0xFFFFFFFFu) emit(u, e, hw[warp][e] + in_warp);
        __syncthreads();
    }
}

// Pass 1: effective expert of every position.  EP: rank += corr[slot][key]
// with slot = p / slot_len (corr == nullptr for a single GPU).
template <int PT>
__global__ void __launch_bounds__(kThreads)
    assign_kernel(const uint32_t* __restrict__ prim, const uint32_t* __restrict__ sec, int64_t n,
                  int E, const int* __restrict__ off, uint64_t capacity,
                  const int64_t* __restrict__ corr, int64_t slot_len,
                  const int32_t* __restrict__ out_index, uint32_t* __restrict__ eff) {
    chunk_ranks<PT>(prim, n, E, off, [&](int64_t p, uint32_t e, int rank) {
        int64_t rk = rank;
        if (corr) rk += corr[(p / slot_len) * E + e];
        const uint32_t v = static_cast<uint64_t>(rk) < capacity ? e : sec[p];
        const int64_t o = out_index ? out_index[p] : p;
        if (o >= 0) eff[o] = v;  // o < 0 only after a failed permutation check
    });
}

// Pass 2 (MoE permutation): unit u goes to row starts[e] + rank of the
// expert-grouped layout; records the token it came from, the output row of
// its expert result (t*k + j) and its gate weight.
template <int PT>
__global__ void __launch_bounds__(kThreads)
    scatter_kernel(const uint32_t* __restrict__ eff, int64_t n, int E, const int* __restrict__ off,
                   const int* __restrict__ starts, int64_t T, int k,
                   const float* __restrict__ val, int32_t* __restrict__ src_token,
                   int32_t* __restrict__ rowmap, float* __restrict__ rowscale,
                   int32_t* __restrict__ dest_of, int64_t half_T) {
    chunk_ranks<PT>(eff, n, E, off, [&](int64_t u, uint32_t e, int rank) {
        const int64_t dest = starts[e] + rank;
        const int64_t j = u / T, t = u % T;
        src_token[dest] = static_cast<int32_t>(t);
        rowmap[dest] = static_cast<int32_t>(t * k + j);
        rowscale[dest] = val[t * k + j];
        if (dest_of) dest_of[u] = static_cast<int32_t>(dest);
    }, T, half_T, k);
}

// Few units (decode steps, single GPU): the whole MoE routing in one CTA --
// units, capacity ranks, effective experts, expert starts and the grouped
// permutation -- with the same stable counting sorts as the kernels above
// (ranks over units in unit order, rounds of kFusedThreads units, warp match
// masks and a cross-warp prefix), so every output is identical; one launch
// instead of seven.
constexpr int kFusedThreads = 512;
constexpr int kFusedWarps = kFusedThreads / 32;
constexpr int64_t kFusedMaxUnits = 2048;

__global__ void __launch_bounds__(kFusedThreads)
    route_fused_kernel(const int32_t* __restrict__ idx, int64_t T, int ldi, int k, int E,
                       uint64_t capacity, const float* __restrict__ val,
                       uint32_t* __restrict__ eff_out, int* __restrict__ starts_out,
                       int32_t* __restrict__ src_token, int32_t* __restrict__ rowmap,
                       float* __restrict__ rowscale, int32_t* __restrict__ dest_of, int* err) {
    __shared__ uint32_t s_prim[kFusedMaxUnits], s_sec[kFusedMaxUnits], s_eff[kFusedMaxUnits];
    __shared__ int run[AEM_MAX_EXPERTS];
    __shared__ int hw[kFusedWarps][AEM_MAX_EXPERTS];
    __shared__ int st[AEM_MAX_EXPERTS + 1];
    const int n = static_cast<int>(T * k);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const unsigned lt = (1u << lane) - 1u;
    for (int u = tid; u < n; u += kFusedThreads) {
        const int64_t j = u / T, t = u % T;
        const int32_t p = idx[t * ldi + j];
        const int32_t q = ldi > k ? idx[t * ldi + k] : p;
        if (p < 0 || p >= E || q < 0 || q >= E) atomicOr(err, ERR_ROUTE_EXPERT);
        s_prim[u] = static_cast<uint32_t>(p);
        s_sec[u] = static_cast<uint32_t>(q);
        s_eff[u] = 0xFFFFFFFFu;  // stays so for a unit with an invalid primary
    }
    for (int e = tid; e < E; e += kFusedThreads) run[e] = 0;
    __syncthreads();
    // stable ranks of keys[u] over u in order, handed to emit(u, e, rank)
    auto ranks = [&](const uint32_t* keys, auto emit) {
        for (int r0 = 0; r0 < n; r0 += kFusedThreads) {
            for (int i = tid; i < kFusedWarps * E; i += kFusedThreads) hw[i / E][i % E] = 0;
            __syncthreads();
            const int u = r0 + tid;
            uint32_t e = u < n ? keys[u] : 0xFFFFFFFFu;
            if (e >= static_cast<uint32_t>(E)) e = 0xFFFFFFFFu;
            const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
            const int in_warp = __popc(peers & lt);
            if (e != 0xFFFFFFFFu && in_warp == 0) hw[warp][e] = __popc(peers);
            __syncthreads();
            for (int x = tid; x < E; x += kFusedThreads) {
                int acc = run[x];
                for (int w = 0; w < kFusedWarps; ++w) {
                    const int v = hw[w][x];
                    hw[w][x] = acc;
                    acc += v;
                }
                run[x] = acc;
            }
            __syncthreads();
            if (e != 0xFFFFFFFFu) emit(u, e, hw[warp][e] + in_warp);
            __syncthreads();
        }
    };
    // pass 1: the capacity rule over primaries
    ranks(s_prim, [&](int u, uint32_t e, int rank) {
        s_eff[u] = static_cast<uint64_t>(rank) < capacity ? e : s_sec[u];
    });
    // expert totals of the effective experts -> starts
    for (int e = tid; e < E; e += kFusedThreads) run[e] = 0;
    __syncthreads();
    for (int u = tid; u < n; u += kFusedThreads)
        if (s_eff[u] < static_cast<uint32_t>(E)) atomicAdd(&run[s_eff[u]], 1);
    __syncthreads();
    if (tid == 0) {
        int acc = 0;
        for (int e = 0; e < E; ++e) {
            st[e] = acc;
            acc += run[e];
        }
        st[E] = acc;
    }
    __syncthreads();
    for (int e = tid; e <= E; e += kFusedThreads) starts_out[e] = st[e];
    for (int e = tid; e < E; e += kFusedThreads) run[e] = 0;
    for (int u = tid; u < n; u += kFusedThreads)
        if (eff_out) eff_out[u] = s_eff[u];
    __syncthreads();
    // pass 2: the expert-grouped permutation
    ranks(s_eff, [&](int u, uint32_t e, int rank) {
        const int dest = st[e] + rank;
        const int64_t j = u / T, t = u % T;
        src_token[dest] = static_cast<int32_t>(t);
        rowmap[dest] = static_cast<int32_t>(t * k + j);
        rowscale[dest] = val[t * k + j];
        if (dest_of) dest_of[u] = dest;
    });
}

}  // namespace

int64_t route_chunks(int64_t n) { return (n + kChunk - 1) / kChunk; }
static int64_t route_chunks_moe(int64_t n) { return (n + kChunkMoe - 1) / kChunkMoe; }

size_t moe_route_workspace(int64_t T, int k, int E) {
    const int64_t n = T * k;
    const int64_t c = route_chunks_moe(n) > 0 ? route_chunks_moe(n) : 1;
    size_t b = 0;
    b += align_up(sizeof(uint32_t) * n, 256) * 3;      // prim, sec, eff
    b += align_up(sizeof(int) * c * E, 256) * 2;        // cnt1, cnt2
    b += align_up(sizeof(int) * (E + 1), 256);          // starts
    return b;
}

aem_status route_moe(const MoeRouteArgs& a, cudaStream_t s) {
    const int64_t n = a.T * a.k;
    if (n == 0) return AEM_OK;
    if (n <= kFusedMaxUnits && a.corr == nullptr && a.half_T == 0 && a.starts_out) {
        int* err = device_error_word(current_device());
        AEM_REQUIRE(err != nullptr, "route: no device error word");
        route_fused_kernel<<<1, kFusedThreads, 0, s>>>(a.idx, a.T, a.ldi, a.k, a.E, a.capacity,
                                                       a.val, a.eff_out, a.starts_out, a.src_token,
                                                       a.rowmap, a.rowscale, a.dest_of, err);
        AEM_CHECK_LAUNCH();
        count_launches(1);
        return AEM_OK;
    }
    const int64_t c = route_chunks_moe(n);
    char* w = static_cast<char*>(a.workspace);
    auto take = [&](size_t bytes) {
        char* p = w;
        w += align_up(bytes, 256);
        return p;
    };
    uint32_t* prim = reinterpret_cast<uint32_t*>(take(sizeof(uint32_t) * n));
    uint32_t* sec = reinterpret_cast<uint32_t*>(take(sizeof(uint32_t) * n));
    uint32_t* eff = a.eff_out ? a.eff_out : reinterpret_cast<uint32_t*>(take(sizeof(uint32_t) * n));
    if (a.eff_out) take(sizeof(uint32_t) * n);
    int* cnt1 = reinterpret_cast<int*>(take(sizeof(int) * c * a.E));
    int* cnt2 = reinterpret_cast<int*>(take(sizeof(int) * c * a.E));
    int* starts = a.starts_out;
    int* err = device_error_word(current_device());
    AEM_REQUIRE(err != nullptr, "route: no device error word");
    const unsigned gb = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 4096));
    build_units_kernel<<<gb, 256, 0, s>>>(a.idx, a.T, a.ldi, a.k, a.E, prim, sec, err);
    AEM_CHECK_LAUNCH();
    chunk_count_kernel<kPerThreadMoe><<<static_cast<unsigned>(c), kThreads, 0, s>>>(prim, n, a.E,
                                                                                 cnt1);
    AEM_CHECK_LAUNCH();
    chunk_scan_kernel<<<1, kScanThreads, 0, s>>>(cnt1, static_cast<int>(c), a.E, nullptr);
    AEM_CHECK_LAUNCH();
    assign_kernel<kPerThreadMoe><<<static_cast<unsigned>(c), kThreads, 0, s>>>(
        prim, sec, n, a.E, cnt1, a.capacity, a.corr, a.T, nullptr, eff);
    AEM_CHECK_LAUNCH();
    chunk_count_kernel<kPerThreadMoe><<<static_cast<unsigned>(c), kThreads, 0, s>>>(
        eff, n, a.E, cnt2, a.T, a.half_T, a.k);
    AEM_CHECK_LAUNCH();
    chunk_scan_kernel<<<1, kScanThreads, 0, s>>>(cnt2, static_cast<int>(c), a.E, starts);
    AEM_CHECK_LAUNCH();
    scatter_kernel<kPerThreadMoe><<<static_cast<unsigned>(c), kThreads, 0, s>>>(
        eff, n, a.E, cnt2, starts, a.T, a.k, a.val, a.src_token, a.rowmap, a.rowscale, a.dest_of,
        a.half_T);
    AEM_CHECK_LAUNCH();
    count_launches(7);
    return AEM_OK;
}

}  // namespace aem

using aem::set_error;

extern "C" {

size_t aem_capacity_route_workspace(int64_t n, int E) {
    if (n < 0 || E < 1) return 0;
    const int64_t c = aem::route_chunks(n) > 0 ? aem::route_chunks(n) : 1;
    size_t b = 0;
    b += aem::align_up(sizeof(int32_t) * n, 256) * 2;   // inv, seen
    b += aem::align_up(sizeof(uint32_t) * n, 256) * 2;  // prim_s, sec_s
    b += aem::align_up(sizeof(int) * c * E, 256);       // chunk counts
    return b;
}

aem_status aem_capacity_route(const uint32_t* primary, const uint32_t* secondary,
                              const uint32_t* batch_position, int64_t n, int E, uint64_t capacity,
                              uint32_t* effective, void* workspace, size_t workspace_bytes,
                              void* stream) {
    AEM_REQUIRE(n >= 0, "aem_capacity_route: n=%lld must be >= 0", (long long)n);
    AEM_REQUIRE(E >= 1 && E <= AEM_MAX_EXPERTS, "aem_capacity_route: E=%d outside [1, %d]", E,
                AEM_MAX_EXPERTS);
    AEM_REQUIRE(n < (1ll << 31), "aem_capacity_route: n too large");
    if (n == 0) return AEM_OK;
    AEM_REQUIRE(primary && secondary && batch_position && effective,
                "aem_capacity_route: NULL buffer");
    auto s = static_cast<cudaStream_t>(stream);
    const size_t need = aem_capacity_route_workspace(n, E);
    bool owned = false;
    if (!workspace) {
        AEM_TRY_CUDA(cudaMallocAsync(&workspace, need, s));
        owned = true;
    } else {
        AEM_REQUIRE(workspace_bytes >= need, "aem_capacity_route: workspace %zu < %zu bytes",
                    workspace_bytes, need);
    }
    char* w = static_cast<char*>(workspace);
    int32_t* inv = reinterpret_cast<int32_t*>(w);
    w += aem::align_up(sizeof(int32_t) * n, 256);
    int32_t* seen = reinterpret_cast<int32_t*>(w);
    w += aem::align_up(sizeof(int32_t) * n, 256);
    uint32_t* prim_s = reinterpret_cast<uint32_t*>(w);
    w += aem::align_up(sizeof(uint32_t) * n, 256);
    uint32_t* sec_s = reinterpret_cast<uint32_t*>(w);
    w += aem::align_up(sizeof(uint32_t) * n, 256);
    int* cnt = reinterpret_cast<int*>(w);
    const int64_t c = aem::route_chunks(n);
    int* err = aem::device_error_word(aem::current_device());
    AEM_REQUIRE(err != nullptr, "aem_capacity_route: no device error word");
    aem_status st = AEM_OK;
    do {
        if (cudaMemsetAsync(seen, 0, sizeof(int32_t) * n, s) != cudaSuccess ||
            cudaMemsetAsync(inv, 0xFF, sizeof(int32_t) * n, s) != cudaSuccess) {
            set_error("aem_capacity_route: memset failed");
            st = AEM_ECUDA;
            break;
        }
        const unsigned gb = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 4096));
        aem::invert_positions_kernel<<<gb, 256, 0, s>>>(batch_position, n, inv, seen, err);
        aem::gather_by_position_kernel<<<gb, 256, 0, s>>>(primary, secondary, inv, n, E, prim_s,
                                                          sec_s, err);
        aem::chunk_count_kernel<aem::kPerThreadApi><<<static_cast<unsigned>(c), aem::kThreads, 0, s>>>(
        prim_s, n, E, cnt);
        aem::chunk_scan_kernel<<<1, aem::kScanThreads, 0, s>>>(cnt, static_cast<int>(c), E, nullptr);
        aem::assign_kernel<aem::kPerThreadApi><<<static_cast<unsigned>(c), aem::kThreads, 0, s>>>(
            prim_s, sec_s, n, E, cnt, capacity, nullptr, 1, inv, effective);
        aem::count_launches(5);
        cudaError_t le = cudaGetLastError();
        if (le != cudaSuccess) {
            set_error("aem_capacity_route: launch failed: %s", cudaGetErrorString(le));
            st = AEM_ECUDA;
        }
    } while (0);
    if (owned) cudaFreeAsync(workspace, s);
    if (st != AEM_OK) return st;
    return aem::check_device_errors(s, "aem_capacity_route");
}

}  // extern "C"

// ============================================================================
// Capacity routing without device allocation.
//
// Some callers cannot allocate device memory while they run: a serving loop
// that reserves its whole memory budget at start-up and forbids growth, or
// one that cannot afford the device-wide synchronisation that cudaFree (and
// often cudaMalloc) implies in the middle of a latency-bound step.  For them
// aem_capacity_route_static keeps its scratch in the file-scope array below,
// sized for AEM_ROUTE_STATIC_MAX_UNITS units and AEM_MAX_EXPERTS experts;
// every GPU that loads this library holds the array until the process exits.
// ============================================================================
namespace aem {
namespace {

constexpr size_t a256(size_t v) { return (v + 255) / 256 * 256; }
constexpr int64_t kStaticUnits = AEM_ROUTE_STATIC_MAX_UNITS;
constexpr int64_t kStaticChunks = (kStaticUnits + kChunk - 1) / kChunk;
constexpr size_t kStaticIdxBytes = a256(sizeof(int32_t) * kStaticUnits);
constexpr size_t kStaticCntBytes = a256(sizeof(int) * kStaticChunks * AEM_MAX_EXPERTS);
// inv, seen, primary and secondary in position order, chunk counts, error word
constexpr size_t kStaticBytes = 4 * kStaticIdxBytes + kStaticCntBytes + 256;
static_assert(kStaticBytes == AEM_ROUTE_STATIC_SCRATCH_BYTES, "scratch size in aem.h");

static __device__ __align__(256) unsigned char g_route_scratch[kStaticBytes];

// Device address of g_route_scratch on the current device.  Host code only
// sees a stand-in symbol, never the address, so it is looked up with the
// device current -- on every call: the lookup allocates nothing, and an
// address cached across calls would dangle after cudaDeviceReset (the
// module, and with it the array, is loaded again into the new context).
aem_status route_scratch_address(void** out) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
    if (e != cudaSuccess || p == nullptr) {
        set_error("aem_capacity_route_static: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
        return AEM_ECUDA;
    }
    *out = p;
    return AEM_OK;
}

}  // namespace
}  // namespace aem

extern "C" aem_status aem_capacity_route_static(const uint32_t* primary, const uint32_t* secondary,
                                                const uint32_t* batch_position, int64_t n, int E,
                                                uint64_t capacity, uint32_t* effective,
                                                void* stream) {
    AEM_REQUIRE(n >= 0, "aem_capacity_route_static: n=%lld must be >= 0", (long long)n);
    AEM_REQUIRE(n <= AEM_ROUTE_STATIC_MAX_UNITS,
                "aem_capacity_route_static: n=%lld exceeds the fixed scratch maximum of %d units "
                "(use aem_capacity_route)",
                (long long)n, AEM_ROUTE_STATIC_MAX_UNITS);
    AEM_REQUIRE(E >= 1 && E <= AEM_MAX_EXPERTS, "aem_capacity_route_static: E=%d outside [1, %d]",
                E, AEM_MAX_EXPERTS);
    if (n == 0) return AEM_OK;
    AEM_REQUIRE(primary && secondary && batch_position && effective,
                "aem_capacity_route_static: NULL buffer");
    auto s = static_cast<cudaStream_t>(stream);
    void* base = nullptr;
    AEM_TRY(aem::route_scratch_address(&base));
    char* w = static_cast<char*>(base);
    int32_t* inv = reinterpret_cast<int32_t*>(w);
    int32_t* seen = reinterpret_cast<int32_t*>(w + aem::kStaticIdxBytes);
    uint32_t* prim_s = reinterpret_cast<uint32_t*>(w + 2 * aem::kStaticIdxBytes);
    uint32_t* sec_s = reinterpret_cast<uint32_t*>(w + 3 * aem::kStaticIdxBytes);
    int* cnt = reinterpret_cast<int*>(w + 4 * aem::kStaticIdxBytes);
    int* err = reinterpret_cast<int*>(w + 4 * aem::kStaticIdxBytes + aem::kStaticCntBytes);
    const int64_t c = aem::route_chunks(n);
    // The array keeps the previous call's contents: reset what must start
    // known (the permutation marks, the inverse, the error word).
    AEM_TRY_CUDA(cudaMemsetAsync(seen, 0, sizeof(int32_t) * n, s));
    AEM_TRY_CUDA(cudaMemsetAsync(inv, 0xFF, sizeof(int32_t) * n, s));
    AEM_TRY_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
    const unsigned gb = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 4096));
    aem::invert_positions_kernel<<<gb, 256, 0, s>>>(batch_position, n, inv, seen, err);
    aem::gather_by_position_kernel<<<gb, 256, 0, s>>>(primary, secondary, inv, n, E, prim_s, sec_s,
                                                      err);
    aem::chunk_count_kernel<aem::kPerThreadApi><<<static_cast<unsigned>(c), aem::kThreads, 0, s>>>(
        prim_s, n, E, cnt);
    aem::chunk_scan_kernel<<<1, aem::kScanThreads, 0, s>>>(cnt, static_cast<int>(c), E, nullptr);
    aem::assign_kernel<aem::kPerThreadApi><<<static_cast<unsigned>(c), aem::kThreads, 0, s>>>(
        prim_s, sec_s, n, E, cnt, capacity, nullptr, 1, inv, effective);
    AEM_CHECK_LAUNCH();
    aem::count_launches(5);
    int bits = 0;
    AEM_TRY_CUDA(cudaMemcpyAsync(&bits, err, sizeof(int), cudaMemcpyDeviceToHost, s));
    AEM_TRY_CUDA(cudaStreamSynchronize(s));
    if (bits & aem::ERR_ROUTE_POSITION) {
        set_error("aem_capacity_route_static: batch_position is not a permutation of [0, n)");
        return AEM_EDEVICE;
    }
    if (bits) {
        set_error("aem_capacity_route_static: expert id out of range (error bits 0x%x)", bits);
        return AEM_EDEVICE;
    }
    return AEM_OK;
}
