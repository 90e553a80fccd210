// Expert-parallel MoE layer: one process per GPU, activations, expert
// outputs and the step's small all-gathers and barriers exchanged by stores
// into the peers' memory over NVLink/NVSwitch.
//
// Replaces the reference's Router scatter/gather over ICollectiveTransport
// (src/orchestration/router.hpp:67-100, collective_transport.hpp:37-51) and
// its tolerant variant (route_batch_tolerant, router.hpp:127-234): the
// routing decision stays Router::assign_effective_experts (router.hpp:249-266)
// and is bit-exact with a single-process run over the global batch, because
// every rank ranks its units by GLOBAL batch_position:
//   units are (token, slot) pairs in slot-major order, u = j*T + t_global, and
//   rank r owns tokens [r*T_l, (r+1)*T_l); so in expert e's group the units of
//   slot j on rank r come after all units of slots < j (every rank) and after
//   slot j of ranks < r.  One all-gather of per-(slot, expert) counts gives
//   each rank that offset; local stable ranks do the rest.
//
// Data movement (no host synchronisation in a step):
//   pairs  -- (token, destination rank): a token's activation row crosses
//             NVLink once per destination rank, not once per unit;
//   units  -- (token, slot): the destination gets, per unit, the row of its
//             pair and its gate weight, at the unit's row in the destination's
//             expert-grouped layout (sources in rank order inside an expert).
//   Step: gating -> slot counts -> [all-gather] -> capacity routing (global
//   ranks) -> pair numbering -> [all-gather of expert starts + pair counts]
//   -> on-device plan -> push pairs + unit metadata into the destinations ->
//   [barrier] -> expand pairs to units -> grouped up GEMM (+ReLU) -> grouped
//   down GEMM, gate-weighted and pre-reduced per pair -> push the pair sums
//   back into the sources -> [barrier] -> per-token sum over destinations.
// The bracketed steps are peer-memory mailboxes and per-step flags: a rank
// writes its payload into every live peer's mailbox, then a flag holding
// (step << 1 | failed) with a system-scope release; a waiter spins on its own
// copy of the flags with a deadline.  A peer that stays silent is recorded
// as suspect and fails the step; a failed step is signalled onward in the
// flags, so every rank that takes part fails it too and every unit of it
// resolves to exactly one outcome (the tolerant contract).
// Receive buffers are sized for the worst case at creation and mapped by
// every peer once (CUDA IPC), so a step never allocates or re-maps.  NCCL only
// bootstraps the mapping and tears it down.
#include <cuda_bf16.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "moe.h"
#include "route.h"
#include "runtime.h"

namespace aem {

// NCCL is resolved at run time, on the first expert-parallel call, not at
// link time: a process that already loaded an NCCL (e.g. the one PyTorch
// ships) keeps using that one, so loading this library never changes which
// NCCL other components of the process see.
struct NcclApi {
    decltype(&::ncclGetUniqueId) GetUniqueId = nullptr;
    decltype(&::ncclCommInitRank) CommInitRank = nullptr;
    decltype(&::ncclCommDestroy) CommDestroy = nullptr;
    decltype(&::ncclCommAbort) CommAbort = nullptr;
    decltype(&::ncclAllGather) AllGather = nullptr;
    decltype(&::ncclAllReduce) AllReduce = nullptr;
    decltype(&::ncclGetErrorString) GetErrorString = nullptr;
};

static std::once_flag g_nccl_once;
static NcclApi g_nccl;
static bool g_nccl_ok = false;
static std::string g_nccl_err;

static const NcclApi* nccl() {
    std::call_once(g_nccl_once, [] {
        // an NCCL already in the process wins; otherwise the loader's default
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char* e = dlerror();
            g_nccl_err = e ? e : "libnccl.so.2 not found";
            return;
        }
        bool ok = true;
        auto sym = [&](auto& fp, const char* name) {
            fp = reinterpret_cast<std::remove_reference_t<decltype(fp)>>(dlsym(h, name));
            if (!fp) {
                ok = false;
                g_nccl_err = std::string("NCCL symbol missing: ") + name;
            }
        };
        sym(g_nccl.GetUniqueId, "ncclGetUniqueId");
        sym(g_nccl.CommInitRank, "ncclCommInitRank");
        sym(g_nccl.CommDestroy, "ncclCommDestroy");
        sym(g_nccl.CommAbort, "ncclCommAbort");
        sym(g_nccl.AllGather, "ncclAllGather");
        sym(g_nccl.AllReduce, "ncclAllReduce");
        sym(g_nccl.GetErrorString, "ncclGetErrorString");
        g_nccl_ok = ok;
    });
    return g_nccl_ok ? &g_nccl : nullptr;
}

}  // namespace aem

#define AEM_TRY_NCCL(expr)                                                              \
    do {                                                                                \
        ncclResult_t aem_n_ = (expr);                                                   \
        if (aem_n_ != ncclSuccess) {                                                    \
            ::aem::set_error("%s:%d: %s failed: %s", __FILE__, __LINE__, #expr,         \
                             ::aem::nccl()->GetErrorString(aem_n_));                    \
            return AEM_ENCCL;                                                           \
        }                                                                               \
    } while (0)

#define AEM_NCCL_OR_FAIL()                                                              \
    do {                                                                                \
        if (!::aem::nccl()) {                                                           \
            ::aem::set_error("NCCL unavailable: %s", ::aem::g_nccl_err.c_str());        \
            return AEM_EUNSUPPORTED;                                                    \
        }                                                                               \
    } while (0)

namespace aem {

// Payload word offsets (see AEM_EP_PAYLOAD): expert starts [E+1], pairs per
// destination [R], live mask [2], half-A units per expert [E], half-A pairs
// per destination [R].
__host__ __device__ constexpr int pay_pairs(int E) { return E + 1; }
__host__ __device__ constexpr int pay_mask(int E, int R) { return E + 1 + R; }
__host__ __device__ constexpr int pay_units_a(int E, int R) { return E + 3 + R; }
__host__ __device__ constexpr int pay_pairs_a(int E, int R) { return 2 * E + 3 + R; }

// Per-step plan of one rank (see aem_ep_peer_plan).  Row s of `all` (stride
// `ld` int32) is rank s's payload.  Only ranks in `live` take part: other
// rows are ignored, and units or pairs addressed to other ranks count as
// absent.  Every rank runs this on the same data, so all agree on `ok`.
// groups: [2][E/R+1], half A's row groups then half B's.
__host__ __device__ inline void plan_peer(const int32_t* all, int ld, int R, int E, int me,
                                          uint64_t live, int64_t ucap, int64_t pcap, int64_t rcap,
                                          aem_ep_peer_plan* pl, int32_t* groups) {
    const int el = E / R;
    const int PP = pay_pairs(E), PUA = pay_units_a(E, R), PPA = pay_pairs_a(E, R);
    auto in = [&](int r) { return ((live >> r) & 1ull) != 0; };
    auto row = [&](int s) { return all + static_cast<int64_t>(s) * ld; };
    auto ut = [&](int s, int e) -> int64_t {  // units of expert e from s
        return (in(s) && in(e / el)) ? row(s)[e + 1] - row(s)[e] : 0;
    };
    auto ua = [&](int s, int e) -> int64_t { return (in(s) && in(e / el)) ? row(s)[PUA + e] : 0; };
    auto pairs = [&](int s, int r) -> int64_t { return (in(s) && in(r)) ? row(s)[PP + r] : 0; };
    auto pairs_a = [&](int s, int r) -> int64_t { return (in(s) && in(r)) ? row(s)[PPA + r] : 0; };
    bool ok = in(me);
    for (int s = 0; s < R && ok; ++s) {
        if (!in(s)) continue;
        const int32_t* a = row(s);
        if (a[0] != 0) ok = false;
        for (int e = 0; e < E; ++e)
            if (a[e + 1] < a[e] || a[PUA + e] < 0 || a[PUA + e] > a[e + 1] - a[e]) ok = false;
        int64_t pout = 0;
        for (int r = 0; r < R; ++r) {
            int64_t u = 0, uA = 0;
            for (int e = r * el; e < (r + 1) * el; ++e) {
                u += ut(s, e);
                uA += ua(s, e);
            }
            const int64_t p = pairs(s, r), pA = pairs_a(s, r);
            // a pair (of a half) exists exactly when the token has a unit there
            if (p < 0 || p > u || ((u > 0) != (p > 0))) ok = false;
            if (pA < 0 || pA > p || pA > uA || ((uA > 0) != (pA > 0))) ok = false;
            if (p - pA > u - uA || ((u - uA > 0) != (p - pA > 0))) ok = false;
            pout += p;
        }
        if (pout > rcap) ok = false;
    }
    for (int r = 0; r < R && ok; ++r) {
        int64_t u = 0, p = 0;
        for (int s = 0; s < R; ++s) {
            for (int e = r * el; e < (r + 1) * el; ++e) u += ut(s, e);
            p += pairs(s, r);
        }
        if (u > ucap || p > pcap) ok = false;
    }
    pl->ok = ok ? 1 : 0;
    pl->units_in = pl->units_in_a = pl->pairs_in = pl->pairs_out = 0;
    for (int r = 0; r < AEM_EP_MAX_RANKS; ++r) {
        pl->dst_pair_off[r] = pl->send_pair_off[r] = pl->send_pair_a[r] = 0;
        pl->recv_pair_off[r] = pl->recv_pair_a[r] = pl->ret_off[r] = 0;
    }
    for (int e = 0; e < AEM_MAX_EXPERTS; ++e) pl->dst_unit_off[0][e] = pl->dst_unit_off[1][e] = 0;
    pl->recv_pair_off[AEM_EP_MAX_RANKS] = 0;
    for (int i = 0; i < 2 * (el + 1); ++i) groups[i] = 0;
    if (!ok) return;
    int64_t acc = 0;
    for (int r = 0; r < R; ++r) {
        pl->send_pair_off[r] = static_cast<int32_t>(acc);
        pl->send_pair_a[r] = static_cast<int32_t>(pairs_a(me, r));
        acc += pairs(me, r);
    }
    pl->pairs_out = static_cast<int32_t>(acc);
    for (int r = 0; r < R; ++r) {
        int64_t p = 0;
        for (int s = 0; s < me; ++s) p += pairs(s, r);
        pl->dst_pair_off[r] = static_cast<int32_t>(p);
        // rank r receives half A then half B, each expert-major with every
        // source's units of one expert contiguous, sources in rank order
        int64_t uA_r = 0;
        for (int e = r * el; e < (r + 1) * el; ++e)
            for (int s = 0; s < R; ++s) uA_r += ua(s, e);
        int64_t u0 = 0, u1 = uA_r;
        for (int e = r * el; e < (r + 1) * el; ++e) {
            int64_t b0 = 0, b1 = 0, t0 = 0, t1 = 0;
            for (int s = 0; s < R; ++s) {
                const int64_t a0 = ua(s, e), a1 = ut(s, e) - ua(s, e);
                if (s < me) {
                    b0 += a0;
                    b1 += a1;
                }
                t0 += a0;
                t1 += a1;
            }
            pl->dst_unit_off[0][e] = static_cast<int32_t>(u0 + b0);
            pl->dst_unit_off[1][e] = static_cast<int32_t>(u1 + b1);
            u0 += t0;
            u1 += t1;
        }
    }
    acc = 0;
    for (int s = 0; s < R; ++s) {
        pl->recv_pair_off[s] = static_cast<int32_t>(acc);
        pl->recv_pair_a[s] = static_cast<int32_t>(pairs_a(s, me));
        acc += pairs(s, me);
        int64_t before = 0;
        for (int r = 0; r < me; ++r) before += pairs(s, r);
        pl->ret_off[s] = static_cast<int32_t>(before);
    }
    pl->recv_pair_off[R] = static_cast<int32_t>(acc);
    pl->pairs_in = static_cast<int32_t>(acc);
    int64_t g = 0;
    for (int h = 0; h < 2; ++h) {
        groups[h * (el + 1)] = static_cast<int32_t>(g);
        for (int e = 0; e < el; ++e) {
            for (int s = 0; s < R; ++s) {
                const int64_t a0 = ua(s, me * el + e);
                g += h == 0 ? a0 : ut(s, me * el + e) - a0;
            }
            groups[h * (el + 1) + e + 1] = static_cast<int32_t>(g);
        }
        if (h == 0) pl->units_in_a = static_cast<int32_t>(g);
    }
    pl->units_in = static_cast<int32_t>(g);
}

namespace {

using namespace aem::dev;

constexpr int kCopyThreads = 256;

// Synchronisation points of a step, one flag per (point, source rank).
enum {
    SYNC_COUNTS = 0,
    SYNC_PLAN = 1,
    SYNC_DISPATCH_A = 2,
    SYNC_DISPATCH_B = 3,
    SYNC_RETURN_A = 4,
    SYNC_RETURN_B = 5,
    kSyncPoints = 6
};

// Base pointers of every rank's exchange region (this rank's own at [me]).
struct EpPeers {
    char* base[AEM_EP_MAX_RANKS];
};

// Byte offsets of the buffers inside an exchange region (identical on all
// ranks because every rank sizes them from the same config and capacity).
struct ExchangeLayout {
    size_t xpair;     // bf16 [pairs_cap][d]    activation rows received
    size_t rowmap;    // int32 [units_cap]      unit -> received pair row
    size_t rowscale;  // f32 [units_cap]        unit -> gate weight
    size_t ret;       // f32 [ret_cap][d]       pair sums returned to this rank
    size_t mail_cnt;  // int64 [R][k*E]         every rank's slot counts
    size_t mail_pay;  // int32 [R][pay_ld]      every rank's starts, pair counts, live mask
    size_t flags;     // uint64 [kSyncPoints][R] (step << 1 | failed) per source rank
    size_t bytes;
};

// Step state on this rank's device.
struct StepState {
    unsigned long long suspect;  // ranks found silent (kept until the host reads them)
    int failed;                  // this step failed (a silent or failed peer, a bad plan)
    int bar;                     // all-reduce word of the teardown barrier
};

// The waits of one synchronisation point: thread r waits for live peer r's
// flag to reach `seq` (or a later step), at most `timeout_ns`.  A silent peer
// becomes suspect; a peer that signalled failure fails this step.  Peers
// already suspect are not waited for.  Ends with __syncthreads().
__device__ void wait_point(const uint64_t* __restrict__ flags, int R, int me, uint64_t live,
                           uint64_t seq, uint64_t timeout_ns, bool tolerant, StepState* st,
                           int* err) {
    const int r = threadIdx.x;
    if (r < R && r != me && ((live >> r) & 1ull) &&
        !((*reinterpret_cast<volatile unsigned long long*>(&st->suspect) >> r) & 1ull)) {
        const uint64_t t0 = globaltimer_ns();
        while (true) {
            const uint64_t v = ld_acquire_sys(flags + r);
            if ((v >> 1) >= seq) {
                if ((v >> 1) == seq && (v & 1ull)) {
                    atomicExch(&st->failed, 1);
                    if (!tolerant) atomicOr(err, ERR_EP_PEER_FAILED);
                }
                break;
            }
            if (globaltimer_ns() - t0 > timeout_ns) {
                atomicOr(&st->suspect, 1ull << r);
                atomicExch(&st->failed, 1);
                if (!tolerant) atomicOr(err, ERR_EP_PEER_TIMEOUT);
                break;
            }
        }
    }
    __syncthreads();
}

__device__ __forceinline__ uint64_t usable(uint64_t live, const StepState* st) {
    return live & ~*reinterpret_cast<const volatile unsigned long long*>(&st->suspect);
}

// Writes `words` 32-bit words of `src` into slot `me` of every usable rank's
// mailbox (offset `slot_off`, slot stride `slot_words`), then, per rank, a
// system-scope fence and the flag (seq << 1 | failed) of `point`.
__global__ void ep_publish_kernel(const uint32_t* __restrict__ src, int words, int slot_words,
                                  EpPeers peers, size_t slot_off, size_t flag_off, int point,
                                  int me, int R, uint64_t live, uint64_t seq, StepState* st) {
    const uint64_t to = usable(live, st);
    for (int r = 0; r < R; ++r) {
        if (!((to >> r) & 1ull)) continue;
        uint32_t* dst = reinterpret_cast<uint32_t*>(peers.base[r] + slot_off) +
                        static_cast<int64_t>(me) * slot_words;
        for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
    const int r = threadIdx.x;
    if (r < R && ((to >> r) & 1ull)) {
        const uint64_t failed = *reinterpret_cast<volatile int*>(&st->failed) ? 1ull : 0ull;
        __threadfence_system();
        uint64_t* f = reinterpret_cast<uint64_t*>(peers.base[r] + flag_off) +
                      static_cast<int64_t>(point) * R + me;
        st_release_sys(f, (seq << 1) | failed);
    }
}

__global__ void ep_wait_kernel(const uint64_t* __restrict__ flags, int R, int me, uint64_t live,
                               uint64_t seq, uint64_t timeout_ns, int tolerant, StepState* st,
                               int* err) {
    wait_point(flags, R, me, live, seq, timeout_ns, tolerant != 0, st, err);
}

// cnt[j][e] = number of local tokens whose slot-j choice is e.
__global__ void slot_count_kernel(const int32_t* __restrict__ idx, int64_t T, int ldi, int k, int E,
                                  unsigned long long* __restrict__ cnt) {
    extern __shared__ unsigned int h[];  // [k][E]
    for (int i = threadIdx.x; i < k * E; i += blockDim.x) h[i] = 0;
    __syncthreads();
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < T * k;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / k;
        const int j = static_cast<int>(i % k);
        const int e = idx[t * ldi + j];
        if (e >= 0 && e < E) atomicAdd(&h[j * E + e], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < k * E; i += blockDim.x)
        if (h[i]) atomicAdd(&cnt[i], static_cast<unsigned long long>(h[i]));
}

// After the counts' point: corr[j][e] = base[j][e] - (local units of expert e
// in slots < j), where base[j][e] = sum_{j'<j} sum_r' all[r'][j'][e] +
// sum_{r'<r} all[r'][j][e] over the usable ranks.
__global__ void ep_corr_kernel(const long long* __restrict__ all, const uint64_t* __restrict__ flags,
                               int R, int k, int E, int rank, uint64_t live, uint64_t seq,
                               uint64_t timeout_ns, int tolerant, StepState* st, int* err,
                               long long* __restrict__ corr) {
    wait_point(flags, R, rank, live, seq, timeout_ns, tolerant != 0, st, err);
    const uint64_t use = usable(live, st) | (1ull << rank);
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        long long before_slots = 0, local_before = 0;
        for (int j = 0; j < k; ++j) {
            long long before_ranks = 0, slot_total = 0;
            for (int r = 0; r < R; ++r) {
                if (!((use >> r) & 1ull)) continue;
                const long long v = all[(static_cast<int64_t>(r) * k + j) * E + e];
                if (r < rank) before_ranks += v;
                slot_total += v;
            }
            corr[j * E + e] = before_slots + before_ranks - local_before;
            before_slots += slot_total;
            local_before += all[(static_cast<int64_t>(rank) * k + j) * E + e];
        }
    }
}

// Expert ids of the gating output in placement order: pos[e] = rank(e)*el +
// (index of e among its rank's experts), so every rank's experts are one
// contiguous range of the routing's expert-sorted units.
__global__ void relabel_kernel(const int32_t* __restrict__ in, int64_t n,
                               const int32_t* __restrict__ pos, int32_t* __restrict__ out) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = pos[in[i]];
}

// Back to expert ids: out[i] = expert[in[i]] (placement position -> id).
__global__ void unlabel_kernel(const uint32_t* __restrict__ in, int64_t n,
                               const int32_t* __restrict__ expert, uint32_t* __restrict__ out) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = static_cast<uint32_t>(expert[in[i]]);
}

// Block r numbers the tokens that have at least one unit on rank r, in token
// order: pair_local[r][t] = that number, or -1 (always -1 for a rank outside
// `live`: its units fail); half-A tokens (t < half_T) come first.  Writes the
// all-gather payload: the expert starts, the pair count per destination, the
// live mask, the half-A units per expert (block 0) and the half-A pairs per
// destination.
__global__ void __launch_bounds__(1024)
    ep_pairs_kernel(const uint32_t* __restrict__ eff, int64_t T, int64_t half_T, int k, int el,
                    int E, int R, uint64_t live, const int* __restrict__ starts,
                    int32_t* __restrict__ pair_local, int32_t* __restrict__ payload) {
    __shared__ int wsum[32];
    __shared__ int running, running_a;
    __shared__ int hist[AEM_MAX_EXPERTS];
    const int r = blockIdx.x;
    const bool on = ((live >> r) & 1ull) != 0;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = blockDim.x >> 5;
    if (r == 0) {
        for (int i = tid; i <= E; i += blockDim.x) payload[i] = starts[i];
        for (int i = tid; i < E; i += blockDim.x) hist[i] = 0;
        if (tid == 0) {
            payload[pay_mask(E, R)] = static_cast<int32_t>(live & 0xFFFFFFFFull);
            payload[pay_mask(E, R) + 1] = static_cast<int32_t>(live >> 32);
        }
        __syncthreads();
        for (int64_t i = tid; i < half_T * k; i += blockDim.x) {  // half-A units per expert
            const int64_t j = i / half_T, t = i % half_T;
            const uint32_t e = eff[j * T + t];
            if (e < static_cast<uint32_t>(E)) atomicAdd(&hist[e], 1);
        }
        __syncthreads();
        for (int i = tid; i < E; i += blockDim.x) payload[pay_units_a(E, R) + i] = hist[i];
    }
    if (tid == 0) running = running_a = 0;
    __syncthreads();
    for (int64_t base = 0; base < T; base += blockDim.x) {
        const int64_t t = base + tid;
        bool f = false;
        if (on && t < T)
            for (int j = 0; j < k; ++j)
                f |= static_cast<int>(eff[static_cast<int64_t>(j) * T + t]) / el == r;
        const unsigned b = __ballot_sync(0xFFFFFFFFu, f);
        const unsigned ba = __ballot_sync(0xFFFFFFFFu, f && t < half_T);
        if (lane == 0 && ba) atomicAdd(&running_a, __popc(ba));
        const int pre = __popc(b & ((1u << lane) - 1u));
        if (lane == 0) wsum[warp] = __popc(b);
        __syncthreads();
        if (warp == 0) {
            int v = lane < nwarps ? wsum[lane] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xFFFFFFFFu, v, o);
                if (lane >= o) v += n;
            }
            wsum[lane] = v;  // inclusive
        }
        __syncthreads();
        const int run = running;
        const int wbase = warp ? wsum[warp - 1] : 0;
        if (t < T) pair_local[static_cast<int64_t>(r) * T + t] = f ? run + wbase + pre : -1;
        __syncthreads();
        if (tid == 0) running = run + wsum[nwarps - 1];
        __syncthreads();
    }
    if (tid == 0) {
        payload[pay_pairs(E) + r] = running;
        payload[pay_pairs_a(E, R) + r] = running_a;
    }
}

// plan_peer for one thread block, in parallel over ranks and experts, with
// the per-rank tables in shared memory (the single-thread form is
// latency-bound on thousands of dependent loads).  Same results as
// plan_peer, field by field; `check_masks` also requires every usable row's
// live mask (words E+1+R, E+2+R) to equal `live`.  Dynamic shared memory:
// plan_block_smem(R, E, ld) bytes.  Returns in every thread whether the plan
// is ok.
__host__ __device__ constexpr size_t plan_block_smem(int R, int E, int ld) {
    return (void)ld, sizeof(int32_t) * (4 * static_cast<size_t>(R) * R + 4 * E) + 16;
}

__device__ bool plan_peer_block(const int32_t* __restrict__ all, int ld, int R, int E, int me,
                                uint64_t live, bool check_masks, bool already_failed, int64_t ucap,
                                int64_t pcap, int64_t rcap, aem_ep_peer_plan* __restrict__ pl,
                                int32_t* __restrict__ groups) {
    extern __shared__ int32_t sm[];
    const int32_t* A = all;               // [R][ld] payload rows (L2; every load independent)
    int32_t* U = sm;                      // [R][R] units s -> r
    int32_t* UA = U + R * R;              // [R][R] half-A units s -> r
    int32_t* P = UA + R * R;              // [R][R] pairs s -> r
    int32_t* PA = P + R * R;              // [R][R] half-A pairs s -> r
    int32_t* colA = PA + R * R;           // [E] half-A units of expert e, every source
    int32_t* colB = colA + E;             // [E] half-B units
    int32_t* befA = colB + E;             // [E] half-A units from sources < me
    int32_t* befB = befA + E;             // [E] half-B units from sources < me
    __shared__ int bad;
    const int tid = threadIdx.x, nt = blockDim.x;
    const int el = E / R;
    const int PP = pay_pairs(E), PM = pay_mask(E, R), PUA = pay_units_a(E, R),
              PPA = pay_pairs_a(E, R);
    auto in = [&](int r) { return ((live >> r) & 1ull) != 0; };
    if (tid == 0) bad = (already_failed || !in(me)) ? 1 : 0;
    __syncthreads();
    for (int i = tid; i < R * (E + 1); i += nt) {
        const int sr = i / (E + 1), e = i % (E + 1);
        if (!in(sr)) continue;
        const int32_t* a = A + sr * ld;
        if (e == 0) {
            if (a[0] != 0) bad = 1;
        } else if (a[e] < a[e - 1] || a[PUA + e - 1] < 0 || a[PUA + e - 1] > a[e] - a[e - 1]) {
            bad = 1;
        }
    }
    for (int i = tid; i < R * R; i += nt) {
        const int sr = i / R, r = i % R;
        const bool on = in(sr) && in(r);
        const int32_t* a = A + sr * ld;
        int32_t u = 0, ua = 0;
        if (on) {
            u = a[(r + 1) * el] - a[r * el];
            for (int e = r * el; e < (r + 1) * el; ++e) ua += a[PUA + e];
        }
        const int32_t p = on ? a[PP + r] : 0;
        const int32_t pa = on ? a[PPA + r] : 0;
        U[i] = u;
        UA[i] = ua;
        P[i] = p;
        PA[i] = pa;
        // a pair (of a half) exists exactly when the token has a unit there
        if (p < 0 || p > u || ((u > 0) != (p > 0))) bad = 1;
        if (pa < 0 || pa > p || pa > ua || ((ua > 0) != (pa > 0))) bad = 1;
        if (p - pa > u - ua || ((u - ua > 0) != (p - pa > 0))) bad = 1;
    }
    if (check_masks)
        for (int sr = tid; sr < R; sr += nt) {
            if (!in(sr)) continue;
            const int32_t* a = A + sr * ld;
            const uint64_t m = static_cast<uint32_t>(a[PM]) |
                               (static_cast<uint64_t>(static_cast<uint32_t>(a[PM + 1])) << 32);
            if (m != live) bad = 1;  // the ranks disagree on who takes part
        }
    for (int e = tid; e < E; e += nt) {
        int32_t ca = 0, cb = 0, ba = 0, bb = 0;
        const bool on = in(e / el);
        for (int sr = 0; sr < R; ++sr) {
            if (!on || !in(sr)) continue;
            const int32_t* a = A + sr * ld;
            const int32_t va = a[PUA + e], vb = a[e + 1] - a[e] - va;
            ca += va;
            cb += vb;
            if (sr < me) {
                ba += va;
                bb += vb;
            }
        }
        colA[e] = ca;
        colB[e] = cb;
        befA[e] = ba;
        befB[e] = bb;
    }
    __syncthreads();
    for (int i = tid; i < 2 * R; i += nt) {
        const int r = i % R;
        int64_t sum = 0;
        if (i < R) {  // everything rank r sends
            for (int q = 0; q < R; ++q) sum += P[r * R + q];
            if (sum > rcap) bad = 1;
        } else {      // everything rank r receives
            int64_t u = 0;
            for (int q = 0; q < R; ++q) {
                u += U[q * R + r];
                sum += P[q * R + r];
            }
            if (u > ucap || sum > pcap) bad = 1;
        }
    }
    __syncthreads();
    const bool ok = bad == 0;
    // every field is written (zeros past R, past E, or for a bad plan)
    for (int i = tid; i < AEM_MAX_EXPERTS; i += nt) {
        pl->dst_unit_off[0][i] = 0;
        pl->dst_unit_off[1][i] = 0;
    }
    for (int i = tid; i <= AEM_EP_MAX_RANKS; i += nt) {
        if (i < AEM_EP_MAX_RANKS) {
            pl->dst_pair_off[i] = 0;
            pl->send_pair_off[i] = 0;
            pl->send_pair_a[i] = 0;
            pl->recv_pair_a[i] = 0;
            pl->ret_off[i] = 0;
        }
        pl->recv_pair_off[i] = 0;
    }
    for (int i = tid; i < 2 * (el + 1); i += nt) groups[i] = 0;
    __syncthreads();
    if (!ok) {
        if (tid == 0) {
            pl->ok = 0;
            pl->units_in = pl->units_in_a = pl->pairs_in = pl->pairs_out = 0;
        }
        return false;
    }
    for (int r = tid; r < R; r += nt) {
        int32_t so = 0, dp = 0, ro = 0, rt = 0;
        for (int q = 0; q < r; ++q) so += P[me * R + q];   // my pairs for ranks < r
        for (int q = 0; q < me; ++q) dp += P[q * R + r];   // pairs to r from ranks < me
        for (int q = 0; q < r; ++q) ro += P[q * R + me];   // pairs I receive from ranks < r
        for (int q = 0; q < me; ++q) rt += P[r * R + q];   // r's pairs for ranks < me
        pl->send_pair_off[r] = so;
        pl->send_pair_a[r] = PA[me * R + r];
        pl->dst_pair_off[r] = dp;
        pl->recv_pair_off[r] = ro;
        pl->recv_pair_a[r] = PA[r * R + me];
        pl->ret_off[r] = rt;
        // rank r receives half A then half B, each expert-major, sources in
        // rank order inside an expert
        int32_t ua_r = 0;
        for (int e = r * el; e < (r + 1) * el; ++e) ua_r += colA[e];
        int32_t u0 = 0, u1 = ua_r;
        for (int e = r * el; e < (r + 1) * el; ++e) {
            pl->dst_unit_off[0][e] = u0 + befA[e];
            pl->dst_unit_off[1][e] = u1 + befB[e];
            u0 += colA[e];
            u1 += colB[e];
        }
    }
    if (tid == 0) {
        int32_t out = 0, inn = 0, g = 0;
        for (int q = 0; q < R; ++q) {
            out += P[me * R + q];
            inn += P[q * R + me];
        }
        for (int h = 0; h < 2; ++h) {
            groups[h * (el + 1)] = g;
            for (int le = 0; le < el; ++le) {
                g += h == 0 ? colA[me * el + le] : colB[me * el + le];
                groups[h * (el + 1) + le + 1] = g;
            }
            if (h == 0) pl->units_in_a = g;
        }
        pl->pairs_out = out;
        pl->pairs_in = inn;
        pl->recv_pair_off[R] = inn;
        pl->units_in = g;
        pl->ok = 1;
    }
    return true;
}

// After the plan's point: the plan over the usable ranks; a failed step
// plans nothing.
__global__ void ep_plan_kernel(const int32_t* __restrict__ all, int ld,
                               const uint64_t* __restrict__ flags, int R, int E, int me,
                               uint64_t live, uint64_t seq, uint64_t timeout_ns, int tolerant,
                               int64_t ucap, int64_t pcap, int64_t rcap, StepState* st,
                               aem_ep_peer_plan* __restrict__ plan, int32_t* __restrict__ groups,
                               int* __restrict__ err) {
    wait_point(flags, R, me, live, seq, timeout_ns, tolerant != 0, st, err);
    const uint64_t use = usable(live, st);
    const bool failed = *reinterpret_cast<volatile int*>(&st->failed) != 0;
    const bool ok = plan_peer_block(all, ld, R, E, me, use, true, failed, ucap, pcap, rcap, plan,
                                    groups);
    if (threadIdx.x == 0 && !ok && !failed) {
        atomicOr(err, ERR_EP_PLAN);
        st->failed = 1;
    }
}

// The block plan on given rows (no waits): the device twin of
// aem_ep_plan_peer, for tests.
__global__ void ep_plan_test_kernel(const int32_t* __restrict__ all, int R, int E, int me,
                                    uint64_t live, int64_t ucap, int64_t pcap, int64_t rcap,
                                    aem_ep_peer_plan* __restrict__ plan,
                                    int32_t* __restrict__ groups) {
    plan_peer_block(all, AEM_EP_PAYLOAD(E, R), R, E, me, live, false, false, ucap, pcap, rcap, plan,
                    groups);
}

// One warp copies one row of d elements (d % 8 == 0) to bf16.
template <typename XT>
__device__ __forceinline__ void copy_row_bf16(const XT* __restrict__ in, __nv_bfloat16* out,
                                              int64_t d, int lane) {
    if constexpr (sizeof(XT) == 2) {
        const uint4* vi = reinterpret_cast<const uint4*>(in);
        uint4* vo = reinterpret_cast<uint4*>(out);
        for (int64_t i = lane; i < d / 8; i += 32) vo[i] = __ldg(vi + i);
    } else {
        const float4* vi = reinterpret_cast<const float4*>(in);
        uint4* vo = reinterpret_cast<uint4*>(out);
        for (int64_t i = lane; i < d / 8; i += 32) {
            const float4 a = __ldg(vi + 2 * i), b = __ldg(vi + 2 * i + 1);
            __nv_bfloat162 p0 = __floats2bfloat162_rn(a.x, a.y);
            __nv_bfloat162 p1 = __floats2bfloat162_rn(a.z, a.w);
            __nv_bfloat162 p2 = __floats2bfloat162_rn(b.x, b.y);
            __nv_bfloat162 p3 = __floats2bfloat162_rn(b.z, b.w);
            uint4 u;
            u.x = *reinterpret_cast<uint32_t*>(&p0);
            u.y = *reinterpret_cast<uint32_t*>(&p1);
            u.z = *reinterpret_cast<uint32_t*>(&p2);
            u.w = *reinterpret_cast<uint32_t*>(&p3);
            vo[i] = u;
        }
    }
}

// Push one half (0 = A: tokens t < half_T, 1 = B): (a) each of its
// (destination, token) pairs' activation row into the destination's pair
// rows; (b) each of its units' (pair row, gate weight) into the destination's
// unit row.  Units of this rank are expert-sorted with half A first inside
// every expert (cnt_a[e] of them), so unit i of expert e lands at
// dst_unit_off[half][e] + its index inside its half.  Units for a rank outside
// the step have no pair and are skipped (they fail).
template <typename XT>
__global__ void __launch_bounds__(kCopyThreads)
    ep_dispatch_kernel(const XT* __restrict__ x, int64_t T, int64_t half_T, int half, int64_t d,
                       int R, int el, const int32_t* __restrict__ pair_local,
                       const int* __restrict__ starts, const int32_t* __restrict__ cnt_a,
                       const int32_t* __restrict__ src_token, const float* __restrict__ rowscale,
                       int k, const aem_ep_peer_plan* __restrict__ plan, EpPeers peers,
                       ExchangeLayout lay, int64_t ucap, int64_t pcap, int* __restrict__ err) {
    __shared__ int bnd[AEM_MAX_EXPERTS + 1];
    __shared__ int ca[AEM_MAX_EXPERTS];
    __shared__ int upos[AEM_MAX_EXPERTS];
    __shared__ int ppos[AEM_EP_MAX_RANKS];
    if (!plan->ok) return;
    const int E = R * el;
    for (int i = threadIdx.x; i <= E; i += blockDim.x) bnd[i] = starts[i];
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
        ca[i] = cnt_a[i];
        upos[i] = plan->dst_unit_off[half][i];
    }
    for (int i = threadIdx.x; i < R; i += blockDim.x) ppos[i] = plan->dst_pair_off[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t t_lo = half ? half_T : 0, t_hi = half ? T : half_T, tn = t_hi - t_lo;
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
         i < R * tn; i += nw) {
        const int r = static_cast<int>(i / tn);
        const int64_t t = t_lo + (i - static_cast<int64_t>(r) * tn);
        const int pl = pair_local[static_cast<int64_t>(r) * T + t];
        if (pl < 0) continue;
        const int64_t row = static_cast<int64_t>(ppos[r]) + pl;
        if (row >= pcap) {
            if (lane == 0) atomicOr(err, ERR_EP_BOUNDS);
            continue;
        }
        auto* dst = reinterpret_cast<__nv_bfloat16*>(peers.base[r] + lay.xpair) + row * d;
        copy_row_bf16<XT>(x + t * d, dst, d, lane);
    }
    const int64_t U = min(static_cast<int64_t>(bnd[E]), T * k);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < U;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int lo = 0, hi = E - 1;  // the expert segment holding sorted unit i
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (bnd[mid] <= i) lo = mid; else hi = mid - 1;
        }
        const int e = lo;
        const int64_t q = i - bnd[e];
        const bool in_a = q < ca[e];
        if (in_a != (half == 0)) continue;
        const int r = e / el;
        const int64_t t = src_token[i];
        const int pl = (t >= 0 && t < T) ? pair_local[static_cast<int64_t>(r) * T + t] : -1;
        if (pl < 0) continue;  // a rank outside the step: the unit fails
        const int64_t pos = upos[e] + (in_a ? q : q - ca[e]);
        if (pos >= ucap) {
            atomicOr(err, ERR_EP_BOUNDS);
            continue;
        }
        reinterpret_cast<int32_t*>(peers.base[r] + lay.rowmap)[pos] = ppos[r] + pl;
        reinterpret_cast<float*>(peers.base[r] + lay.rowscale)[pos] = __ldg(rowscale + i);
    }
}

// The pair row p received by this rank belongs to half A when it is among the
// first recv_pair_a[s] rows from its source s.  Returns s and sets *in_a.
__device__ __forceinline__ int pair_source(int64_t p, const int* off, const int* pa, int R,
                                           bool* in_a) {
    int s = 0;
    while (s + 1 < R && p >= off[s + 1]) ++s;
    *in_a = p - off[s] < pa[s];
    return s;
}

// Destination side, after one half's dispatch point: that half's unit rows
// from the received pair rows (the grouped GEMM input), and its zeroed pair
// sums for the down GEMM to accumulate into.
__global__ void __launch_bounds__(kCopyThreads)
    ep_expand_kernel(const __nv_bfloat16* __restrict__ xpair, int32_t* __restrict__ rowmap_in,
                     float* __restrict__ rowscale_in, const aem_ep_peer_plan* __restrict__ plan,
                     const StepState* st, int half, int R, int64_t d,
                     __nv_bfloat16* __restrict__ xu, float* __restrict__ ret_acc,
                     int* __restrict__ err) {
    __shared__ int off[AEM_EP_MAX_RANKS + 1];
    __shared__ int pa[AEM_EP_MAX_RANKS];
    if (!plan->ok || *reinterpret_cast<const volatile int*>(&st->failed)) return;
    for (int i = threadIdx.x; i <= R; i += blockDim.x) off[i] = plan->recv_pair_off[i];
    for (int i = threadIdx.x; i < R; i += blockDim.x) pa[i] = plan->recv_pair_a[i];
    __syncthreads();
    const int64_t u_lo = half ? plan->units_in_a : 0;
    const int64_t u_hi = half ? plan->units_in : plan->units_in_a;
    const int64_t pairs = plan->pairs_in;
    const int lane = threadIdx.x & 31;
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t u = u_lo + blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) +
                     (threadIdx.x >> 5);
         u < u_hi; u += nw) {
        const int64_t p = rowmap_in[u];
        uint4* vo = reinterpret_cast<uint4*>(xu + u * d);
        if (p < 0 || p >= pairs) {  // a unit row no source wrote: contributes nothing
            __syncwarp();
            if (lane == 0) {
                atomicOr(err, ERR_EP_BOUNDS);
                rowmap_in[u] = 0;
                rowscale_in[u] = 0.0f;
            }
            for (int64_t i = lane; i < d / 8; i += 32) vo[i] = make_uint4(0, 0, 0, 0);
            continue;
        }
        const uint4* vi = reinterpret_cast<const uint4*>(xpair + p * d);
        for (int64_t i = lane; i < d / 8; i += 32) vo[i] = vi[i];
    }
    // zero this half's pair sums: one warp per pair row
    for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
         p < pairs; p += nw) {
        bool in_a;
        pair_source(p, off, pa, R, &in_a);
        if (in_a != (half == 0)) continue;
        float4* z = reinterpret_cast<float4*>(ret_acc + p * d);
        for (int64_t i = lane; i < d / 4; i += 32) z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Return one half: pair sum p (from source s) into row ret_off[s] +
// (p - recv_pair_off[s]) of s's return rows; the sums of this rank's own
// pairs are not copied (the combine reads them where the down GEMM left them).
__global__ void __launch_bounds__(kCopyThreads)
    ep_return_kernel(const float* __restrict__ ret_acc, const aem_ep_peer_plan* __restrict__ plan,
                     const StepState* st, int half, int R, int me, int64_t d, EpPeers peers,
                     ExchangeLayout lay, int64_t rcap, int* __restrict__ err) {
    __shared__ int off[AEM_EP_MAX_RANKS + 1];
    __shared__ int pa[AEM_EP_MAX_RANKS];
    __shared__ int ret[AEM_EP_MAX_RANKS];
    if (!plan->ok || *reinterpret_cast<const volatile int*>(&st->failed)) return;
    for (int i = threadIdx.x; i <= R; i += blockDim.x) off[i] = plan->recv_pair_off[i];
    for (int i = threadIdx.x; i < R; i += blockDim.x) {
        pa[i] = plan->recv_pair_a[i];
        ret[i] = plan->ret_off[i];
    }
    __syncthreads();
    const int64_t pairs = off[R];
    const int lane = threadIdx.x & 31;
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
         p < pairs; p += nw) {
        bool in_a;
        const int s = pair_source(p, off, pa, R, &in_a);
        if (s == me || in_a != (half == 0)) continue;  // own sums stay where they are
        const int64_t row = ret[s] + (p - off[s]);
        if (row >= rcap) {
            if (lane == 0) atomicOr(err, ERR_EP_BOUNDS);
            continue;
        }
        const float4* vi = reinterpret_cast<const float4*>(ret_acc + p * d);
        float4* vo = reinterpret_cast<float4*>(reinterpret_cast<float*>(peers.base[s] + lay.ret) +
                                               row * d);
        for (int64_t i = lane; i < d / 4; i += 32) vo[i] = vi[i];
    }
}

// After the return point: out[t] = sum over destination ranks r (increasing)
// of the returned pair sum; unit_failed[j*T + t] = 1 for a unit whose expert's
// rank is outside the step, or for every unit of a failed step (out = 0).
// One warp per token: the token's present pair rows are compacted once (in
// rank order), then every 16-byte column block loads them independently.
template <typename OT>
__global__ void __launch_bounds__(kCopyThreads)
    ep_combine_kernel(const float* __restrict__ ret_in, const float* __restrict__ ret_own,
                      const int32_t* __restrict__ pair_local,
                      const aem_ep_peer_plan* __restrict__ plan, const StepState* st,
                      const uint32_t* __restrict__ eff, int k, int el, uint64_t live, int64_t T,
                      int R, int me, int64_t d, OT* __restrict__ out,
                      uint8_t* __restrict__ unit_failed) {
    __shared__ const float* rows_s[kCopyThreads / 32][AEM_EP_MAX_RANKS];
    const int lane = threadIdx.x & 31;
    const int wib = threadIdx.x >> 5;
    const bool ok = plan->ok != 0 && !*reinterpret_cast<const volatile int*>(&st->failed);
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const int64_t d4 = d / 4;
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + wib; t < T; t += nw) {
        if (unit_failed)
            for (int j = lane; j < k; j += 32) {
                const int64_t u = static_cast<int64_t>(j) * T + t;
                const int r = static_cast<int>(eff[u]) / el;
                unit_failed[u] = (!ok || !((live >> r) & 1ull)) ? 1 : 0;
            }
        int n = 0;  // compact this token's pair rows, rank order
        if (ok)
            for (int r0 = 0; r0 < R; r0 += 32) {
                const int r = r0 + lane;
                const float* row = nullptr;
                if (r < R) {
                    const int pl = pair_local[static_cast<int64_t>(r) * T + t];
                    if (pl >= 0)  // own pairs: the down GEMM's sums, at this rank's receive rows
                        row = r == me ? ret_own + (static_cast<int64_t>(plan->recv_pair_off[me]) +
                                                   pl) * d
                                      : ret_in + (static_cast<int64_t>(plan->send_pair_off[r]) +
                                                  pl) * d;
                }
                const unsigned m = __ballot_sync(0xFFFFFFFFu, row != nullptr);
                if (row) rows_s[wib][n + __popc(m & ((1u << lane) - 1u))] = row;
                n += __popc(m);
            }
        __syncwarp();
        for (int64_t c = lane; c < d4; c += 32) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            int i = 0;
            for (; i + 4 <= n; i += 4) {
                float4 v[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) v[q] = reinterpret_cast<const float4*>(rows_s[wib][i + q])[c];
#pragma unroll
                for (int q = 0; q < 4; ++q) {  // rank order kept: ((a + b) + c) + d
                    acc.x += v[q].x;
                    acc.y += v[q].y;
                    acc.z += v[q].z;
                    acc.w += v[q].w;
                }
            }
            for (; i < n; ++i) {
                const float4 v = reinterpret_cast<const float4*>(rows_s[wib][i])[c];
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
                reinterpret_cast<uint2*>(out + t * d)[c] = u;
            } else {
                reinterpret_cast<float4*>(out + t * d)[c] = acc;
            }
        }
        __syncwarp();
    }
}

size_t align256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

}  // namespace

struct Ep {
    aem_moe_config cfg{};
    int rank = 0, world = 1, device = 0, e_loc = 0;
    ncclComm_t comm = nullptr;
    Gate* gate = nullptr;
    QWeight* up = nullptr;
    QWeight* down = nullptr;
    Moe loc;  // routing buffers of the single-GPU layer (sized for T_cap tokens)
    int64_t T_cap = 0;
    int64_t units_cap = 0, pairs_cap = 0, ret_cap = 0;
    int pay_ld = 0;  // int32 words per payload row, AEM_EP_PAYLOAD(E, R)
    // exchange region: this rank's own, and every rank's mapping of it
    ExchangeLayout lay{};
    void* xreg = nullptr;
    EpPeers peers{};
    bool mapped[AEM_EP_MAX_RANKS] = {};
    // local buffers
    void* lbuf = nullptr;
    unsigned long long* cnt = nullptr;  // [k][E]
    long long* corr = nullptr;          // [k][E]
    int32_t* payload = nullptr;         // [pay_ld]
    aem_ep_peer_plan* plan = nullptr;
    int32_t* groups = nullptr;          // [2][E/R+1] received rows per local expert, per half
    int32_t* pair_local = nullptr;      // [R][T]
    StepState* st = nullptr;
    void* xu = nullptr;                 // bf16 [units_cap][d]
    void* hu = nullptr;                 // bf16 [units_cap][ffn]
    float* ret_acc = nullptr;           // f32 [pairs_cap][d]
    int32_t* idx_pos = nullptr;         // [T_cap][ksel] gating ids in placement order
    int32_t* pos_of = nullptr;          // [E] expert id -> placement position
    int32_t* expert_at = nullptr;       // [E] placement position -> expert id
    bool placed = false;                // placement is not the contiguous map
    std::vector<int32_t> h_pos;         // host copy of pos_of
    // health
    uint64_t seq = 0;                   // steps issued (every taking-part rank in lockstep)
    uint64_t unhealthy = 0;             // ranks left out of every later step
    uint64_t timeout_ns = 2000000000ull;
    unsigned long long* h_suspect = nullptr;  // pinned copy for aem_ep_health
    int pipeline = -1;                  // two-half pipeline: -1 automatic (off), 0 off, 1 on
    // second stream of the two-half pipeline and its joins
    cudaStream_t aux = nullptr;
    cudaEvent_t ev_plan = nullptr, ev_disp_b = nullptr, ev_down_a = nullptr, ev_ret_a = nullptr;
    int64_t last_T = 0;
    PhaseProfiler prof;

    aem_status init(int64_t max_tokens);
    aem_status map_peers(cudaStream_t s);
    void release();
    uint64_t all_mask() const { return world >= 64 ? ~0ull : ((1ull << world) - 1ull); }
    aem_status forward(const void* x, aem_dtype xd, int64_t T, void* out, aem_dtype od,
                       uint8_t* unit_failed, bool tolerant, cudaStream_t s);
};

aem_status Ep::init(int64_t max_tokens) {
    const int k = cfg.top_k, E = cfg.num_experts, R = world;
    const int64_t d = cfg.d_model, f = cfg.d_ffn;
    T_cap = std::max<int64_t>(max_tokens, 1);
    units_cap = static_cast<int64_t>(R) * T_cap * k;  // every unit of every rank
    pairs_cap = static_cast<int64_t>(R) * T_cap;      // every token of every rank
    ret_cap = T_cap * std::min(R, k);                 // a token has <= min(R, k) destinations
    pay_ld = AEM_EP_PAYLOAD(E, R);                    // 16-byte rows
    AEM_REQUIRE(units_cap < (1ll << 31) && pairs_cap * d < (1ll << 40),
                "aem_ep_create: max_tokens_local=%lld too large for %d ranks x top-%d",
                (long long)max_tokens, R, k);
    AEM_TRY(loc.reserve(T_cap, false));
    size_t off = 0;
    auto slot = [&](size_t bytes) {
        const size_t o = off;
        off += align256(bytes);
        return o;
    };
    lay.xpair = slot(2 * pairs_cap * d);
    lay.rowmap = slot(sizeof(int32_t) * units_cap);
    lay.rowscale = slot(sizeof(float) * units_cap);
    lay.ret = slot(sizeof(float) * ret_cap * d);
    lay.mail_cnt = slot(sizeof(long long) * R * k * E);
    lay.mail_pay = slot(sizeof(int32_t) * R * pay_ld);
    lay.flags = slot(sizeof(uint64_t) * kSyncPoints * R);
    lay.bytes = off;
    AEM_TRY_CUDA(cudaMalloc(&xreg, lay.bytes));
    AEM_TRY_CUDA(cudaMemset(xreg, 0, lay.bytes));
    off = 0;
    const int ksel = k < E ? k + 1 : k;
    const size_t o_cnt = slot(sizeof(unsigned long long) * k * E);
    const size_t o_corr = slot(sizeof(long long) * k * E);
    const size_t o_pay = slot(sizeof(int32_t) * pay_ld);
    const size_t o_plan = slot(sizeof(aem_ep_peer_plan));
    const size_t o_groups = slot(sizeof(int32_t) * 2 * (E + 1));
    const size_t o_pl = slot(sizeof(int32_t) * R * T_cap);
    const size_t o_st = slot(sizeof(StepState));
    const size_t o_ipos = slot(sizeof(int32_t) * T_cap * ksel);
    const size_t o_pos = slot(sizeof(int32_t) * E);
    const size_t o_exp = slot(sizeof(int32_t) * E);
    const size_t o_xu = slot(2 * units_cap * d);
    const size_t o_hu = slot(2 * units_cap * f);
    const size_t o_ret = slot(sizeof(float) * pairs_cap * d);
    AEM_TRY_CUDA(cudaMalloc(&lbuf, off));
    AEM_TRY_CUDA(cudaMemset(lbuf, 0, o_xu));  // everything but the big row buffers
    char* b = static_cast<char*>(lbuf);
    cnt = reinterpret_cast<unsigned long long*>(b + o_cnt);
    corr = reinterpret_cast<long long*>(b + o_corr);
    payload = reinterpret_cast<int32_t*>(b + o_pay);
    plan = reinterpret_cast<aem_ep_peer_plan*>(b + o_plan);
    groups = reinterpret_cast<int32_t*>(b + o_groups);
    pair_local = reinterpret_cast<int32_t*>(b + o_pl);
    st = reinterpret_cast<StepState*>(b + o_st);
    idx_pos = reinterpret_cast<int32_t*>(b + o_ipos);
    pos_of = reinterpret_cast<int32_t*>(b + o_pos);
    expert_at = reinterpret_cast<int32_t*>(b + o_exp);
    xu = b + o_xu;
    hu = b + o_hu;
    ret_acc = reinterpret_cast<float*>(b + o_ret);
    std::vector<int32_t> at(E);
    for (int e = 0; e < E; ++e) at[h_pos[e]] = e;
    AEM_TRY_CUDA(cudaMemcpy(pos_of, h_pos.data(), sizeof(int32_t) * E, cudaMemcpyHostToDevice));
    AEM_TRY_CUDA(cudaMemcpy(expert_at, at.data(), sizeof(int32_t) * E, cudaMemcpyHostToDevice));
    AEM_TRY_CUDA(cudaMallocHost(&h_suspect, sizeof(unsigned long long)));
    AEM_TRY_CUDA(cudaStreamCreateWithFlags(&aux, cudaStreamNonBlocking));
    for (cudaEvent_t* e : {&ev_plan, &ev_disp_b, &ev_down_a, &ev_ret_a})
        AEM_TRY_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    return AEM_OK;
}

// All-gathers every rank's IPC handle, device and sizes; maps every peer's region.
aem_status Ep::map_peers(cudaStream_t s) {
    const int R = world;
    struct Record {
        cudaIpcMemHandle_t h;
        int64_t bytes, T_cap, d, f, E, k, placement;
        uint8_t uuid[16];
        uint8_t pad[256 - sizeof(cudaIpcMemHandle_t) - 7 * sizeof(int64_t) - 16];
    };
    static_assert(sizeof(Record) == 256, "record size");
    Record mine{};
    AEM_TRY_CUDA(cudaIpcGetMemHandle(&mine.h, xreg));
    mine.bytes = static_cast<int64_t>(lay.bytes);
    mine.T_cap = T_cap;
    mine.d = cfg.d_model;
    mine.f = cfg.d_ffn;
    mine.E = cfg.num_experts;
    mine.k = cfg.top_k;
    uint64_t hsh = 1469598103934665603ull;  // FNV-1a of the placement
    for (int32_t p : h_pos) hsh = (hsh ^ static_cast<uint32_t>(p)) * 1099511628211ull;
    mine.placement = static_cast<int64_t>(hsh);
    cudaDeviceProp prop;
    AEM_TRY_CUDA(cudaGetDeviceProperties(&prop, device));
    memcpy(mine.uuid, &prop.uuid, 16);
    void* dev = nullptr;
    AEM_TRY_CUDA(cudaMalloc(&dev, sizeof(Record) * R));
    std::vector<Record> all(R);
    aem_status st_ = AEM_OK;
    do {
        cudaError_t e = cudaMemcpyAsync(static_cast<char*>(dev) + sizeof(Record) * rank, &mine,
                                        sizeof(Record), cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) {
            set_error("aem_ep_create: %s", cudaGetErrorString(e));
            st_ = AEM_ECUDA;
            break;
        }
        ncclResult_t n = nccl()->AllGather(static_cast<char*>(dev) + sizeof(Record) * rank, dev,
                                           sizeof(Record), ncclUint8, comm, s);
        if (n != ncclSuccess) {
            set_error("aem_ep_create: handle all-gather failed: %s", nccl()->GetErrorString(n));
            st_ = AEM_ENCCL;
            break;
        }
        e = cudaMemcpyAsync(all.data(), dev, sizeof(Record) * R, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) {
            set_error("aem_ep_create: %s", cudaGetErrorString(e));
            st_ = AEM_ECUDA;
        }
    } while (0);
    cudaFree(dev);
    if (st_ != AEM_OK) return st_;
    for (int r = 0; r < R; ++r) {
        const Record& a = all[r];
        AEM_REQUIRE(a.bytes == mine.bytes && a.T_cap == mine.T_cap && a.d == mine.d &&
                        a.f == mine.f && a.E == mine.E && a.k == mine.k &&
                        a.placement == mine.placement,
                    "aem_ep_create: rank %d has a different config, placement or "
                    "max_tokens_local", r);
        for (int q = 0; q < r; ++q)
            AEM_REQUIRE(memcmp(all[q].uuid, a.uuid, 16) != 0,
                        "aem_ep_create: ranks %d and %d share one GPU (one rank per GPU)", q, r);
    }
    peers.base[rank] = static_cast<char*>(xreg);
    for (int r = 0; r < R; ++r) {
        if (r == rank) continue;
        void* p = nullptr;
        AEM_TRY_CUDA(cudaIpcOpenMemHandle(&p, all[r].h, cudaIpcMemLazyEnablePeerAccess));
        peers.base[r] = static_cast<char*>(p);
        mapped[r] = true;
    }
    return AEM_OK;
}

void Ep::release() {
    for (int r = 0; r < world; ++r)
        if (mapped[r]) {
            cudaIpcCloseMemHandle(peers.base[r]);
            mapped[r] = false;
        }
}

aem_status Ep::forward(const void* x, aem_dtype xd, int64_t T, void* out, aem_dtype od,
                       uint8_t* unit_failed, bool tolerant, cudaStream_t s) {
    const int k = cfg.top_k, E = cfg.num_experts, R = world, el = e_loc;
    const int ksel = k < E ? k + 1 : k;
    const int64_t d = cfg.d_model, f = cfg.d_ffn, U = T * k;
    AEM_REQUIRE(T <= T_cap, "aem_ep_forward: T_local=%lld > max_tokens_local=%lld", (long long)T,
                (long long)T_cap);
    const uint64_t live = (all_mask() & ~unhealthy) | (1ull << rank);
    if (!tolerant && live != all_mask()) {
        set_error("aem_ep_forward: rank(s) 0x%llx are unhealthy; aem_ep_forward_tolerant "
                  "routes around them",
                  static_cast<unsigned long long>(all_mask() & ~live));
        return AEM_ETIMEOUT;
    }
    const int dev = current_device();
    const int sms = sm_count(dev);
    int* err = device_error_word(dev);
    AEM_REQUIRE(err != nullptr, "aem_ep_forward: no device error word");
    const int tol = tolerant ? 1 : 0;
    StepTimer timer(AEM_METRIC_EP_STEP, s);
    const uint64_t q = ++seq;
    const size_t plan_smem = plan_block_smem(R, E, pay_ld);
    if (plan_smem > 48 * 1024)
        AEM_TRY_CUDA(cudaFuncSetAttribute(ep_plan_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(plan_smem)));
    char* mine = static_cast<char*>(xreg);
    const uint64_t* flags = reinterpret_cast<const uint64_t*>(mine + lay.flags);
    last_T = T;
    AEM_TRY_CUDA(cudaMemsetAsync(&st->failed, 0, sizeof(int), s));
    // 1. gating and local per-(slot, expert) counts
    prof.begin(AEM_PHASE_GATING, s);
    if (T > 0)
        AEM_TRY(launch_gating(*gate, x, xd, T, k, ksel, cfg.gating_mode, loc.idx, loc.val, s));
    const int32_t* ridx = loc.idx;  // routing works on placement positions
    if (placed && T > 0) {
        const unsigned g = static_cast<unsigned>(std::min<int64_t>((T * ksel + 255) / 256, 1024));
        relabel_kernel<<<g, 256, 0, s>>>(loc.idx, T * ksel, pos_of, idx_pos);
        AEM_CHECK_LAUNCH();
        count_launches(1);
        ridx = idx_pos;
    }
    prof.end(AEM_PHASE_GATING, s);
    prof.begin(AEM_PHASE_EXCHANGE, s);
    AEM_TRY_CUDA(cudaMemsetAsync(cnt, 0, sizeof(unsigned long long) * k * E, s));
    if (T > 0) {
        const unsigned g = static_cast<unsigned>(std::min<int64_t>((U + 255) / 256, 1024));
        slot_count_kernel<<<g, 256, sizeof(unsigned) * k * E, s>>>(ridx, T, ksel, k, E, cnt);
        AEM_CHECK_LAUNCH();
        count_launches(1);
    }
    // 2. all-gather counts -> global rank offsets
    ep_publish_kernel<<<1, 256, 0, s>>>(reinterpret_cast<const uint32_t*>(cnt), 2 * k * E, 2 * k * E,
                                        peers, lay.mail_cnt, lay.flags, SYNC_COUNTS, rank, R, live,
                                        q, st);
    AEM_CHECK_LAUNCH();
    ep_corr_kernel<<<1, 256, 0, s>>>(reinterpret_cast<const long long*>(mine + lay.mail_cnt),
                                     flags + SYNC_COUNTS * R, R, k, E, rank, live, q, timeout_ns,
                                     tol, st, err, corr);
    AEM_CHECK_LAUNCH();
    count_launches(2);
    prof.end(AEM_PHASE_EXCHANGE, s);
    // 3. capacity routing with global ranks + expert-grouped permutation
    //    (half A's units first inside every expert), then the
    //    (destination, token) pairs
    // two-half pipeline: off unless asked for (at 2 and 4 ranks of a
    // 16384-token batch the halves' smaller GEMMs and the pushes' SMs beside
    // them cost more than the hidden transfers save)
    const bool split = pipeline > 0;
    const int64_t half_T = split ? (T + 1) / 2 : T;
    prof.begin(AEM_PHASE_ROUTE, s);
    if (T > 0) {
        MoeRouteArgs ra;
        ra.idx = ridx;
        ra.T = T;
        ra.ldi = ksel;
        ra.k = k;
        ra.E = E;
        ra.capacity = cfg.capacity;
        ra.val = loc.val;
        ra.corr = reinterpret_cast<const int64_t*>(corr);
        ra.workspace = loc.route_ws;
        ra.eff_out = loc.eff;
        ra.starts_out = loc.starts;
        ra.src_token = loc.src_token;
        ra.rowmap = loc.rowmap;
        ra.rowscale = loc.rowscale;
        ra.half_T = half_T;
        AEM_TRY(route_moe(ra, s));
    } else {
        AEM_TRY_CUDA(cudaMemsetAsync(loc.starts, 0, sizeof(int) * (E + 1), s));
    }
    ep_pairs_kernel<<<R, 1024, 0, s>>>(loc.eff, T, half_T, k, el, E, R, live, loc.starts,
                                       pair_local, payload);
    AEM_CHECK_LAUNCH();
    count_launches(1);
    prof.end(AEM_PHASE_ROUTE, s);
    // 4. all-gather every rank's payload; every rank plans on the device
    prof.begin(AEM_PHASE_EXCHANGE, s);
    ep_publish_kernel<<<1, 256, 0, s>>>(reinterpret_cast<const uint32_t*>(payload), pay_ld, pay_ld,
                                        peers, lay.mail_pay, lay.flags, SYNC_PLAN, rank, R, live, q,
                                        st);
    AEM_CHECK_LAUNCH();
    ep_plan_kernel<<<1, 256, plan_smem, s>>>(
        reinterpret_cast<const int32_t*>(mine + lay.mail_pay), pay_ld, flags + SYNC_PLAN * R, R,
        E, rank, live, q, timeout_ns, tol, units_cap, pairs_cap, ret_cap, st, plan, groups, err);
    AEM_CHECK_LAUNCH();
    count_launches(2);
    prof.end(AEM_PHASE_EXCHANGE, s);
    // 5-7. two-half pipeline: half B's dispatch (second stream) runs under
    //    half A's GEMMs, half A's return (second stream) under half B's GEMMs
    const int32_t* cnt_a = payload + pay_units_a(E, R);
    auto dispatch = [&](int half, cudaStream_t st_) -> aem_status {
        const unsigned g = static_cast<unsigned>(sms * 4);
        if (xd == AEM_BF16)
            ep_dispatch_kernel<__nv_bfloat16><<<g, kCopyThreads, 0, st_>>>(
                static_cast<const __nv_bfloat16*>(x), T, half_T, half, d, R, el, pair_local,
                loc.starts, cnt_a, loc.src_token, loc.rowscale, k, plan, peers, lay, units_cap,
                pairs_cap, err);
        else
            ep_dispatch_kernel<float><<<g, kCopyThreads, 0, st_>>>(
                static_cast<const float*>(x), T, half_T, half, d, R, el, pair_local, loc.starts,
                cnt_a, loc.src_token, loc.rowscale, k, plan, peers, lay, units_cap, pairs_cap,
                err);
        AEM_CHECK_LAUNCH();
        ep_publish_kernel<<<1, 64, 0, st_>>>(nullptr, 0, 0, peers, 0, lay.flags,
                                             half ? SYNC_DISPATCH_B : SYNC_DISPATCH_A, rank, R,
                                             live, q, st);
        AEM_CHECK_LAUNCH();
        count_launches(2);
        return AEM_OK;
    };
    auto receive = [&](int half) -> aem_status {
        ep_wait_kernel<<<1, 64, 0, s>>>(flags + (half ? SYNC_DISPATCH_B : SYNC_DISPATCH_A) * R, R,
                                        rank, live, q, timeout_ns, tol, st, err);
        AEM_CHECK_LAUNCH();
        ep_expand_kernel<<<static_cast<unsigned>(sms * 4), kCopyThreads, 0, s>>>(
            reinterpret_cast<const __nv_bfloat16*>(mine + lay.xpair),
            reinterpret_cast<int32_t*>(mine + lay.rowmap),
            reinterpret_cast<float*>(mine + lay.rowscale), plan, st, half, R, d,
            static_cast<__nv_bfloat16*>(xu), ret_acc, err);
        AEM_CHECK_LAUNCH();
        count_launches(2);
        return AEM_OK;
    };
    // local expert FFN of one half, one row group per local expert; the down
    // GEMM scales by the gate weight and sums the units of each pair
    auto ffn = [&](int half) -> aem_status {
        const int64_t hint = std::max<int64_t>(U / 2, 1);  // expected received units
        GemmArgs up_a;
        up_a.w = up;
        up_a.G = el;
        up_a.group_rows = groups + half * (el + 1);
        up_a.M = units_cap;
        up_a.max_rows = units_cap;
        up_a.rows_hint = hint;
        up_a.x_hi = xu;
        up_a.out = hu;
        up_a.out_bf16 = true;
        up_a.ldo = f;
        up_a.relu = true;
        prof.begin(AEM_PHASE_UP, s);
        AEM_TRY(launch_qgemm(up_a, s));
        prof.end(AEM_PHASE_UP, s);
        GemmArgs dn;
        dn.w = down;
        dn.G = el;
        dn.group_rows = groups + half * (el + 1);
        dn.M = units_cap;
        dn.max_rows = units_cap;
        dn.rows_hint = hint;
        dn.x_hi = hu;
        dn.out = ret_acc;
        dn.ldo = d;
        dn.atomic_add = true;
        dn.rowmap = reinterpret_cast<const int32_t*>(mine + lay.rowmap);
        dn.rowscale = reinterpret_cast<const float*>(mine + lay.rowscale);
        prof.begin(AEM_PHASE_DOWN, s);
        AEM_TRY(launch_qgemm(dn, s));
        prof.end(AEM_PHASE_DOWN, s);
        return AEM_OK;
    };
    auto give_back = [&](int half, cudaStream_t st_) -> aem_status {
        const unsigned g = static_cast<unsigned>(sms * 4);
        ep_return_kernel<<<g, kCopyThreads, 0, st_>>>(
            ret_acc, plan, st, half, R, rank, d, peers, lay, ret_cap, err);
        AEM_CHECK_LAUNCH();
        ep_publish_kernel<<<1, 64, 0, st_>>>(nullptr, 0, 0, peers, 0, lay.flags,
                                             half ? SYNC_RETURN_B : SYNC_RETURN_A, rank, R, live,
                                             q, st);
        AEM_CHECK_LAUNCH();
        count_launches(2);
        return AEM_OK;
    };
    prof.begin(AEM_PHASE_DISPATCH, s);
    AEM_TRY(dispatch(0, s));
    if (split) {
        // half B's pushes start once half A's are out, under half A's receive and GEMMs
        AEM_TRY_CUDA(cudaEventRecord(ev_plan, s));
        AEM_TRY_CUDA(cudaStreamWaitEvent(aux, ev_plan, 0));
        AEM_TRY(dispatch(1, aux));
        AEM_TRY_CUDA(cudaEventRecord(ev_disp_b, aux));
    }
    AEM_TRY(receive(0));
    prof.end(AEM_PHASE_DISPATCH, s);
    AEM_TRY(ffn(0));
    if (split) {
        AEM_TRY_CUDA(cudaEventRecord(ev_down_a, s));
        AEM_TRY_CUDA(cudaStreamWaitEvent(aux, ev_down_a, 0));
        AEM_TRY(give_back(0, aux));  // half A's sums go back under half B's GEMMs
        AEM_TRY_CUDA(cudaEventRecord(ev_ret_a, aux));
        prof.begin(AEM_PHASE_DISPATCH, s);
        AEM_TRY_CUDA(cudaStreamWaitEvent(s, ev_disp_b, 0));  // this rank's own half-B pushes
        AEM_TRY(receive(1));
        prof.end(AEM_PHASE_DISPATCH, s);
        AEM_TRY(ffn(1));
    }
    prof.begin(AEM_PHASE_RETURN, s);
    if (split) {
        AEM_TRY(give_back(1, s));
        AEM_TRY_CUDA(cudaStreamWaitEvent(s, ev_ret_a, 0));  // joins the second stream
        ep_wait_kernel<<<1, 64, 0, s>>>(flags + SYNC_RETURN_B * R, R, rank, live, q, timeout_ns,
                                        tol, st, err);
        AEM_CHECK_LAUNCH();
        count_launches(1);
    } else {
        AEM_TRY(give_back(0, s));
    }
    ep_wait_kernel<<<1, 64, 0, s>>>(flags + SYNC_RETURN_A * R, R, rank, live, q, timeout_ns, tol,
                                    st, err);
    AEM_CHECK_LAUNCH();
    count_launches(1);
    prof.end(AEM_PHASE_RETURN, s);
    // 8. per-token sum over destination ranks, failed flags
    prof.begin(AEM_PHASE_COMBINE, s);
    if (T > 0) {
        const float* ret_in = reinterpret_cast<const float*>(mine + lay.ret);
        const unsigned g = static_cast<unsigned>(std::min<int64_t>((T + 7) / 8, sms * 8));
        if (od == AEM_BF16)
            ep_combine_kernel<__nv_bfloat16><<<g, kCopyThreads, 0, s>>>(
                ret_in, ret_acc, pair_local, plan, st, loc.eff, k, el, live, T, R, rank, d,
                static_cast<__nv_bfloat16*>(out), unit_failed);
        else
            ep_combine_kernel<float><<<g, kCopyThreads, 0, s>>>(
                ret_in, ret_acc, pair_local, plan, st, loc.eff, k, el, live, T, R, rank, d,
                static_cast<float*>(out), unit_failed);
        AEM_CHECK_LAUNCH();
        count_launches(1);
    }
    prof.end(AEM_PHASE_COMBINE, s);
    prof.step();
    return AEM_OK;
}

}  // namespace aem

using aem::set_error;

extern "C" {

aem_status aem_ep_plan_bases(const int64_t* counts, int R, int k, int E, int rank, int64_t* base) {
    AEM_REQUIRE(counts && base, "aem_ep_plan_bases: NULL buffer");
    AEM_REQUIRE(R >= 1 && k >= 1 && E >= 1 && rank >= 0 && rank < R,
                "aem_ep_plan_bases: bad R=%d k=%d E=%d rank=%d", R, k, E, rank);
    for (int e = 0; e < E; ++e) {
        int64_t before_slots = 0;
        for (int j = 0; j < k; ++j) {
            int64_t before_ranks = 0, slot_total = 0;
            for (int r = 0; r < R; ++r) {
                const int64_t v = counts[(static_cast<int64_t>(r) * k + j) * E + e];
                if (r < rank) before_ranks += v;
                slot_total += v;
            }
            base[j * E + e] = before_slots + before_ranks;
            before_slots += slot_total;
        }
    }
    return AEM_OK;
}

aem_status aem_ep_plan_exchange(const int32_t* starts, int R, int E, int rank, int64_t* send_off,
                                int64_t* send_cnt, int64_t* recv_off, int64_t* recv_cnt,
                                int32_t* groups) {
    AEM_REQUIRE(starts && send_off && send_cnt && recv_off && recv_cnt && groups,
                "aem_ep_plan_exchange: NULL buffer");
    AEM_REQUIRE(R >= 1 && E >= R && E % R == 0 && rank >= 0 && rank < R,
                "aem_ep_plan_exchange: bad R=%d E=%d rank=%d", R, E, rank);
    const int e_loc = E / R;
    const int32_t* my = starts + static_cast<int64_t>(rank) * (E + 1);
    int64_t rtot = 0;
    groups[0] = 0;
    for (int p = 0; p < R; ++p) {
        send_off[p] = my[p * e_loc];
        send_cnt[p] = my[(p + 1) * e_loc] - my[p * e_loc];
        const int32_t* ps = starts + static_cast<int64_t>(p) * (E + 1);
        recv_off[p] = rtot;
        for (int e = 0; e < e_loc; ++e) {
            const int64_t c = ps[rank * e_loc + e + 1] - ps[rank * e_loc + e];
            AEM_REQUIRE(c >= 0, "aem_ep_plan_exchange: rank %d's expert starts decrease", p);
            rtot += c;
            groups[p * e_loc + e + 1] = static_cast<int32_t>(rtot);
        }
        recv_cnt[p] = rtot - recv_off[p];
    }
    return AEM_OK;
}

aem_status aem_ep_plan_peer(const int32_t* all, int R, int E, int rank, uint64_t live,
                            int64_t units_cap, int64_t pairs_cap, int64_t ret_cap,
                            aem_ep_peer_plan* plan, int32_t* groups) {
    AEM_REQUIRE(all && plan && groups, "aem_ep_plan_peer: NULL buffer");
    AEM_REQUIRE(R >= 1 && R <= AEM_EP_MAX_RANKS && E >= R && E % R == 0 && rank >= 0 && rank < R,
                "aem_ep_plan_peer: bad R=%d E=%d rank=%d", R, E, rank);
    aem::plan_peer(all, AEM_EP_PAYLOAD(E, R), R, E, rank, live, units_cap, pairs_cap, ret_cap, plan,
                   groups);
    return AEM_OK;
}

aem_status aem_ep_plan_peer_device(const int32_t* all, int R, int E, int rank, uint64_t live,
                                   int64_t units_cap, int64_t pairs_cap, int64_t ret_cap,
                                   aem_ep_peer_plan* plan, int32_t* groups, void* stream) {
    AEM_REQUIRE(all && plan && groups, "aem_ep_plan_peer_device: NULL buffer");
    AEM_REQUIRE(R >= 1 && R <= AEM_EP_MAX_RANKS && E >= R && E % R == 0 && E <= AEM_MAX_EXPERTS &&
                    rank >= 0 && rank < R,
                "aem_ep_plan_peer_device: bad R=%d E=%d rank=%d", R, E, rank);
    const size_t smem = aem::plan_block_smem(R, E, AEM_EP_PAYLOAD(E, R));
    if (smem > 48 * 1024)
        AEM_TRY_CUDA(cudaFuncSetAttribute(aem::ep_plan_test_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem)));
    aem::ep_plan_test_kernel<<<1, 256, smem, static_cast<cudaStream_t>(stream)>>>(
        all, R, E, rank, live, units_cap, pairs_cap, ret_cap, plan, groups);
    AEM_CHECK_LAUNCH();
    aem::count_launches(1);
    return AEM_OK;
}

aem_status aem_ep_unique_id(uint8_t out[128]) {
    AEM_REQUIRE(out != nullptr, "aem_ep_unique_id: out is NULL");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    AEM_NCCL_OR_FAIL();
    ncclUniqueId id;
    AEM_TRY_NCCL(::aem::nccl()->GetUniqueId(&id));
    memcpy(out, &id, 128);
    return AEM_OK;
}

static void ep_destroy(aem::Ep* ep, bool abort_comm) {
    ep->release();
    if (ep->comm && aem::nccl()) {
        if (abort_comm)
            aem::nccl()->CommAbort(ep->comm);
        else
            aem::nccl()->CommDestroy(ep->comm);
    }
    cudaFree(ep->xreg);
    cudaFree(ep->lbuf);
    cudaFree(ep->loc.buf);
    cudaFreeHost(ep->h_suspect);
    if (ep->aux) cudaStreamDestroy(ep->aux);
    for (cudaEvent_t e : {ep->ev_plan, ep->ev_disp_b, ep->ev_down_a, ep->ev_ret_a})
        if (e) cudaEventDestroy(e);
    delete ep;
}

aem_status aem_ep_create(const aem_moe_config* cfg, int rank, int world, const uint8_t uid[128],
                         aem_gate_t gate, aem_qweight_t up_local, aem_qweight_t down_local,
                         const int32_t* expert_to_rank, int64_t max_tokens_local, aem_ep_t* out) {
    AEM_REQUIRE(out != nullptr, "aem_ep_create: out is NULL");
    *out = nullptr;
    AEM_REQUIRE(cfg && uid && gate && up_local && down_local, "aem_ep_create: NULL argument");
    AEM_REQUIRE(world >= 1 && world <= AEM_EP_MAX_RANKS && rank >= 0 && rank < world,
                "aem_ep_create: bad rank %d / world %d (at most %d ranks)", rank, world,
                AEM_EP_MAX_RANKS);
    AEM_REQUIRE(cfg->num_experts % world == 0,
                "aem_ep_create: num_experts=%d not divisible by world=%d", cfg->num_experts, world);
    AEM_REQUIRE(max_tokens_local >= 1, "aem_ep_create: max_tokens_local must be >= 1");
    AEM_REQUIRE(cfg->d_model % 8 == 0, "aem_ep_create: d_model=%lld must be a multiple of 8",
                (long long)cfg->d_model);
    auto* g = reinterpret_cast<aem::Gate*>(gate);
    auto* u = reinterpret_cast<aem::QWeight*>(up_local);
    auto* dn = reinterpret_cast<aem::QWeight*>(down_local);
    const int e_loc = cfg->num_experts / world;
    AEM_REQUIRE(cfg->top_k >= 1 && cfg->top_k <= AEM_MAX_TOPK && cfg->top_k <= cfg->num_experts,
                "aem_ep_create: bad top_k");
    AEM_REQUIRE(g->E == cfg->num_experts && g->D == cfg->d_model, "aem_ep_create: gate shape");
    AEM_REQUIRE(u->G == e_loc && u->K == cfg->d_model && u->N == cfg->d_ffn,
                "aem_ep_create: up weight must hold the %d local experts [%lld -> %lld]", e_loc,
                (long long)cfg->d_model, (long long)cfg->d_ffn);
    AEM_REQUIRE(dn->G == e_loc && dn->K == cfg->d_ffn && dn->N == cfg->d_model,
                "aem_ep_create: down weight shape");
    std::vector<int32_t> pos(cfg->num_experts);
    bool placed = false;
    {
        std::vector<int> fill(world, 0);
        for (int e = 0; e < cfg->num_experts; ++e) {
            const int r = expert_to_rank ? expert_to_rank[e] : e / e_loc;
            AEM_REQUIRE(r >= 0 && r < world, "aem_ep_create: expert_to_rank[%d]=%d outside [0, %d)",
                        e, r, world);
            AEM_REQUIRE(fill[r] < e_loc, "aem_ep_create: rank %d is given more than %d experts", r,
                        e_loc);
            pos[e] = r * e_loc + fill[r]++;
            placed |= pos[e] != e;
        }
    }
    AEM_NCCL_OR_FAIL();
    auto* ep = new aem::Ep();
    ep->h_pos = pos;
    ep->placed = placed;
    ep->cfg = *cfg;
    ep->rank = rank;
    ep->world = world;
    ep->device = g->device;
    ep->e_loc = e_loc;
    ep->gate = g;
    ep->up = u;
    ep->down = dn;
    ep->loc.cfg = *cfg;
    ep->loc.gate = g;
    ep->loc.up = u;
    ep->loc.down = dn;
    cudaSetDevice(g->device);
    ncclUniqueId id;
    memcpy(&id, uid, 128);
    ncclResult_t r = ::aem::nccl()->CommInitRank(&ep->comm, world, id, rank);
    if (r != ncclSuccess) {
        set_error("aem_ep_create: ncclCommInitRank failed: %s", ::aem::nccl()->GetErrorString(r));
        delete ep;
        return AEM_ENCCL;
    }
    aem_status st = ep->init(max_tokens_local);
    if (st == AEM_OK) {
        cudaStream_t s = nullptr;
        if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) {
            set_error("aem_ep_create: cudaStreamCreate failed");
            st = AEM_ECUDA;
        } else {
            st = ep->map_peers(s);
            cudaStreamDestroy(s);
        }
    }
    if (st != AEM_OK) {
        ep_destroy(ep, true);
        return st;
    }
    *out = reinterpret_cast<aem_ep_t>(ep);
    return AEM_OK;
}

aem_status aem_ep_free(aem_ep_t h) {
    if (!h) return AEM_OK;
    auto* ep = reinterpret_cast<aem::Ep*>(h);
    cudaSetDevice(ep->device);
    cudaDeviceSynchronize();
    unsigned long long suspect = 0;
    cudaMemcpy(&suspect, &ep->st->suspect, sizeof(suspect), cudaMemcpyDeviceToHost);
    const bool healthy = ep->unhealthy == 0 && suspect == 0;
    aem_status st = AEM_OK;
    if (healthy) {
        // Collective: nobody unmaps or frees until every rank's last step
        // ended, and nobody frees its region while a peer still maps it.
        int* bar = &ep->st->bar;
        cudaStream_t s = nullptr;
        if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess) {
            ncclResult_t n = aem::nccl()->AllReduce(bar, bar, 1, ncclInt32, ncclSum, ep->comm, s);
            if (n == ncclSuccess) cudaStreamSynchronize(s);
            ep->release();
            if (n == ncclSuccess)
                n = aem::nccl()->AllReduce(bar, bar, 1, ncclInt32, ncclSum, ep->comm, s);
            if (n == ncclSuccess) cudaStreamSynchronize(s);
            if (n != ncclSuccess) {
                set_error("aem_ep_free: %s", aem::nccl()->GetErrorString(n));
                st = AEM_ENCCL;
            }
            cudaStreamDestroy(s);
        }
    }
    // With a rank gone there is no collective to wait on: unmap, free, abort.
    ep_destroy(ep, !healthy || st != AEM_OK);
    return st;
}

static aem_status ep_forward_checked(aem_ep_t h, const void* x, aem_dtype x_dtype, int64_t T_local,
                                     void* out, aem_dtype out_dtype, uint8_t* unit_failed,
                                     bool tolerant, void* stream) {
    AEM_REQUIRE(h != nullptr, "aem_ep_forward: NULL layer");
    AEM_REQUIRE(T_local >= 0 && T_local < (1ll << 28), "aem_ep_forward: T out of range");
    AEM_REQUIRE(T_local == 0 || (x && out), "aem_ep_forward: NULL buffer");
    AEM_REQUIRE(x_dtype == AEM_F32 || x_dtype == AEM_BF16, "aem_ep_forward: bad x dtype");
    AEM_REQUIRE(out_dtype == AEM_F32 || out_dtype == AEM_BF16, "aem_ep_forward: bad out dtype");
    auto* ep = reinterpret_cast<aem::Ep*>(h);
    return ep->forward(x, x_dtype, T_local, out, out_dtype, unit_failed, tolerant,
                       static_cast<cudaStream_t>(stream));
}

aem_status aem_ep_forward(aem_ep_t h, const void* x, aem_dtype x_dtype, int64_t T_local, void* out,
                          aem_dtype out_dtype, void* stream) {
    return ep_forward_checked(h, x, x_dtype, T_local, out, out_dtype, nullptr, false, stream);
}

aem_status aem_ep_forward_tolerant(aem_ep_t h, const void* x, aem_dtype x_dtype, int64_t T_local,
                                   void* out, aem_dtype out_dtype, uint8_t* unit_failed,
                                   void* stream) {
    return ep_forward_checked(h, x, x_dtype, T_local, out, out_dtype, unit_failed, true, stream);
}

aem_status aem_ep_forward_host(aem_context_t ctx, aem_ep_t h, const void* x, aem_dtype x_dtype,
                               int64_t T_local, void* out, aem_dtype out_dtype) {
    AEM_REQUIRE(ctx != nullptr && h != nullptr, "aem_ep_forward_host: NULL argument");
    AEM_REQUIRE(T_local >= 0 && T_local < (1ll << 28), "aem_ep_forward_host: T out of range");
    AEM_REQUIRE(T_local == 0 || (x && out), "aem_ep_forward_host: NULL buffer");
    auto* c = reinterpret_cast<aem::Context*>(ctx);
    auto* ep = reinterpret_cast<aem::Ep*>(h);
    AEM_TRY_CUDA(cudaSetDevice(c->device));
    const int64_t d = ep->cfg.d_model;
    const size_t xb = static_cast<size_t>(T_local) * d * (x_dtype == AEM_F32 ? 4 : 2);
    const size_t ob = static_cast<size_t>(T_local) * d * (out_dtype == AEM_F32 ? 4 : 2);
    const size_t o1 = aem::align_up(xb, 256);
    AEM_TRY(c->reserve_device(o1 + ob + 256));
    char* dv = static_cast<char*>(c->dev);
    if (xb) AEM_TRY_CUDA(cudaMemcpyAsync(dv, x, xb, cudaMemcpyHostToDevice, c->stream));
    AEM_TRY(ep_forward_checked(h, dv, x_dtype, T_local, dv + o1, out_dtype, nullptr, false,
                               c->stream));
    if (ob) AEM_TRY_CUDA(cudaMemcpyAsync(out, dv + o1, ob, cudaMemcpyDeviceToHost, c->stream));
    return aem::check_device_errors(c->stream, "aem_ep_forward_host");
}

aem_status aem_ep_submit_host(aem_context_t ctx, aem_ep_t h, const void* x, aem_dtype x_dtype,
                              int64_t T_local, void* out, aem_dtype out_dtype, uint64_t* ticket) {
    AEM_REQUIRE(ctx != nullptr && h != nullptr && ticket != nullptr,
                "aem_ep_submit_host: NULL argument");
    AEM_REQUIRE(T_local >= 1 && T_local < (1ll << 28), "aem_ep_submit_host: T out of range");
    AEM_REQUIRE(x && out, "aem_ep_submit_host: NULL buffer");
    AEM_REQUIRE(x_dtype == AEM_F32 || x_dtype == AEM_BF16, "aem_ep_submit_host: bad x dtype");
    AEM_REQUIRE(out_dtype == AEM_F32 || out_dtype == AEM_BF16, "aem_ep_submit_host: bad out dtype");
    auto* c = reinterpret_cast<aem::Context*>(ctx);
    auto* ep = reinterpret_cast<aem::Ep*>(h);
    const int64_t d = ep->cfg.d_model;
    const size_t xb = static_cast<size_t>(T_local) * d * (x_dtype == AEM_F32 ? 4 : 2);
    const size_t ob = static_cast<size_t>(T_local) * d * (out_dtype == AEM_F32 ? 4 : 2);
    return aem::pipe_submit(
        c, x, xb, out, ob,
        [&](const void* din, void* dout, cudaStream_t s) {
            return ep_forward_checked(h, din, x_dtype, T_local, dout, out_dtype, nullptr, false, s);
        },
        ticket);
}

aem_status aem_ep_mark_unhealthy(aem_ep_t h, int rank) {
    AEM_REQUIRE(h != nullptr, "aem_ep_mark_unhealthy: NULL layer");
    auto* ep = reinterpret_cast<aem::Ep*>(h);
    AEM_REQUIRE(rank >= 0 && rank < ep->world, "aem_ep_mark_unhealthy: bad rank %d", rank);
    AEM_REQUIRE(rank != ep->rank, "aem_ep_mark_unhealthy: rank %d is this rank", rank);
    ep->unhealthy |= 1ull << rank;
    return AEM_OK;
}

aem_status aem_ep_health(aem_ep_t h, uint64_t* unhealthy, void* stream) {
    AEM_REQUIRE(h != nullptr && unhealthy != nullptr, "aem_ep_health: NULL argument");
    auto* ep = reinterpret_cast<aem::Ep*>(h);
    auto s = static_cast<cudaStream_t>(stream);
    AEM_TRY_CUDA(cudaMemcpyAsync(ep->h_suspect, &ep->st->suspect, sizeof(unsigned long long),
                                 cudaMemcpyDeviceToHost, s));
    AEM_TRY_CUDA(cudaStreamSynchronize(s));
    ep->unhealthy |= *ep->h_suspect & ~(1ull << ep->rank);
    *unhealthy = ep->unhealthy;
    return AEM_OK;
}

aem_status aem_ep_set_pipeline(aem_ep_t h, int mode) {
    AEM_REQUIRE(h != nullptr, "aem_ep_set_pipeline: NULL layer");
    AEM_REQUIRE(mode >= -1 && mode <= 1, "aem_ep_set_pipeline: mode %d not in {-1, 0, 1}", mode);
    reinterpret_cast<aem::Ep*>(h)->pipeline = mode;
    return AEM_OK;
}

aem_status aem_ep_set_timeout(aem_ep_t h, double seconds) {
    AEM_REQUIRE(h != nullptr, "aem_ep_set_timeout: NULL layer");
    AEM_REQUIRE(seconds > 0.0 && seconds <= 3600.0, "aem_ep_set_timeout: %g s out of range",
                seconds);
    reinterpret_cast<aem::Ep*>(h)->timeout_ns = static_cast<uint64_t>(seconds * 1e9);
    return AEM_OK;
}

aem_status aem_ep_profile(aem_ep_t h, int enable) {
    AEM_REQUIRE(h != nullptr, "aem_ep_profile: NULL layer");
    reinterpret_cast<aem::Ep*>(h)->prof.enable(enable != 0);
    return AEM_OK;
}

aem_status aem_ep_profile_read(aem_ep_t h, double* ms, int64_t* steps) {
    AEM_REQUIRE(h != nullptr, "aem_ep_profile_read: NULL layer");
    return reinterpret_cast<aem::Ep*>(h)->prof.read(ms, steps);
}

aem_status aem_ep_last_routing(aem_ep_t h, int32_t* idx, float* val, uint32_t* effective,
                               void* stream) {
    AEM_REQUIRE(h != nullptr, "aem_ep_last_routing: NULL layer");
    auto* ep = reinterpret_cast<aem::Ep*>(h);
    auto s = static_cast<cudaStream_t>(stream);
    const int64_t T = ep->last_T;
    if (T == 0) return AEM_OK;
    const int k = ep->cfg.top_k;
    const int ksel = k < ep->cfg.num_experts ? k + 1 : k;
    if (idx)
        AEM_TRY_CUDA(cudaMemcpyAsync(idx, ep->loc.idx, sizeof(int32_t) * T * ksel,
                                     cudaMemcpyDeviceToDevice, s));
    if (val)
        AEM_TRY_CUDA(cudaMemcpyAsync(val, ep->loc.val, sizeof(float) * T * k,
                                     cudaMemcpyDeviceToDevice, s));
    if (effective) {
        if (ep->placed) {
            const unsigned g = static_cast<unsigned>(std::min<int64_t>((T * k + 255) / 256, 1024));
            aem::unlabel_kernel<<<g, 256, 0, s>>>(ep->loc.eff, T * k, ep->expert_at, effective);
            AEM_CHECK_LAUNCH();
            aem::count_launches(1);
        } else {
            AEM_TRY_CUDA(cudaMemcpyAsync(effective, ep->loc.eff, sizeof(uint32_t) * T * k,
                                         cudaMemcpyDeviceToDevice, s));
        }
    }
    return AEM_OK;
}

}  // extern "C"
