// Expert-parallel MoE layer over NCCL (one process per GPU, NVLink/NVSwitch).
//
// Replaces the reference's Router scatter/gather over ICollectiveTransport
// (src/orchestration/router.hpp:67-100, collective_transport.hpp:37-51): the
// routing decision stays Router::assign_effective_experts (router.hpp:249-266)
// and is bit-exact with a single-process run over the global batch, because
// every rank ranks its units by GLOBAL batch_position:
//   units are (token, slot) pairs in slot-major order, u = j*T + t_global, and
//   rank r owns tokens [r*T_l, (r+1)*T_l); so in expert e's group the units of
//   slot j on rank r come after all units of slots < j (every rank) and after
//   slot j of ranks < r.  One all-gather of per-(slot, expert) counts gives
//   each rank that offset; local stable ranks do the rest.
// Step: gating -> slot counts -> all-gather -> capacity routing (global ranks)
// -> expert-grouped send buffer -> all-gather of per-expert send counts (the
// one host sync: NCCL needs sizes) -> grouped send/recv dispatch -> local
// grouped GEMMs on the received (source, expert) segments -> send/recv of the
// float32 expert outputs back -> weighted combine in token order.
#include <cuda_bf16.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <mutex>
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
    decltype(&::ncclAllGather) AllGather = nullptr;
    decltype(&::ncclGroupStart) GroupStart = nullptr;
    decltype(&::ncclGroupEnd) GroupEnd = nullptr;
    decltype(&::ncclSend) Send = nullptr;
    decltype(&::ncclRecv) Recv = nullptr;
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
        sym(g_nccl.AllGather, "ncclAllGather");
        sym(g_nccl.GroupStart, "ncclGroupStart");
        sym(g_nccl.GroupEnd, "ncclGroupEnd");
        sym(g_nccl.Send, "ncclSend");
        sym(g_nccl.Recv, "ncclRecv");
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

namespace {

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

// corr[j][e] = base[j][e] - (local units of expert e in slots < j), where
// base[j][e] = sum_{j'<j} sum_r' all[r'][j'][e] + sum_{r'<r} all[r'][j][e].
__global__ void ep_corr_kernel(const long long* __restrict__ all, int R, int k, int E, int rank,
                               long long* __restrict__ corr) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        long long before_slots = 0, local_before = 0;
        for (int j = 0; j < k; ++j) {
            long long before_ranks = 0, slot_total = 0;
            for (int r = 0; r < R; ++r) {
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

// out[t] = sum_j val[t,j] * y[dest_of[j*T + t]]  (j in increasing order).
template <typename OT>
__global__ void combine_gather_kernel(const float* __restrict__ y, const int32_t* __restrict__ dest_of,
                                      const float* __restrict__ val, int64_t T, int k, int64_t d,
                                      OT* __restrict__ out) {
    const int64_t total = T * d;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / d, c = i % d;
        float acc = 0.0f;
        for (int j = 0; j < k; ++j) {
            const int64_t row = dest_of[static_cast<int64_t>(j) * T + t];
            acc += val[t * k + j] * y[row * d + c];
        }
        if constexpr (sizeof(OT) == 2)
            out[i] = __float2bfloat16_rn(acc);
        else
            out[i] = acc;
    }
}

ncclDataType_t nccl_dtype(int bytes) { return bytes == 2 ? ncclBfloat16 : ncclFloat32; }

}  // namespace

struct Ep {
    aem_moe_config cfg{};
    int rank = 0, world = 1, device = 0, e_loc = 0;
    ncclComm_t comm = nullptr;
    Gate* gate = nullptr;
    QWeight* up = nullptr;
    QWeight* down = nullptr;
    Moe loc;  // local buffers (routing, send rows) of the single-GPU layer
    // collective scratch
    unsigned long long* cnt = nullptr;  // [k][E]
    long long* cnt_all = nullptr;       // [R][k][E]
    long long* corr = nullptr;          // [k][E]
    int* starts_all = nullptr;          // [R][E+1]
    int32_t* dest_of = nullptr;         // [U]
    int* h_starts = nullptr;            // pinned [R][E+1]
    int* h_groups = nullptr;            // pinned [R*e_loc+1]
    int* d_groups = nullptr;            // [R*e_loc+1]
    int64_t u_cap = 0;                  // capacity of dest_of
    // receive side (grow-only)
    int64_t r_cap = 0;
    void* xr = nullptr;   // bf16 [r_cap, d]
    void* hr = nullptr;   // bf16 [r_cap, ffn]
    float* yr = nullptr;  // f32 [r_cap, d]
    float* yb = nullptr;  // f32 [u_cap, d] expert outputs back in grouped order
    int64_t last_T = 0;
    PhaseProfiler prof;

    aem_status init_buffers();
    aem_status reserve_units(int64_t U);
    aem_status reserve_recv(int64_t rows);
    aem_status forward(const void* x, aem_dtype xd, int64_t T, void* out, aem_dtype od,
                       cudaStream_t s);
};

aem_status Ep::init_buffers() {
    const int k = cfg.top_k, E = cfg.num_experts, R = world;
    AEM_TRY_CUDA(cudaMalloc(&cnt, sizeof(unsigned long long) * k * E));
    AEM_TRY_CUDA(cudaMalloc(&cnt_all, sizeof(long long) * R * k * E));
    AEM_TRY_CUDA(cudaMalloc(&corr, sizeof(long long) * k * E));
    AEM_TRY_CUDA(cudaMalloc(&starts_all, sizeof(int) * R * (E + 1)));
    AEM_TRY_CUDA(cudaMalloc(&d_groups, sizeof(int) * (R * e_loc + 1)));
    AEM_TRY_CUDA(cudaMallocHost(&h_starts, sizeof(int) * R * (E + 1)));
    AEM_TRY_CUDA(cudaMallocHost(&h_groups, sizeof(int) * (R * e_loc + 1)));
    return AEM_OK;
}

aem_status Ep::reserve_units(int64_t U) {
    if (U <= u_cap) return AEM_OK;
    AEM_TRY_CUDA(cudaDeviceSynchronize());
    cudaFree(dest_of);
    cudaFree(yb);
    dest_of = nullptr;
    yb = nullptr;
    AEM_TRY_CUDA(cudaMalloc(&dest_of, sizeof(int32_t) * U));
    AEM_TRY_CUDA(cudaMalloc(&yb, sizeof(float) * U * cfg.d_model));
    u_cap = U;
    return AEM_OK;
}

aem_status Ep::reserve_recv(int64_t rows) {
    if (rows <= r_cap) return AEM_OK;
    AEM_TRY_CUDA(cudaDeviceSynchronize());
    cudaFree(xr);
    cudaFree(hr);
    cudaFree(yr);
    xr = hr = nullptr;
    yr = nullptr;
    const int64_t want = rows + rows / 4 + 256;
    AEM_TRY_CUDA(cudaMalloc(&xr, 2 * want * cfg.d_model));
    AEM_TRY_CUDA(cudaMalloc(&hr, 2 * want * cfg.d_ffn));
    AEM_TRY_CUDA(cudaMalloc(&yr, sizeof(float) * want * cfg.d_model));
    r_cap = want;
    return AEM_OK;
}

aem_status Ep::forward(const void* x, aem_dtype xd, int64_t T, void* out, aem_dtype od,
                       cudaStream_t s) {
    const int k = cfg.top_k, E = cfg.num_experts, R = world;
    const int ksel = k < E ? k + 1 : k;
    const int64_t d = cfg.d_model, f = cfg.d_ffn, U = T * k;
    last_T = T;
    AEM_TRY(loc.reserve(std::max<int64_t>(T, 1)));
    AEM_TRY(reserve_units(std::max<int64_t>(U, 1)));
    // 1. gating and local per-(slot, expert) counts
    prof.begin(AEM_PHASE_GATING, s);
    if (T > 0)
        AEM_TRY(launch_gating(*gate, x, xd, T, k, ksel, cfg.gating_mode, loc.idx, loc.val, s));
    prof.end(AEM_PHASE_GATING, s);
    prof.begin(AEM_PHASE_EXCHANGE, s);
    AEM_TRY_CUDA(cudaMemsetAsync(cnt, 0, sizeof(unsigned long long) * k * E, s));
    if (T > 0) {
        const unsigned g = static_cast<unsigned>(std::min<int64_t>((U + 255) / 256, 1024));
        slot_count_kernel<<<g, 256, sizeof(unsigned) * k * E, s>>>(loc.idx, T, ksel, k, E, cnt);
        AEM_CHECK_LAUNCH();
        count_launches(1);
    }
    // 2. all-gather counts -> global rank offsets
    AEM_TRY_NCCL(::aem::nccl()->AllGather(cnt, cnt_all, static_cast<size_t>(k) * E, ncclInt64, comm, s));
    ep_corr_kernel<<<1, 256, 0, s>>>(cnt_all, R, k, E, rank, corr);
    AEM_CHECK_LAUNCH();
    count_launches(1);
    prof.end(AEM_PHASE_EXCHANGE, s);
    // 3. capacity routing with global ranks + expert-grouped permutation
    prof.begin(AEM_PHASE_ROUTE, s);
    if (T > 0) {
        MoeRouteArgs ra;
        ra.idx = loc.idx;
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
        ra.dest_of = dest_of;
        AEM_TRY(route_moe(ra, s));
        AEM_TRY(gather_rows(x, xd, loc.src_token, U, d, loc.xperm, s));
    } else {
        AEM_TRY_CUDA(cudaMemsetAsync(loc.starts, 0, sizeof(int) * (E + 1), s));
    }
    prof.end(AEM_PHASE_ROUTE, s);
    // 4. all-gather per-expert starts; sizes to the host (the one sync)
    AEM_TRY_NCCL(::aem::nccl()->AllGather(loc.starts, starts_all, static_cast<size_t>(E + 1), ncclInt32, comm, s));
    AEM_TRY_CUDA(cudaMemcpyAsync(h_starts, starts_all, sizeof(int) * R * (E + 1),
                                 cudaMemcpyDeviceToHost, s));
    AEM_TRY_CUDA(cudaStreamSynchronize(s));
    std::vector<int64_t> send_off(R), send_cnt(R), recv_off(R), recv_cnt(R);
    AEM_TRY(aem_ep_plan_exchange(h_starts, R, E, rank, send_off.data(), send_cnt.data(),
                                 recv_off.data(), recv_cnt.data(), h_groups));
    const int64_t rtot = recv_off[R - 1] + recv_cnt[R - 1];
    AEM_TRY(reserve_recv(std::max<int64_t>(rtot, 1)));
    AEM_TRY_CUDA(cudaMemcpyAsync(d_groups, h_groups, sizeof(int) * (R * e_loc + 1),
                                 cudaMemcpyHostToDevice, s));
    // 5. dispatch: bf16 rows, grouped by destination rank, to the expert owners
    prof.begin(AEM_PHASE_DISPATCH, s);
    AEM_TRY_NCCL(::aem::nccl()->GroupStart());
    for (int p = 0; p < R; ++p) {
        if (send_cnt[p] > 0)
            AEM_TRY_NCCL(::aem::nccl()->Send(static_cast<char*>(loc.xperm) + 2 * send_off[p] * d,
                                  send_cnt[p] * d, ncclBfloat16, p, comm, s));
        if (recv_cnt[p] > 0)
            AEM_TRY_NCCL(::aem::nccl()->Recv(static_cast<char*>(xr) + 2 * recv_off[p] * d, recv_cnt[p] * d,
                                  ncclBfloat16, p, comm, s));
    }
    AEM_TRY_NCCL(::aem::nccl()->GroupEnd());
    prof.end(AEM_PHASE_DISPATCH, s);
    // 6. local expert FFN on the (source, expert) segments
    if (rtot > 0) {
        GemmArgs up_a;
        up_a.w = up;
        up_a.G = R * e_loc;
        up_a.wmod = e_loc;
        up_a.group_rows = d_groups;
        up_a.M = rtot;
        up_a.max_rows = rtot;
        up_a.x_hi = xr;
        up_a.out = hr;
        up_a.out_bf16 = true;
        up_a.ldo = f;
        up_a.relu = true;
        prof.begin(AEM_PHASE_UP, s);
        AEM_TRY(launch_qgemm(up_a, s));
        prof.end(AEM_PHASE_UP, s);
        GemmArgs dn;
        dn.w = down;
        dn.G = R * e_loc;
        dn.wmod = e_loc;
        dn.group_rows = d_groups;
        dn.M = rtot;
        dn.max_rows = rtot;
        dn.x_hi = hr;
        dn.out = yr;
        dn.ldo = d;
        prof.begin(AEM_PHASE_DOWN, s);
        AEM_TRY(launch_qgemm(dn, s));
        prof.end(AEM_PHASE_DOWN, s);
    }
    // 7. expert outputs back to the token owners (same segments, reversed)
    prof.begin(AEM_PHASE_RETURN, s);
    AEM_TRY_NCCL(::aem::nccl()->GroupStart());
    for (int p = 0; p < R; ++p) {
        if (recv_cnt[p] > 0)
            AEM_TRY_NCCL(::aem::nccl()->Send(yr + recv_off[p] * d, recv_cnt[p] * d, ncclFloat32, p, comm, s));
        if (send_cnt[p] > 0)
            AEM_TRY_NCCL(::aem::nccl()->Recv(yb + send_off[p] * d, send_cnt[p] * d, ncclFloat32, p, comm, s));
    }
    AEM_TRY_NCCL(::aem::nccl()->GroupEnd());
    prof.end(AEM_PHASE_RETURN, s);
    // 8. weighted combine in token order
    prof.begin(AEM_PHASE_COMBINE, s);
    if (T > 0) {
        const unsigned g = static_cast<unsigned>(std::min<int64_t>((T * d + 255) / 256, 148 * 16));
        if (od == AEM_BF16)
            combine_gather_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(
                yb, dest_of, loc.val, T, k, d, static_cast<__nv_bfloat16*>(out));
        else
            combine_gather_kernel<float><<<g, 256, 0, s>>>(yb, dest_of, loc.val, T, k, d,
                                                           static_cast<float*>(out));
        AEM_CHECK_LAUNCH();
        count_launches(1);
    }
    prof.end(AEM_PHASE_COMBINE, s);
    prof.step();
    (void)nccl_dtype;
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

aem_status aem_ep_unique_id(uint8_t out[128]) {
    AEM_REQUIRE(out != nullptr, "aem_ep_unique_id: out is NULL");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    AEM_NCCL_OR_FAIL();
    ncclUniqueId id;
    AEM_TRY_NCCL(::aem::nccl()->GetUniqueId(&id));
    memcpy(out, &id, 128);
    return AEM_OK;
}

aem_status aem_ep_create(const aem_moe_config* cfg, int rank, int world, const uint8_t uid[128],
                         aem_gate_t gate, aem_qweight_t up_local, aem_qweight_t down_local,
                         aem_ep_t* out) {
    AEM_REQUIRE(out != nullptr, "aem_ep_create: out is NULL");
    *out = nullptr;
    AEM_REQUIRE(cfg && uid && gate && up_local && down_local, "aem_ep_create: NULL argument");
    AEM_REQUIRE(world >= 1 && rank >= 0 && rank < world, "aem_ep_create: bad rank %d / world %d",
                rank, world);
    AEM_REQUIRE(cfg->num_experts % world == 0,
                "aem_ep_create: num_experts=%d not divisible by world=%d", cfg->num_experts, world);
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
    AEM_NCCL_OR_FAIL();
    auto* ep = new aem::Ep();
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
    aem_status st = ep->init_buffers();
    if (st != AEM_OK) {
        ::aem::nccl()->CommDestroy(ep->comm);
        delete ep;
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
    if (ep->comm && aem::nccl()) aem::nccl()->CommDestroy(ep->comm);
    cudaFree(ep->cnt);
    cudaFree(ep->cnt_all);
    cudaFree(ep->corr);
    cudaFree(ep->starts_all);
    cudaFree(ep->dest_of);
    cudaFree(ep->d_groups);
    cudaFree(ep->xr);
    cudaFree(ep->hr);
    cudaFree(ep->yr);
    cudaFree(ep->yb);
    cudaFree(ep->loc.buf);
    cudaFreeHost(ep->h_starts);
    cudaFreeHost(ep->h_groups);
    delete ep;
    return AEM_OK;
}

aem_status aem_ep_forward(aem_ep_t h, const void* x, aem_dtype x_dtype, int64_t T_local, void* out,
                          aem_dtype out_dtype, void* stream) {
    AEM_REQUIRE(h != nullptr, "aem_ep_forward: NULL layer");
    AEM_REQUIRE(T_local >= 0 && T_local < (1ll << 28), "aem_ep_forward: T out of range");
    AEM_REQUIRE(T_local == 0 || (x && out), "aem_ep_forward: NULL buffer");
    auto* ep = reinterpret_cast<aem::Ep*>(h);
    return ep->forward(x, x_dtype, T_local, out, out_dtype, static_cast<cudaStream_t>(stream));
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
    if (effective)
        AEM_TRY_CUDA(cudaMemcpyAsync(effective, ep->loc.eff, sizeof(uint32_t) * T * k,
                                     cudaMemcpyDeviceToDevice, s));
    return AEM_OK;
}

}  // extern "C"
