// Shared host/device infrastructure of the AetherMoE B200 library:
// thread-local error reporting, status macros, the per-device error word that
// kernels report failed in-kernel checks and bounded-wait timeouts into, and
// inline-PTX wrappers for mbarriers, TMA and tcgen05 (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "aem.h"

namespace aem {

// ---------------------------------------------------------------- errors
void set_error(const char* fmt, ...);
void clear_error();

#define AEM_TRY_CUDA(expr)                                                              \
    do {                                                                                \
        cudaError_t aem_e_ = (expr);                                                    \
        if (aem_e_ != cudaSuccess) {                                                    \
            ::aem::set_error("%s:%d: %s failed: %s", __FILE__, __LINE__, #expr,         \
                             cudaGetErrorString(aem_e_));                               \
            return aem_e_ == cudaErrorMemoryAllocation ? AEM_ENOMEM : AEM_ECUDA;        \
        }                                                                               \
    } while (0)

#define AEM_REQUIRE(cond, ...)                                                          \
    do {                                                                                \
        if (!(cond)) {                                                                  \
            ::aem::set_error(__VA_ARGS__);                                              \
            return AEM_EINVAL;                                                          \
        }                                                                               \
    } while (0)

#define AEM_TRY(expr)                                                                   \
    do {                                                                                \
        aem_status aem_s_ = (expr);                                                     \
        if (aem_s_ != AEM_OK) return aem_s_;                                            \
    } while (0)

// Launch-error check right after a <<<>>> launch.
#define AEM_CHECK_LAUNCH() AEM_TRY_CUDA(cudaGetLastError())

// Bits of the per-device error word.
enum : int {
    ERR_ROUTE_POSITION = 1 << 0,  // batch_position not a permutation of [0, n)
    ERR_ROUTE_EXPERT = 1 << 1,    // expert id >= E
    ERR_GEMM_TIMEOUT = 1 << 2,    // a bounded mbarrier wait in the GEMM gave up
    ERR_GEMM_GROUPS = 1 << 3,     // group table inconsistent
    ERR_EP_PLAN = 1 << 4,         // expert-parallel counts do not fit the receive buffers
    ERR_EP_BOUNDS = 1 << 5,       // expert-parallel row index outside its buffer (skipped)
    ERR_EP_PEER_TIMEOUT = 1 << 6, // a peer rank did not signal within the deadline
    ERR_EP_PEER_FAILED = 1 << 7,  // a peer rank signalled that its step failed
};


// Device int that kernels atomicOr error bits into (one per device, lazily
// allocated, zero-initialised).  Returns nullptr on allocation failure.
int* device_error_word(int device);
// Synchronises `stream`, reads and clears the error word of the current
// device; returns AEM_EDEVICE / AEM_ETIMEOUT with a message if bits were set.
aem_status check_device_errors(cudaStream_t stream, const char* what);

int current_device();
int sm_count(int device);
bool is_sm100(int device);

// ---------------------------------------------------------------- TMA descriptors
// 2-D tiled tensor map over a row-major [rows, cols] matrix (cols innermost).
aem_status make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                        int elem_bytes, uint64_t cols, uint64_t rows, uint32_t box_cols,
                        uint32_t box_rows, CUtensorMapSwizzle swizzle);

}  // namespace aem

// ================================================================ device side
#ifdef __CUDACC__
namespace aem {
namespace dev {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Vector float32 reduction into global memory (16-byte aligned address).
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
                 "f"(d)
                 : "memory");
}

// System-scope acquire load / release store (flags written by peer GPUs).
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// ---- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with `parity` of `bar` to complete.  Gives up
// after `limit_ns` of wall time or as soon as `*abort` is set, records `code`
// in the error word and sets `*abort`; returns false then.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort, int* err, int code,
                                                  uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > limit_ns) {
            *abort = 1;
            atomicOr(err, code);
            return false;
        }
    }
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- TMA (no multicast anywhere in this library)
__device__ __forceinline__ void tma_prefetch_desc(const void* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const void* map, uint64_t* bar, int x,
                                            int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Non-tensor bulk copy global -> shared (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 in, f32 accumulate).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16: A is M = 128 rows in the
// 128 TMEM lanes (row m in lane m), K along the columns, two bf16 per 32-bit
// column (even K in the low half); one K = 16 step spans 8 columns.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Thread i of the warp writes lane (warp's lane base + i), columns [col, col+32).
__device__ __forceinline__ void tc_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tc_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// Arrive (once) on `bar` when all previously issued tcgen05 ops of this thread complete.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tc_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane
// (warp's lane base + i), columns [col, col+32).
__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
        "[%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
// 32 lanes x 16 columns.
__device__ __forceinline__ void tc_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

// ---- thread-block clusters and the tcgen05 SM pair (cta_group::2)
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// All threads of every CTA of the cluster (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared::cluster address of the object at `local`'s offset in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_u32(const void* local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
    return r;
}
// One arrival on the mbarrier at `local_twin`'s offset in CTA `rank` of the
// cluster (the default release semantics, as for a local arrival).
__device__ __forceinline__ void mbar_arrive_remote(const uint64_t* local_twin, uint32_t rank) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(mapa_u32(local_twin, rank))
                 : "memory");
}
// TMA 2-D tile load into this CTA's shared memory whose completion (bytes)
// is counted on the mbarrier at `bar_local_twin`'s offset in CTA `bar_rank`
// of this CTA's tcgen05 pair (no multicast).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* map,
                                                 const uint64_t* bar_local_twin,
                                                 uint32_t bar_rank, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(mapa_u32(bar_local_twin, bar_rank)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void st_remote_u32(const void* local_twin, uint32_t rank, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(mapa_u32(local_twin, rank)), "r"(v)
                 : "memory");
}
// try_wait with acquire at cluster scope (the phase is completed by arrivals
// from another CTA of the cluster).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
// D[tmem of both CTAs] (+)= A[smem of both] * B[smem, N split over the pair]^T,
// issued in the pair's even CTA by one elected lane of a warp that runs the
// issue loop together (its operands then stay warp-uniform).
__device__ __forceinline__ void tc_mma_f16_pair_elect(uint32_t d_tmem, uint64_t a_desc,
                                                      uint64_t b_desc, uint32_t idesc,
                                                      uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive (once) on the mbarrier at `bar`'s offset in every CTA of `cta_mask`
// when all tcgen05 ops previously issued by the elected lane complete (the
// lane that issued the MMAs: elect.sync picks the lowest active lane every
// time).
__device__ __forceinline__ void tc_commit_pair_elect(uint64_t* bar, uint16_t cta_mask) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "h"(cta_mask)
        : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored in the
// 128-byte-swizzle layout: rows of 128 bytes (64 bf16 along K), 8-row atoms
// of 1024 bytes stacked contiguously (stride byte offset 1024).  Fields:
// start address >> 4 in [0,14), leading byte offset (16 B units; 1 for
// swizzled K-major) in [16,30), stride byte offset >> 4 in [32,46),
// descriptor version 1 in [46,48), layout SWIZZLE_128B (2) in [61,64).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= 1ull << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= 1ull << 46;
    d |= 2ull << 61;
    return d;
}

// Instruction descriptor of kind::f16: bf16 A and B (K-major), f32 D,
// M = 128, N = n (multiple of 16, 16..256).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(uint32_t m, uint32_t n) {
    return (1u << 4)              // D format f32
           | (1u << 7)            // A format bf16
           | (1u << 10)           // B format bf16
           | ((n >> 3) << 17)     // N >> 3
           | ((m >> 4) << 24);    // M >> 4
}

}  // namespace dev

}  // namespace aem
#endif  // __CUDACC__
