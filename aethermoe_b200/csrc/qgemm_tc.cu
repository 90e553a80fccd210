// Grouped INT8 weight-only GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
//   out[r, n] = epilogue( scale[g][n] * sum_k x[r, k] * q[g][n, k] )   for row r of group g
//
// This is the B200 form of fused_quantized_matmul (src/kernels/quantized_gemm.py:99-138,
// :184-226): weights stay INT8 in HBM and are dequantised at multiply time.  The
// multiply itself runs on the 5th-generation tensor cores, so the kernel is
// organised weights-stationary: a tile is 128 output channels (the MMA's M) by BT
// activation rows (the MMA's N, 16..256), which keeps decode-size batches (a handful
// of rows) on the tensor cores with the int8 weight stream as the only large read.
//
// Per CTA (one per SM, persistent over tiles), 19 warps and two smem rings: the
// int8 weight ring and the operand ring, whose stage holds one K step's
// activation tile and its converted bf16 weights under one full and one empty
// barrier:
//   warp 16     int8 weight producer: one contiguous 8 KB bulk copy per [128 x 64 B]
//               tile of the pre-tiled weight layout -- the HBM stream.
//   warp 18     activation producer: TMA of the bf16 [BT x 128 B] tile(s) (128-byte
//               swizzle) into the stage, arriving on its full barrier.
//   warps 0-7   converters, in groups that take K steps round-robin: int8 -> bf16
//               (exact: |q| <= 127 fits bf16's 8-bit significand) written straight
//               into the 128-byte-swizzled K-major layout the MMA reads, then
//               fence.proxy.async and one arrival per warp on the stage's full barrier.
//   warp 17     MMA issuer (one thread): one wait per K step, 4 x tcgen05.mma
//               kind::f16 (K=16 each), x2 for split float32 activations (hi + lo),
//               accumulating float32 in a double-buffered TMEM accumulator; one
//               tcgen05.commit frees the stage and, at the end of a tile, one hands
//               the accumulator over.
//   warps 8-15  epilogue, two warps per TMEM lane quarter splitting the columns:
//               tcgen05.ld 32 lanes x 16 columns, per-channel scale, per-row output
//               index and multiplier (fetched once per 16 columns, broadcast by
//               shuffles), ReLU, bf16/f32 store or red.add (split-K / fused combine).
// Every mbarrier wait is bounded (globaltimer); on timeout the kernel records an
// error bit, all roles drain out, and TMEM is released.  No multicast is used.
#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "runtime.h"

namespace aem {

aem_status launch_qgemm_simt(const GemmArgs& a, cudaStream_t s);
aem_status launch_qgemm_decode(const GemmArgs& a, cudaStream_t s);
aem_status launch_qgemm_gemv(const GemmArgs& a, cudaStream_t s);

namespace {

using namespace aem::dev;

constexpr int kCh = 128;      // output channels per tile = MMA M
constexpr int kKT = 64;       // K per stage: one 128-byte bf16 row
// Warp roles.  Converter warps come first; the epilogue warps start at a
// warpgroup boundary so that warp (kEpiWarp0 + i) owns TMEM lanes
// [32*(i%4), 32*(i%4)+32) -- two epilogue warps per lane quarter, each taking
// half of the tile's columns.
constexpr int kConvWarps = 8;
constexpr int kConvThreads = kConvWarps * 32;
// Converter warps form groups that take K steps round-robin, so several K
// steps are in conversion at once (one group's convert -> proxy fence ->
// arrive latency no longer serialises the stream of K steps).  The group
// count must not exceed the operand ring depth: a group handling K step kc
// has finished kc - G, whose wait proved K step kc - G - D retired, so with
// G <= D the slot's previous phase (kc - D) is at most one phase ahead of the
// barrier and the parity wait cannot alias an older phase.  The int8 ring's
// depth is a multiple of G, for the same reason (see Cfg::S8).
#ifndef AEM_PAIR_W16_STAGES
#define AEM_PAIR_W16_STAGES 4     // SM-pair form: converted-weight slots
#endif
#ifndef AEM_PAIR_W8_STAGES
#define AEM_PAIR_W8_STAGES 8      // SM-pair form: int8 weight slots, at least
#endif
#ifndef AEM_PAIR_X_STAGES_MAX
#define AEM_PAIR_X_STAGES_MAX 8   // SM-pair form: activation slots, at most
#endif
#ifndef AEM_QGEMM_MAX_CONV_GROUPS
#define AEM_QGEMM_MAX_CONV_GROUPS 4
#endif
constexpr int kEpiWarp0 = 8;
constexpr int kEpiWarps = 8;
constexpr int kW8Warp = 16;   // int8 weight producer
constexpr int kMmaWarp = 17;  // MMA issuer + TMEM allocation
constexpr int kXWarp = 18;    // activation producer
constexpr int kThreads = 19 * 32;
constexpr int kMmaWarpX = 19;  // further MMA issuers (TMEM weights, small token tiles)
static_assert(kEpiWarp0 % 4 == 0, "epilogue warps must start at a warpgroup boundary");
constexpr int kMaxGroups = 256;

struct TcParams {
    int G;
    int64_t group_base;
    int wmod;               // weight group of row group g: group_base + (wmod ? g % wmod : g)
    const int* group_rows;  // nullptr: one group of M rows
    int64_t M;
    int K;
    int N;
    int ksplit;
    const float* scale;     // [Gw][N]
    const int8_t* wq;       // tiled int8 weights [Gw][NT][KT][128][64]
    int64_t NT, KT;
    void* out;
    void* out_lo;           // bf16 out only: low half of a split output (nullable)
    int64_t ldo;
    int out_bf16;
    int relu;
    int atomic_add;
    int red_v4;             // atomic_add with N, ldo multiples of 4: 16-byte reductions
    int stream_k;           // split the (tile, K step) space evenly over the CTAs (atomic_add)
    const int* rowmap;
    const float* rowscale;
    int* err;
};

constexpr int pow2_cols(int c) { return c <= 32 ? 32 : c <= 64 ? 64 : c <= 128 ? 128 : c <= 256 ? 256 : 512; }

// TSA: the converted bf16 weights go to TMEM (the MMA's A operand read from
// tensor memory) instead of shared memory; the operand ring's stage then holds
// only the activation tile in shared memory, and its weights occupy a 32-column
// slot of TMEM beside the two accumulators.
template <int BT, int SPLIT, bool TSA = false, int NI = 1>
struct Cfg {
    // NI MMA-issuing warps, each with its own accumulators, take the K steps
    // round-robin: one thread issues a tcgen05.mma only every ~100 cycles
    // whatever N is, so small token tiles need several issuers to keep the
    // tensor pipe (and the weight stream) busy; the epilogue adds the NI
    // partial accumulators.
    static constexpr int THREADS = (kMmaWarpX + NI - 1) * 32;
    static constexpr int W8 = kCh * kKT;           // int8 weight tile, bytes
    static constexpr int W16 = TSA ? 0 : kCh * kKT * 2;  // bf16 weight tile in smem (MMA A)
    static constexpr int XB = BT * kKT * 2;        // bf16 activation tile (MMA B), per part
    static constexpr int XS = SPLIT * XB;          // one activation stage
    // Two rings.  A stage of the operand ring holds one K step's activation
    // tile (TMA) and its converted bf16 weights; one barrier says both are
    // in (the TMA's bytes plus one arrival per converter warp) and one
    // commit frees both, so the single MMA-issuing thread does one wait and
    // one commit per K step -- its synchronisation, not the tensor core,
    // bounded the step rate when each ring had its own barriers.  The int8
    // ring streams the weights from HBM; it gets what the operand ring
    // leaves of the budget.
    static constexpr int BUDGET = 216 * 1024;
    static constexpr int DS_RAW = (BUDGET - 8 * W8) / (W16 + XS);  // 8 int8 stages first
    static constexpr int DS_TMEM = TSA ? (512 - 2 * NI * BT) / 32 : 8;  // TMEM weight slots
    static constexpr int DS_CAP = DS_TMEM < 8 ? DS_TMEM : 8;
    static constexpr int DS_FIT = DS_RAW > DS_CAP ? DS_CAP : (DS_RAW < 2 ? 2 : DS_RAW);
    // a multiple of NI: issuer i then owns the stages s = i mod NI, and its
    // wait for K step kc follows its own wait for kc - DS (no parity aliasing)
    static constexpr int DS = (DS_FIT / NI) * NI;
    static constexpr int S8_RAW = (BUDGET - DS * (W16 + XS)) / W8;
    // converter groups: with TMEM weights a group is one warpgroup (its four
    // warps reach the four TMEM lane quarters)
    static constexpr int CG_RAW = TSA ? 2 : (DS >= 4 ? 4 : (DS >= 2 ? 2 : 1));
    static constexpr int CG = CG_RAW < AEM_QGEMM_MAX_CONV_GROUPS ? CG_RAW : AEM_QGEMM_MAX_CONV_GROUPS;
    // The int8 ring's depth is a multiple of the group count: then the
    // previous fill of the slot a group waits on (K step kc - S8) was that same
    // group's, so it has landed, and the parity wait for kc cannot mistake the
    // slot's older phase for kc's (bulk copies may land out of order, so a
    // fill owned by another group would give no such guarantee).
    static constexpr int S8 = ((S8_RAW > 12 ? 12 : S8_RAW) / CG) * CG;
    static constexpr int A_COL0 = 2 * NI * BT;     // first TMEM weight slot (TSA)
    static constexpr int TMEM_COLS = pow2_cols(2 * NI * BT + (TSA ? 32 * DS : 0));
    static constexpr int BAR_BYTES = (2 * DS + 2 * S8 + 4) * 8 + 16;
    static constexpr int TAB_BYTES = 2 * (kMaxGroups + 1) * 4;
    static constexpr int SMEM = 1024 + DS * (W16 + XS) + S8 * W8 + BAR_BYTES + TAB_BYTES;
    static constexpr int CG_WARPS = kConvWarps / CG;        // warps per converter group
    static constexpr int CG_THREADS = CG_WARPS * 32;
    static constexpr int EPI_COLS = BT >= 32 ? BT / 2 : BT;  // columns per epilogue warp
    static_assert(CG <= DS && S8 >= CG && S8 % CG == 0 && kConvWarps % CG == 0,
                  "converter groups vs rings");
    static_assert(S8 >= 2 && DS >= 2, "pipeline needs two stages per ring");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static_assert(BT % 16 == 0 && BT >= 16 && BT <= 256, "MMA N for M=128");
    static_assert(!TSA || (CG_WARPS == 4 && 2 * NI * BT + 32 * DS <= 512), "TMEM weight slots");
    static_assert(NI == 1 || (TSA && DS % NI == 0 && DS >= NI), "several issuers need TMEM weights");
};

struct TileInfo {
    int g;
    int wg;  // weight group (absolute)
    int n0;
    int64_t row0;
    int nrows;
    int kt0;
    int kt1;
};

template <int BT>
__device__ __forceinline__ TileInfo decode_tile(int t, const int* s_rows, const int* s_tiles,
                                                const TcParams& p, int nch, int nkt, int kper) {
    int lo = 0, hi = p.G;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (s_tiles[mid] <= t) lo = mid; else hi = mid;
    }
    TileInfo ti;
    ti.g = lo;
    ti.wg = static_cast<int>(p.group_base) + (p.wmod ? lo % p.wmod : lo);
    int r = t - s_tiles[lo];
    const int cnt = s_rows[lo + 1] - s_rows[lo];
    const int ntc = (cnt + BT - 1) / BT;
    const int tc = r % ntc;
    r /= ntc;
    const int ks = r % p.ksplit;
    const int nc = r / p.ksplit;
    ti.n0 = nc * kCh;
    ti.row0 = static_cast<int64_t>(s_rows[lo]) + static_cast<int64_t>(tc) * BT;
    ti.nrows = min(BT, cnt - tc * BT);
    ti.kt0 = ks * kper;
    ti.kt1 = min(nkt, ti.kt0 + kper);
    (void)nch;
    return ti;
}

// The work of one CTA, item by item: whole tiles round-robin (tile t =
// blockIdx.x + i * gridDim.x, each over its K range), or, with stream-K, an
// equal contiguous share of the flattened (tile, K step) space -- a share may
// start or end inside a tile, whose partial sums the epilogue then adds into
// the zeroed output -- so every CTA streams the same number of weight tiles.
struct WorkCursor {
    int t;
    int64_t w, w1;
};
__device__ __forceinline__ WorkCursor work_begin(const TcParams& p, int total, int nkt) {
    WorkCursor c;
    c.t = blockIdx.x;
    const int64_t units = static_cast<int64_t>(total) * nkt;
    c.w = p.stream_k ? units * blockIdx.x / gridDim.x : 0;
    c.w1 = p.stream_k ? units * (blockIdx.x + 1) / gridDim.x : 0;
    return c;
}
template <int BT>
__device__ __forceinline__ bool work_next(WorkCursor& c, TileInfo& ti, const int* s_rows,
                                          const int* s_tiles, const TcParams& p, int total,
                                          int nch, int nkt, int kper) {
    if (!p.stream_k) {
        if (c.t >= total) return false;
        ti = decode_tile<BT>(c.t, s_rows, s_tiles, p, nch, nkt, kper);
        c.t += gridDim.x;
        return true;
    }
    if (c.w >= c.w1) return false;
    const int t = static_cast<int>(c.w / nkt);
    const int k0 = static_cast<int>(c.w % nkt);
    const int k1 = static_cast<int>(min(static_cast<int64_t>(nkt), k0 + (c.w1 - c.w)));
    ti = decode_tile<BT>(t, s_rows, s_tiles, p, nch, nkt, nkt);  // ksplit is 1 here
    ti.kt0 = k0;
    ti.kt1 = k1;
    c.w += k1 - k0;
    return true;
}

// Two floats rounded to bf16 (nearest even), packed: `lo` in the low half,
// the lower address of the pair in memory.
__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// 4 signed bytes -> 2 words of bf16x2 (exact).  Each byte b becomes the float
// 2^23 + (b + 128) by byte permutation, minus (2^23 + 128); the bf16 is the
// float's upper half (integers |b| <= 128 have no low mantissa bits).
__device__ __forceinline__ uint2 i8x4_to_bf16x4(uint32_t v) {
    const uint32_t u = v ^ 0x80808080u;
    const float2 m = make_float2(-8388736.0f, -8388736.0f);  // two subtractions per packed op
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

template <int BT, int SPLIT, bool TSA, int NI>
__global__ void __launch_bounds__(Cfg<BT, SPLIT, TSA, NI>::THREADS, 1)
    qgemm_tc_kernel(const __grid_constant__ CUtensorMap tm_xh,
                    const __grid_constant__ CUtensorMap tm_xl, const TcParams p) {
    using C = Cfg<BT, SPLIT, TSA, NI>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* w16_ring = smem;                          // DS x bf16 W (MMA A, 128B swizzle)
    uint8_t* x_ring = w16_ring + C::DS * C::W16;       // DS x [X hi | X lo] (MMA B)
    uint8_t* w8_ring = x_ring + C::DS * C::XS;         // S8 x int8 W
    uint64_t* st_full = reinterpret_cast<uint64_t*>(w8_ring + C::S8 * C::W8);
    uint64_t* st_empty = st_full + C::DS;
    uint64_t* w8_full = st_empty + C::DS;
    uint64_t* w8_empty = w8_full + C::S8;
    uint64_t* accf_bar = w8_empty + C::S8;  // [2]
    uint64_t* acce_bar = accf_bar + 2;      // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce_bar + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* s_rows = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(st_full) + C::BAR_BYTES);
    int* s_tiles = s_rows + (kMaxGroups + 1);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;

    // ---- setup: barriers, group table, TMEM
    if (tid == 0) {
        for (int s = 0; s < C::DS; ++s) {
            // the activation producer's arrive.expect_tx + one arrival per converter warp
            mbar_init(&st_full[s], C::CG_WARPS + 1);
            mbar_init(&st_empty[s], 1);
        }
        for (int s = 0; s < C::S8; ++s) {
            mbar_init(&w8_full[s], 1);
            mbar_init(&w8_empty[s], C::CG_WARPS);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accf_bar[b], NI);  // one commit per issuer
            mbar_init(&acce_bar[b], kEpiWarps);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    for (int i = tid; i <= p.G; i += C::THREADS)
        s_rows[i] = p.group_rows ? p.group_rows[i] : (i == 0 ? 0 : static_cast<int>(p.M));
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == kXWarp && lane == 0) {
        tma_prefetch_desc(&tm_xh);
        if (SPLIT == 2) tma_prefetch_desc(&tm_xl);
    }
    const int nch = (p.N + kCh - 1) / kCh;
    const int nkt = (p.K + kKT - 1) / kKT;
    const int kper = (nkt + p.ksplit - 1) / p.ksplit;
    __syncthreads();
    if (tid == 0) {
        int acc = 0;
        bool bad = false;
        for (int g = 0; g < p.G; ++g) {
            s_tiles[g] = acc;
            const int cnt = s_rows[g + 1] - s_rows[g];
            if (cnt < 0) bad = true;
            acc += (cnt > 0 ? (cnt + BT - 1) / BT : 0) * nch * p.ksplit;
        }
        s_tiles[p.G] = acc;
        if (bad) {
            atomicOr(p.err, ERR_GEMM_GROUPS);
            s_tiles[p.G] = 0;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = s_tiles[p.G];

    if (warp == kW8Warp) {
        // ================= int8 weight producer (HBM stream)
        if (lane == 0) {
            int s8 = 0;
            uint32_t ph8 = 0;
            bool ok = true;
            TileInfo ti;
            for (WorkCursor wc = work_begin(p, total, nkt);
                 ok && !*abort_flag && work_next<BT>(wc, ti, s_rows, s_tiles, p, total, nch, nkt, kper);) {
                // the tile's 8 KB blocks along K are consecutive in the tiled layout
                const int8_t* wsrc =
                    p.wq + ((static_cast<int64_t>(ti.wg) * p.NT + ti.n0 / kCh) * p.KT) * (kCh * kKT);
                for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
                    if (!mbar_wait_bounded(&w8_empty[s8], ph8 ^ 1, abort_flag, p.err,
                                           ERR_GEMM_TIMEOUT)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&w8_full[s8], C::W8);
                    bulk_load(w8_ring + s8 * C::W8, wsrc + static_cast<int64_t>(kt) * C::W8, C::W8,
                              &w8_full[s8]);
                    if (++s8 == C::S8) {
                        s8 = 0;
                        ph8 ^= 1;
                    }
                }
            }
        }
    } else if (warp == kXWarp) {
        // ================= activation producer
        if (lane == 0) {
            int sx = 0;
            uint32_t phx = 0;
            bool ok = true;
            TileInfo ti;
            for (WorkCursor wc = work_begin(p, total, nkt);
                 ok && !*abort_flag && work_next<BT>(wc, ti, s_rows, s_tiles, p, total, nch, nkt, kper);) {
                for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
                    if (!mbar_wait_bounded(&st_empty[sx], phx ^ 1, abort_flag, p.err,
                                           ERR_GEMM_TIMEOUT)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = x_ring + sx * C::XS;
                    mbar_arrive_expect_tx(&st_full[sx], C::XS);
                    tma_load_2d(st, &tm_xh, &st_full[sx], kt * kKT, static_cast<int>(ti.row0));
                    if (SPLIT == 2)
                        tma_load_2d(st + C::XB, &tm_xl, &st_full[sx], kt * kKT,
                                    static_cast<int>(ti.row0));
                    if (++sx == C::DS) {
                        sx = 0;
                        phx ^= 1;
                    }
                }
            }
        }
    } else if (warp == kMmaWarp || (warp >= kMmaWarpX && warp < kMmaWarpX + NI - 1)) {
        // ================= MMA issuer ii of NI: K steps kc = ii mod NI, into
        // accumulator (b, ii) at TMEM columns (b * NI + ii) * BT
        if (lane == 0) {
            const int ii = warp == kMmaWarp ? 0 : warp - kMmaWarpX + 1;
            uint32_t kc = 0;  // K steps so far, in the order every role walks them
            int it = 0;
            bool ok = true;
            TileInfo ti;
            for (WorkCursor wc = work_begin(p, total, nkt);
                 ok && !*abort_flag && work_next<BT>(wc, ti, s_rows, s_tiles, p, total, nch, nkt, kper);
                 ++it) {
                const int b = it & 1;
                const uint32_t aph = (it >> 1) & 1;
                // every issuer waits, even one without K steps in this tile:
                // its commit below then cannot count toward the buffer's
                // previous tile
                if (!mbar_wait_bounded(&acce_bar[b], aph ^ 1, abort_flag, p.err, ERR_GEMM_TIMEOUT))
                    break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>((b * NI + ii) * BT);
                // a group's last tile may hold fewer rows: the MMA's N covers
                // only those (a multiple of 16), the rest of the slot is unused
                const int n_eff = min(BT, (ti.nrows + 15) & ~15);
                const uint32_t idesc = idesc_bf16_f32(kCh, static_cast<uint32_t>(n_eff));
                bool first = true;
                for (int kt = ti.kt0; kt < ti.kt1; ++kt, ++kc) {
                    if (NI > 1 && static_cast<int>(kc % NI) != ii) continue;
                    const int ss = static_cast<int>(kc % C::DS);
                    const uint32_t phs = (kc / C::DS) & 1;
                    // activations and converted weights of this K step are in
                    if (!mbar_wait_bounded(&st_full[ss], phs, abort_flag, p.err, ERR_GEMM_TIMEOUT)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bdesc = smem_desc_sw128(smem_u32(x_ring + ss * C::XS));
                    const uint64_t ldesc = smem_desc_sw128(smem_u32(x_ring + ss * C::XS + C::XB));
                    if constexpr (TSA) {
                        // weights in TMEM slot ss: 8 columns per UMMA_K=16 step
                        const uint32_t a_tmem =
                            tmem_base + static_cast<uint32_t>(C::A_COL0 + 32 * ss);
#pragma unroll
                        for (int kk = 0; kk < kKT / 16; ++kk) {
                            tc_mma_f16_ts(d_tmem, a_tmem + 8 * kk, bdesc + 2 * kk, idesc,
                                          (!first || kk > 0) ? 1u : 0u);
                            if (SPLIT == 2)
                                tc_mma_f16_ts(d_tmem, a_tmem + 8 * kk, ldesc + 2 * kk, idesc, 1u);
                        }
                    } else {
                        const uint64_t adesc = smem_desc_sw128(smem_u32(w16_ring + ss * C::W16));
#pragma unroll
                        for (int kk = 0; kk < kKT / 16; ++kk) {
                            // +32 bytes along K per UMMA_K=16 step (start address field, >>4)
                            tc_mma_f16(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc,
                                       (!first || kk > 0) ? 1u : 0u);
                            if (SPLIT == 2)
                                tc_mma_f16(d_tmem, adesc + 2 * kk, ldesc + 2 * kk, idesc, 1u);
                        }
                    }
                    // the stage is free once these MMAs retire
                    tc_commit(&st_empty[ss]);
                    first = false;
                }
                if (!ok) break;
                tc_commit(&accf_bar[b]);
            }
        }
    } else if (warp < kConvWarps) {
        // ================= converters: int8 [128 x 64B] -> bf16 SW128 [128 x 128B]
        const int group = warp / C::CG_WARPS;
        const int gtid = tid % C::CG_THREADS;
        uint32_t kc = 0;  // K steps so far, in the order every role walks them
        bool ok = true;
        TileInfo ti;
        for (WorkCursor wc = work_begin(p, total, nkt);
             ok && !*abort_flag && work_next<BT>(wc, ti, s_rows, s_tiles, p, total, nch, nkt, kper);) {
            for (int kt = ti.kt0; kt < ti.kt1; ++kt, ++kc) {
                if (static_cast<int>(kc % C::CG) != group) continue;
                const int s16 = static_cast<int>(kc % C::DS);
                const uint32_t ph16 = (kc / C::DS) & 1;
                const int s8 = static_cast<int>(kc % C::S8);
                const uint32_t ph8 = (kc / C::S8) & 1;
                // int8 tile landed, and the bf16 slot is free (its last MMA retired)
                if (!mbar_wait_bounded(&w8_full[s8], ph8, abort_flag, p.err, ERR_GEMM_TIMEOUT) ||
                    !mbar_wait_bounded(&st_empty[s16], ph16 ^ 1, abort_flag, p.err,
                                       ERR_GEMM_TIMEOUT)) {
                    ok = false;
                    break;
                }
                const uint8_t* w8 = w8_ring + s8 * C::W8;
                if constexpr (TSA) {
                    // thread = one channel row = its TMEM lane: the row's 64 int8
                    // (4 chunks, logical K order) -> 32 bf16x2 columns of slot s16
                    tc_fence_after();  // after the MMAs that last read the slot
                    const int r = 32 * (warp & 3) + lane;
                    uint4 v[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        v[c] = *reinterpret_cast<const uint4*>(w8 + r * 64 + wtile_chunk(r, c) * 16);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&w8_empty[s8]);
                    uint32_t a[32];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint32_t wv[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const uint2 o = i8x4_to_bf16x4(wv[e]);
                            a[8 * c + 2 * e] = o.x;
                            a[8 * c + 2 * e + 1] = o.y;
                        }
                    }
                    tc_st_32x32b_x32(tmem_base + (static_cast<uint32_t>(32 * (warp & 3)) << 16) +
                                         static_cast<uint32_t>(C::A_COL0 + 32 * s16),
                                     a);
                    tc_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&st_full[s16]);
                    continue;
                }
                uint8_t* st = w16_ring + s16 * C::W16;
#pragma unroll
                for (int i = 0; i < 512 / C::CG_THREADS; ++i) {
                    const int item = gtid + C::CG_THREADS * i;  // 128 rows x 4 chunks
                    const int r = item >> 2;
                    const int ch = item & 3;
                    const uint4 v =
                        *reinterpret_cast<const uint4*>(w8 + r * 64 + wtile_chunk(r, ch) * 16);
                    const uint2 a0 = i8x4_to_bf16x4(v.x);
                    const uint2 a1 = i8x4_to_bf16x4(v.y);
                    const uint2 a2 = i8x4_to_bf16x4(v.z);
                    const uint2 a3 = i8x4_to_bf16x4(v.w);
                    uint8_t* row = st + r * 128;
                    const int sw = r & 7;
                    *reinterpret_cast<uint4*>(row + (((2 * ch) ^ sw) << 4)) =
                        make_uint4(a0.x, a0.y, a1.x, a1.y);
                    *reinterpret_cast<uint4*>(row + (((2 * ch + 1) ^ sw) << 4)) =
                        make_uint4(a2.x, a2.y, a3.x, a3.y);
                }
                // make this thread's generic-proxy stores visible to the tensor core,
                // then one arrival per warp
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&st_full[s16]);
                    mbar_arrive(&w8_empty[s8]);
                }
            }
        }
    } else if (warp < kEpiWarp0 + kEpiWarps) {
        // ================= epilogue: warp kEpiWarp0+i owns TMEM lanes of quarter q = i%4
        // and columns [h*EPI_COLS, (h+1)*EPI_COLS) with h = i/4
        const int ei = warp - kEpiWarp0;
        const int q = ei & 3;
        const int h = ei >> 2;
        int it = 0;
        uint32_t kc = 0;  // K steps so far (which issuers took part in a tile)
        // loop exits are warp-uniform: the TMEM loads below are warp-collective
        TileInfo ti;
        for (WorkCursor wc = work_begin(p, total, nkt);
             !__any_sync(0xFFFFFFFFu, *abort_flag != 0) &&
             work_next<BT>(wc, ti, s_rows, s_tiles, p, total, nch, nkt, kper);
             ++it) {
            // issuer i accumulated into this tile iff one of its K steps
            // (kc = i mod NI) falls in [kc0, kc0 + steps)
            const uint32_t kc0 = kc;
            const int steps = ti.kt1 - ti.kt0;
            kc += static_cast<uint32_t>(steps);
            const int b = it & 1;
            const uint32_t aph = (it >> 1) & 1;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&accf_bar[b], aph, abort_flag, p.err,
                                                           ERR_GEMM_TIMEOUT)))
                break;
            tc_fence_after();
            const int n = ti.n0 + q * 32 + lane;
            const bool nvalid = n < p.N;
            const float sc =
                nvalid ? __ldg(p.scale + static_cast<int64_t>(ti.wg) * p.N + n) : 0.0f;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(b * NI * BT);
            const int cbeg = h * C::EPI_COLS;
            const int cend = min(cbeg + C::EPI_COLS, ti.nrows);
#pragma unroll 1
            for (int c0 = cbeg; c0 < cend; c0 += 16) {
                // lanes 0..15 fetch the output row and row multiplier of the 16
                // columns of this chunk; shuffles hand them to every lane
                int my_orow = 0;
                float my_rs = 1.0f;
                const int64_t my_row = ti.row0 + c0 + (lane & 15);
                if (lane < 16 && c0 + lane < ti.nrows) {
                    my_orow = p.rowmap ? __ldg(p.rowmap + my_row) : static_cast<int>(my_row);
                    if (p.rowscale) my_rs = __ldg(p.rowscale + my_row);
                }
                uint32_t r[16];
                if constexpr (NI == 1) {
                    tc_ld_32x32b_x16(tbase + c0, r);
                    tc_wait_ld();
                } else {
                    // the sum of the issuers' partial accumulators
                    float sum[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) sum[j] = 0.0f;
#pragma unroll
                    for (int i = 0; i < NI; ++i) {
                        if ((i - static_cast<int>(kc0 % NI) + NI) % NI >= steps) continue;
                        uint32_t t[16];
                        tc_ld_32x32b_x16(tbase + static_cast<uint32_t>(i * BT + c0), t);
                        tc_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j) sum[j] += __uint_as_float(t[j]);
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(sum[j]);
                }
                if (p.red_v4) {
                    // 16-byte reductions: a 4x4 transpose inside each lane quad
                    // gives lane 4m+i the four channels of quad m at column i,
                    // so one red.v4 replaces four scalar ones.
                    const int qi = lane & 3;
                    const bool qvalid = ti.n0 + q * 32 + (lane & ~3) < p.N;  // N % 4 == 0
                    float* obase = reinterpret_cast<float*>(p.out) + ti.n0 + q * 32 + (lane & ~3);
#pragma unroll
                    for (int j4 = 0; j4 < 16; j4 += 4) {
                        float a[4];
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            a[c] = __uint_as_float(r[j4 + c]) * sc *
                                   __shfl_sync(0xFFFFFFFFu, my_rs, j4 + c);
                        {
                            const float s0 = (qi & 1) ? a[0] : a[1];
                            const float s1 = (qi & 1) ? a[2] : a[3];
                            const float t0 = __shfl_xor_sync(0xFFFFFFFFu, s0, 1);
                            const float t1 = __shfl_xor_sync(0xFFFFFFFFu, s1, 1);
                            if (qi & 1) {
                                a[0] = t0;
                                a[2] = t1;
                            } else {
                                a[1] = t0;
                                a[3] = t1;
                            }
                        }
                        {
                            const float s0 = (qi & 2) ? a[0] : a[2];
                            const float s1 = (qi & 2) ? a[1] : a[3];
                            const float t0 = __shfl_xor_sync(0xFFFFFFFFu, s0, 2);
                            const float t1 = __shfl_xor_sync(0xFFFFFFFFu, s1, 2);
                            if (qi & 2) {
                                a[0] = t0;
                                a[1] = t1;
                            } else {
                                a[2] = t0;
                                a[3] = t1;
                            }
                        }
                        const int64_t orow = __shfl_sync(0xFFFFFFFFu, my_orow, j4 + qi);
                        if (qvalid && c0 + j4 + qi < ti.nrows)
                            red_add_v4(obase + orow * p.ldo, a[0], a[1], a[2], a[3]);
                    }
                    continue;
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int64_t orow = __shfl_sync(0xFFFFFFFFu, my_orow, j);
                    const float rs = __shfl_sync(0xFFFFFFFFu, my_rs, j);
                    if (nvalid && c0 + j < ti.nrows) {
                        float v = __uint_as_float(r[j]) * sc * rs;
                        if (p.relu) v = fmaxf(v, 0.0f);
                        if (p.out_bf16) {
                            const __nv_bfloat16 hi = __float2bfloat16_rn(v);
                            reinterpret_cast<__nv_bfloat16*>(p.out)[orow * p.ldo + n] = hi;
                            if (p.out_lo)
                                reinterpret_cast<__nv_bfloat16*>(p.out_lo)[orow * p.ldo + n] =
                                    __float2bfloat16_rn(v - __bfloat162float(hi));
                        } else if (p.atomic_add) {
                            atomicAdd(reinterpret_cast<float*>(p.out) + orow * p.ldo + n, v);
                        } else {
                            reinterpret_cast<float*>(p.out)[orow * p.ldo + n] = v;
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce_bar[b]);
        }
    }

    // ---- teardown
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// ============================================================================
// SM-pair form (tcgen05 cta_group::2) for large token tiles.
//
// A cluster of two CTAs on two SMs shares one tile of 256 output channels x BT
// token rows: CTA c converts ITS 128 channels (channel block 2*pair + c) into
// its own shared memory -- the A operand is split by M over the pair -- and
// TMA-loads HALF of the tile's token rows -- the B operand is split by N -- so
// one tcgen05.mma.cta_group::2 (M = 256) issued by the even CTA multiplies
// both SMs' halves, and each CTA's TMEM receives its 128 channels x all BT
// columns.  Per SM and K step this moves 8 + 16 + BT/2*128 bytes into shared
// memory instead of 8 + 16 + BT*128 (and reads as much back), and one thread
// issues the MMAs of two SMs.
// The activation tiles and the converted weights sit in two rings of their
// own depths (DX and DW slots; K step kc uses slots kc % DX and kc % DW),
// synchronised per K step through NB barrier slots (kc % NB): the activation
// TMA, issued when its slot frees and landing 1000-2000 cycles later, gets
// the deep ring, the conversion, which starts once the int8 tile is in, the
// shallow one.  A producer reuses slot kc % D after the MMAs of K step
// kc - D completed, i.e. it waits on st_empty[(kc - D) % NB] for phase
// (kc - D) / NB.  That parity wait is exact because NB >= D (the barrier
// cannot have completed K step kc - D + NB, which needs this very tile) and
// the producer already saw K step kc - D - NB complete (its own earlier
// wait; for converter groups NB is a multiple of the group count).
// Synchronisation (same barrier offsets in both CTAs; every wait and arrival
// uses the default CTA-scope semantics, as the tcgen05 pipelines of CUTLASS do):
//   st_full[j]   even CTA: both CTAs' activation TMA bytes (the odd CTA's
//                loads complete on the even CTA's barrier, .cta_group::2),
//                its producer's expect-tx arrival and one arrival per
//                converter warp of BOTH CTAs (the odd CTA's arrive remotely);
//   st_empty[j]  both: one tcgen05.commit multicast to the pair per K step;
//   accf[b]      both: the commit of a tile's last K step (multicast);
//   acce[b]      even CTA: 8 local + 8 remote epilogue-warp arrivals.
// Every wait is bounded; a timeout sets the abort flag in both CTAs.  The pair
// meets at a cluster barrier after set-up and before teardown, so no CTA
// exits while its peer may still touch its shared memory.
template <int BT, int SPLIT>
struct Cfg2 {
    static constexpr int HB = BT / 2;              // token rows per CTA (MMA N / 2)
    static constexpr int W8 = kCh * kKT;
    static constexpr int W16 = kCh * kKT * 2;
    static constexpr int XB = HB * kKT * 2;        // bf16 activation half-tile, per part
    static constexpr int XS = SPLIT * XB;
    static constexpr int BUDGET = 216 * 1024;
    static constexpr int CG = 4 < AEM_QGEMM_MAX_CONV_GROUPS ? 4 : AEM_QGEMM_MAX_CONV_GROUPS;
    // eight int8 slots measured 1-2% ahead of four at the layer bench's
    // shapes; with float32 activations (two 16 KB parts per slot) four leave
    // room for three activation slots
    static constexpr int S8_WANT = SPLIT == 2 ? 4 : AEM_PAIR_W8_STAGES;
    static constexpr int S8_MIN = ((S8_WANT + CG - 1) / CG) * CG;
    static constexpr int DW = AEM_PAIR_W16_STAGES;
    static constexpr int DX_RAW = (BUDGET - S8_MIN * W8 - DW * W16) / XS;
    static constexpr int DX = DX_RAW > AEM_PAIR_X_STAGES_MAX ? AEM_PAIR_X_STAGES_MAX : DX_RAW;
    // the int8 ring, whose tiles are re-read from L2 by every token tile,
    // takes what is left (a multiple of the converter groups)
    static constexpr int S8_RAW = (BUDGET - DX * XS - DW * W16) / W8;
    static constexpr int S8 = ((S8_RAW > 12 ? 12 : S8_RAW) / CG) * CG;
    static constexpr int NB_RAW = DX > DW ? DX : DW;
    static constexpr int NB = ((NB_RAW + CG - 1) / CG) * CG;
    static constexpr int TMEM_COLS = 2 * BT < 32 ? 32 : 2 * BT;
    static constexpr int BAR_BYTES = (2 * NB + 2 * S8 + 4) * 8 + 16;
    static constexpr int TAB_BYTES = 2 * (kMaxGroups + 1) * 4;
    static constexpr int SMEM = 1024 + DW * W16 + DX * XS + S8 * W8 + BAR_BYTES + TAB_BYTES;
    static constexpr int CG_WARPS = kConvWarps / CG;
    static constexpr int CG_THREADS = CG_WARPS * 32;
    static constexpr int EPI_COLS = BT >= 32 ? BT / 2 : BT;
    static_assert(S8 >= CG && S8 % CG == 0 && kConvWarps % CG == 0, "converter groups vs rings");
    static_assert(NB >= DX && NB >= DW && NB % CG == 0, "barrier slots vs rings");
    static_assert(S8 >= 2 && DX >= 2 && DW >= 2, "pipeline needs two stages per ring");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static_assert(BT % 32 == 0 && BT >= 32 && BT <= 256, "MMA N for M=256 (N/2 rows per CTA)");
};

// Tile t of the pair schedule: group g, channel pair pb (channels
// [256 pb, 256 pb + 256)), token tile tc, K range.
template <int BT>
__device__ __forceinline__ TileInfo decode_tile_pair(int t, const int* s_rows, const int* s_tiles,
                                                     const TcParams& p, int npair, int nkt,
                                                     int kper) {
    int lo = 0, hi = p.G;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (s_tiles[mid] <= t) lo = mid; else hi = mid;
    }
    TileInfo ti;
    ti.g = lo;
    ti.wg = static_cast<int>(p.group_base) + (p.wmod ? lo % p.wmod : lo);
    int r = t - s_tiles[lo];
    const int cnt = s_rows[lo + 1] - s_rows[lo];
    const int ntc = (cnt + BT - 1) / BT;
    const int tc = r % ntc;
    r /= ntc;
    const int ks = r % p.ksplit;
    const int pb = r / p.ksplit;
    ti.n0 = pb * 2 * kCh;  // first channel of the pair; CTA c owns [n0 + 128 c, +128)
    ti.row0 = static_cast<int64_t>(s_rows[lo]) + static_cast<int64_t>(tc) * BT;
    ti.nrows = min(BT, cnt - tc * BT);
    ti.kt0 = ks * kper;
    ti.kt1 = min(nkt, ti.kt0 + kper);
    (void)npair;
    return ti;
}

// Bounded wait that, on giving up, raises the abort flag of both CTAs.
__device__ __forceinline__ bool pair_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint32_t peer, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > 2000000000ull) {
            *abort_flag = 1;
            st_remote_u32(const_cast<int*>(abort_flag), peer, 1u);
            atomicOr(err, ERR_GEMM_TIMEOUT);
            return false;
        }
    }
}

template <int BT, int SPLIT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    qgemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tm_xh,
                         const __grid_constant__ CUtensorMap tm_xl, const TcParams p) {
    using C = Cfg2<BT, SPLIT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* w16_ring = smem;
    uint8_t* x_ring = w16_ring + C::DW * C::W16;
    uint8_t* w8_ring = x_ring + C::DX * C::XS;
    uint64_t* st_full = reinterpret_cast<uint64_t*>(w8_ring + C::S8 * C::W8);
    uint64_t* st_empty = st_full + C::NB;
    uint64_t* w8_full = st_empty + C::NB;
    uint64_t* w8_empty = w8_full + C::S8;
    uint64_t* accf_bar = w8_empty + C::S8;  // [2]
    uint64_t* acce_bar = accf_bar + 2;      // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce_bar + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* s_rows = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(st_full) + C::BAR_BYTES);
    int* s_tiles = s_rows + (kMaxGroups + 1);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const uint32_t cta = cluster_rank();  // 0: issues the MMAs; 1: its peer
    const uint32_t peer = cta ^ 1u;
    const int pair = blockIdx.x >> 1;
    const int npairs = gridDim.x >> 1;

    if (tid == 0) {
        for (int s = 0; s < C::NB; ++s) {
            mbar_init(&st_full[s], 2 * C::CG_WARPS + 1);  // used in the even CTA
            mbar_init(&st_empty[s], 1);
        }
        for (int s = 0; s < C::S8; ++s) {
            mbar_init(&w8_full[s], 1);
            mbar_init(&w8_empty[s], C::CG_WARPS);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accf_bar[b], 1);
            mbar_init(&acce_bar[b], 2 * kEpiWarps);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    for (int i = tid; i <= p.G; i += kThreads)
        s_rows[i] = p.group_rows ? p.group_rows[i] : (i == 0 ? 0 : static_cast<int>(p.M));
    if (warp == kMmaWarp) {
        tmem_alloc_pair(tmem_slot, C::TMEM_COLS);  // the same warp of both CTAs
        tmem_relinquish_pair();
    }
    if (warp == kXWarp && lane == 0) {
        tma_prefetch_desc(&tm_xh);
        if (SPLIT == 2) tma_prefetch_desc(&tm_xl);
    }
    const int nch = (p.N + kCh - 1) / kCh;
    const int npair = (nch + 1) / 2;
    const int nkt = (p.K + kKT - 1) / kKT;
    const int kper = (nkt + p.ksplit - 1) / p.ksplit;
    __syncthreads();
    if (tid == 0) {
        int acc = 0;
        bool bad = false;
        for (int g = 0; g < p.G; ++g) {
            s_tiles[g] = acc;
            const int cnt = s_rows[g + 1] - s_rows[g];
            if (cnt < 0) bad = true;
            acc += (cnt > 0 ? (cnt + BT - 1) / BT : 0) * npair * p.ksplit;
        }
        s_tiles[p.G] = acc;
        if (bad) {
            atomicOr(p.err, ERR_GEMM_GROUPS);
            s_tiles[p.G] = 0;
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers are initialised before any remote arrival
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = s_tiles[p.G];

    if (warp == kW8Warp) {
        // ================= int8 weight producer: this CTA's 128-channel block
        if (lane == 0) {
            int s8 = 0;
            uint32_t ph8 = 0;
            bool ok = true;
            for (int t = pair; t < total && ok && !*abort_flag; t += npairs) {
                const TileInfo ti = decode_tile_pair<BT>(t, s_rows, s_tiles, p, npair, nkt, kper);
                // an odd channel count leaves the last pair's odd block past N: it
                // streams the last real block again (results past N are never stored)
                const int nb = min(ti.n0 / kCh + static_cast<int>(cta), nch - 1);
                const int8_t* wsrc =
                    p.wq + ((static_cast<int64_t>(ti.wg) * p.NT + nb) * p.KT) * (kCh * kKT);
                for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
                    if (!pair_wait(&w8_empty[s8], ph8 ^ 1, abort_flag, peer, p.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&w8_full[s8], C::W8);
                    bulk_load(w8_ring + s8 * C::W8, wsrc + static_cast<int64_t>(kt) * C::W8, C::W8,
                              &w8_full[s8]);
                    if (++s8 == C::S8) {
                        s8 = 0;
                        ph8 ^= 1;
                    }
                }
            }
        }
    } else if (warp == kXWarp) {
        // ================= activation producer: this CTA's half of the token rows
        if (lane == 0) {
            uint32_t kc = 0;
            bool ok = true;
            for (int t = pair; t < total && ok && !*abort_flag; t += npairs) {
                const TileInfo ti = decode_tile_pair<BT>(t, s_rows, s_tiles, p, npair, nkt, kper);
                const int n_eff = min(BT, (ti.nrows + 31) & ~31);  // MMA N: halves of >= 16 rows
                const int row = static_cast<int>(ti.row0) + static_cast<int>(cta) * (n_eff / 2);
                for (int kt = ti.kt0; kt < ti.kt1; ++kt, ++kc) {
                    if (kc >= static_cast<uint32_t>(C::DX)) {  // slot kc % DX: K step kc - DX done
                        const uint32_t j = kc - C::DX;
                        if (!pair_wait(&st_empty[j % C::NB], (j / C::NB) & 1, abort_flag, peer,
                                       p.err)) {
                            ok = false;
                            break;
                        }
                    }
                    uint8_t* st = x_ring + (kc % C::DX) * C::XS;
                    uint64_t* full = &st_full[kc % C::NB];
                    // both halves' bytes complete on the even CTA's barrier
                    if (cta == 0) mbar_arrive_expect_tx(full, 2 * C::XS);
                    tma_load_2d_pair(st, &tm_xh, full, 0, kt * kKT, row);
                    if (SPLIT == 2) tma_load_2d_pair(st + C::XB, &tm_xl, full, 0, kt * kKT, row);
                }
            }
        }
    } else if (warp == kMmaWarp) {
        if (cta == 0) {
            // ================= MMA issuer of the pair: the whole warp runs the
            // loop (warp-uniform values), one elected lane issues -- 4-5%
            // faster than one lane running it alone (dense 4096 x 4096 x 14336)
            int sb = 0, sw = 0, sx = 0;  // kc % NB, kc % DW, kc % DX
            uint32_t phb = 0;            // (kc / NB) & 1
            int it = 0;
            bool ok = true;
            // (the abort vote keeps the warp's lanes on one path)
            for (int t = pair; t < total && ok && !__any_sync(0xFFFFFFFFu, *abort_flag != 0);
                 t += npairs, ++it) {
                const TileInfo ti = decode_tile_pair<BT>(t, s_rows, s_tiles, p, npair, nkt, kper);
                const int b = it & 1;
                const uint32_t aph = (it >> 1) & 1;
                // both CTAs' epilogues have drained accumulator b
                if (!__all_sync(0xFFFFFFFFu,
                                pair_wait(&acce_bar[b], aph ^ 1, abort_flag, peer, p.err)))
                    break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * BT);
                const int n_eff = min(BT, (ti.nrows + 31) & ~31);
                const uint32_t idesc = idesc_bf16_f32(2 * kCh, static_cast<uint32_t>(n_eff));
                for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
                    // both CTAs' activation halves and converted weights are in
                    if (!__all_sync(0xFFFFFFFFu,
                                    pair_wait(&st_full[sb], phb, abort_flag, peer, p.err))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t adesc = smem_desc_sw128(smem_u32(w16_ring + sw * C::W16));
                    const uint64_t bdesc = smem_desc_sw128(smem_u32(x_ring + sx * C::XS));
                    const uint64_t ldesc = smem_desc_sw128(smem_u32(x_ring + sx * C::XS + C::XB));
#pragma unroll
                    for (int kk = 0; kk < kKT / 16; ++kk) {
                        tc_mma_f16_pair_elect(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc,
                                              (kt > ti.kt0 || kk > 0) ? 1u : 0u);
                        if (SPLIT == 2)
                            tc_mma_f16_pair_elect(d_tmem, adesc + 2 * kk, ldesc + 2 * kk, idesc,
                                                  1u);
                    }
                    tc_commit_pair_elect(&st_empty[sb], 0x3);  // frees K step kc's slots in both CTAs
                    if (++sb == C::NB) {
                        sb = 0;
                        phb ^= 1;
                    }
                    if (++sw == C::DW) sw = 0;
                    if (++sx == C::DX) sx = 0;
                }
                if (!ok) break;
                tc_commit_pair_elect(&accf_bar[b], 0x3);
            }
        }
    } else if (warp < kConvWarps) {
        // ================= converters (this CTA's channel block)
        const int group = warp / C::CG_WARPS;
        const int gtid = tid % C::CG_THREADS;
        uint32_t kc = 0;
        bool ok = true;
        for (int t = pair; t < total && ok && !*abort_flag; t += npairs) {
            const TileInfo ti = decode_tile_pair<BT>(t, s_rows, s_tiles, p, npair, nkt, kper);
            for (int kt = ti.kt0; kt < ti.kt1; ++kt, ++kc) {
                if (static_cast<int>(kc % C::CG) != group) continue;
                const int s8 = static_cast<int>(kc % C::S8);
                const uint32_t ph8 = (kc / C::S8) & 1;
                // slot kc % DW is free once K step kc - DW's MMAs completed
                const uint32_t j = kc - C::DW;
                if (!pair_wait(&w8_full[s8], ph8, abort_flag, peer, p.err) ||
                    (kc >= static_cast<uint32_t>(C::DW) &&
                     !pair_wait(&st_empty[j % C::NB], (j / C::NB) & 1, abort_flag, peer, p.err))) {
                    ok = false;
                    break;
                }
                uint8_t* st = w16_ring + (kc % C::DW) * C::W16;
                const uint8_t* w8 = w8_ring + s8 * C::W8;
#pragma unroll
                for (int i = 0; i < 512 / C::CG_THREADS; ++i) {
                    const int item = gtid + C::CG_THREADS * i;
                    const int r = item >> 2;
                    const int ch = item & 3;
                    const uint4 v =
                        *reinterpret_cast<const uint4*>(w8 + r * 64 + wtile_chunk(r, ch) * 16);
                    const uint2 a0 = i8x4_to_bf16x4(v.x);
                    const uint2 a1 = i8x4_to_bf16x4(v.y);
                    const uint2 a2 = i8x4_to_bf16x4(v.z);
                    const uint2 a3 = i8x4_to_bf16x4(v.w);
                    uint8_t* row = st + r * 128;
                    const int sw = r & 7;
                    *reinterpret_cast<uint4*>(row + (((2 * ch) ^ sw) << 4)) =
                        make_uint4(a0.x, a0.y, a1.x, a1.y);
                    *reinterpret_cast<uint4*>(row + (((2 * ch + 1) ^ sw) << 4)) =
                        make_uint4(a2.x, a2.y, a3.x, a3.y);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if (cta == 0)
                        mbar_arrive(&st_full[kc % C::NB]);
                    else
                        mbar_arrive_remote(&st_full[kc % C::NB], 0);
                    mbar_arrive(&w8_empty[s8]);
                }
            }
        }
    } else if (warp < kEpiWarp0 + kEpiWarps) {
        // ================= epilogue: this CTA's 128 channels x the tile's columns
        const int ei = warp - kEpiWarp0;
        const int q = ei & 3;
        const int h = ei >> 2;
        int it = 0;
        for (int t = pair; t < total && !__any_sync(0xFFFFFFFFu, *abort_flag != 0);
             t += npairs, ++it) {
            const TileInfo ti = decode_tile_pair<BT>(t, s_rows, s_tiles, p, npair, nkt, kper);
            const int b = it & 1;
            const uint32_t aph = (it >> 1) & 1;
            if (!__all_sync(0xFFFFFFFFu,
                            pair_wait(&accf_bar[b], aph, abort_flag, peer, p.err)))
                break;
            tc_fence_after();
            const int n0 = ti.n0 + static_cast<int>(cta) * kCh;
            const int n = n0 + q * 32 + lane;
            const bool nvalid = n < p.N;
            const float sc =
                nvalid ? __ldg(p.scale + static_cast<int64_t>(ti.wg) * p.N + n) : 0.0f;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(b * BT);
            const int cbeg = h * C::EPI_COLS;
            const int cend = min(cbeg + C::EPI_COLS, ti.nrows);
            // bf16 output without a low half: each lane stores 8 channels of a
            // row at once (16 bytes) after an 8x8 transpose inside its group
            // of 8 lanes -- 2 stores per 16-column chunk instead of 16 (the
            // per-row 2-byte stores queued behind the converters' shared-memory
            // traffic and made the epilogue as long as a tile's main loop)
            const bool v8 = !p.red_v4 && p.out_bf16 && !p.out_lo && !p.atomic_add &&
                            ((p.N | static_cast<int>(p.ldo & 7)) & 7) == 0 &&
                            (reinterpret_cast<uintptr_t>(p.out) & 15) == 0;
            // output row and row scale of row c0 + lane (lanes < 16; loading
            // them a chunk ahead measured no faster)
            auto row_info = [&](int c0, int& orow, float& rs) {
                orow = 0;
                rs = 1.0f;
                const int64_t row = ti.row0 + c0 + (lane & 15);
                if (lane < 16 && c0 + lane < ti.nrows) {
                    orow = p.rowmap ? __ldg(p.rowmap + row) : static_cast<int>(row);
                    if (p.rowscale) rs = __ldg(p.rowscale + row);
                }
            };
#pragma unroll 1
            for (int c0 = cbeg; c0 < cend; c0 += 16) {
                int my_orow;
                float my_rs;
                row_info(c0, my_orow, my_rs);
                uint32_t r[16];
                tc_ld_32x32b_x16(tbase + c0, r);
                tc_wait_ld();
                if (p.red_v4) {
                    const int qi = lane & 3;
                    const bool qvalid = n0 + q * 32 + (lane & ~3) < p.N;
                    float* obase = reinterpret_cast<float*>(p.out) + n0 + q * 32 + (lane & ~3);
#pragma unroll
                    for (int j4 = 0; j4 < 16; j4 += 4) {
                        float a[4];
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            a[c] = __uint_as_float(r[j4 + c]) * sc *
                                   __shfl_sync(0xFFFFFFFFu, my_rs, j4 + c);
                        {
                            const float s0 = (qi & 1) ? a[0] : a[1];
                            const float s1 = (qi & 1) ? a[2] : a[3];
                            const float t0 = __shfl_xor_sync(0xFFFFFFFFu, s0, 1);
                            const float t1 = __shfl_xor_sync(0xFFFFFFFFu, s1, 1);
                            if (qi & 1) {
                                a[0] = t0;
                                a[2] = t1;
                            } else {
                                a[1] = t0;
                                a[3] = t1;
                            }
                        }
                        {
                            const float s0 = (qi & 2) ? a[0] : a[2];
                            const float s1 = (qi & 2) ? a[1] : a[3];
                            const float t0 = __shfl_xor_sync(0xFFFFFFFFu, s0, 2);
                            const float t1 = __shfl_xor_sync(0xFFFFFFFFu, s1, 2);
                            if (qi & 2) {
                                a[0] = t0;
                                a[1] = t1;
                            } else {
                                a[2] = t0;
                                a[3] = t1;
                            }
                        }
                        const int64_t orow = __shfl_sync(0xFFFFFFFFu, my_orow, j4 + qi);
                        if (qvalid && c0 + j4 + qi < ti.nrows)
                            red_add_v4(obase + orow * p.ldo, a[0], a[1], a[2], a[3]);
                    }
                } else if (v8) {
                    float a[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        float v = __uint_as_float(r[j]) * sc;
                        if (p.rowscale) v *= __shfl_sync(0xFFFFFFFFu, my_rs, j);
                        if (p.relu) v = fmaxf(v, 0.0f);
                        a[j] = v;
                    }
                    // lane 8g + i holds channel 8g + i of rows 0..15; after the
                    // butterfly (distances 4, 2, 1; both 8-row blocks) it holds
                    // channels 8g..8g+7 of rows i (a[0..7]) and 8 + i (a[8..15])
                    const int li = lane & 7;
#pragma unroll
                    for (int sd = 4; sd >= 1; sd >>= 1) {
#pragma unroll
                        for (int blk = 0; blk < 16; blk += 8) {
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                if (j & sd) continue;
                                const float send = (li & sd) ? a[blk + j] : a[blk + j + sd];
                                const float got = __shfl_xor_sync(0xFFFFFFFFu, send, sd);
                                if (li & sd)
                                    a[blk + j] = got;
                                else
                                    a[blk + j + sd] = got;
                            }
                        }
                    }
                    const int nb = n0 + q * 32 + 8 * (lane >> 3);  // this lane's first channel
#pragma unroll
                    for (int blk = 0; blk < 16; blk += 8) {
                        const int rr = blk + li;  // row within the chunk
                        const int64_t orow = __shfl_sync(0xFFFFFFFFu, my_orow, rr);
                        if (c0 + rr < ti.nrows && nb < p.N) {
                            uint4 v;
                            v.x = bf16x2_bits(a[blk + 0], a[blk + 1]);
                            v.y = bf16x2_bits(a[blk + 2], a[blk + 3]);
                            v.z = bf16x2_bits(a[blk + 4], a[blk + 5]);
                            v.w = bf16x2_bits(a[blk + 6], a[blk + 7]);
                            *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) +
                                                      orow * p.ldo + nb) = v;
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int64_t orow = __shfl_sync(0xFFFFFFFFu, my_orow, j);
                        const float rs = __shfl_sync(0xFFFFFFFFu, my_rs, j);
                        if (nvalid && c0 + j < ti.nrows) {
                            float v = __uint_as_float(r[j]) * sc * rs;
                            if (p.relu) v = fmaxf(v, 0.0f);
                            if (p.out_bf16) {
                                const __nv_bfloat16 hi = __float2bfloat16_rn(v);
                                reinterpret_cast<__nv_bfloat16*>(p.out)[orow * p.ldo + n] = hi;
                                if (p.out_lo)
                                    reinterpret_cast<__nv_bfloat16*>(p.out_lo)[orow * p.ldo + n] =
                                        __float2bfloat16_rn(v - __bfloat162float(hi));
                            } else if (p.atomic_add) {
                                atomicAdd(reinterpret_cast<float*>(p.out) + orow * p.ldo + n, v);
                            } else {
                                reinterpret_cast<float*>(p.out)[orow * p.ldo + n] = v;
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (cta == 0)
                    mbar_arrive(&acce_bar[b]);
                else
                    mbar_arrive_remote(&acce_bar[b], 0);
            }
        }
    }

    // ---- teardown: the pair's MMAs, commits and remote arrivals are all done
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    if (warp == kMmaWarp) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
}

template <int BT, int SPLIT, bool TSA, int NI = 1>
aem_status launch_tc(const GemmArgs& a, const TcParams& p, int grid, cudaStream_t s) {
    using C = Cfg<BT, SPLIT, TSA, NI>;
    const QWeight& w = *a.w;
    CUtensorMap th, tl;
    AEM_TRY(make_tmap_2d(&th, a.x_hi, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                         static_cast<uint64_t>(w.K), static_cast<uint64_t>(a.M), kKT, BT,
                         CU_TENSOR_MAP_SWIZZLE_128B));
    if (SPLIT == 2)
        AEM_TRY(make_tmap_2d(&tl, a.x_lo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                             static_cast<uint64_t>(w.K), static_cast<uint64_t>(a.M), kKT, BT,
                             CU_TENSOR_MAP_SWIZZLE_128B));
    else
        tl = th;
    auto kern = qgemm_tc_kernel<BT, SPLIT, TSA, NI>;
    AEM_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    kern<<<grid, C::THREADS, C::SMEM, s>>>(th, tl, p);
    AEM_CHECK_LAUNCH();
    count_launches(1);
    return AEM_OK;
}

template <int BT, int SPLIT>
aem_status launch_tc_pair(const GemmArgs& a, const TcParams& p, int pairs, cudaStream_t s) {
    using C = Cfg2<BT, SPLIT>;
    const QWeight& w = *a.w;
    CUtensorMap th, tl;
    AEM_TRY(make_tmap_2d(&th, a.x_hi, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                         static_cast<uint64_t>(w.K), static_cast<uint64_t>(a.M), kKT, C::HB,
                         CU_TENSOR_MAP_SWIZZLE_128B));
    if (SPLIT == 2)
        AEM_TRY(make_tmap_2d(&tl, a.x_lo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                             static_cast<uint64_t>(w.K), static_cast<uint64_t>(a.M), kKT, C::HB,
                             CU_TENSOR_MAP_SWIZZLE_128B));
    else
        tl = th;
    auto kern = qgemm_tc_pair_kernel<BT, SPLIT>;
    AEM_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    kern<<<2 * pairs, kThreads, C::SMEM, s>>>(th, tl, p);
    AEM_CHECK_LAUNCH();
    count_launches(1);
    return AEM_OK;
}

template <int SPLIT>
aem_status launch_pair_bt(int bt, const GemmArgs& a, const TcParams& p, int pairs,
                          cudaStream_t s) {
    switch (bt) {
        case 64: return launch_tc_pair<64, SPLIT>(a, p, pairs, s);
        case 128: return launch_tc_pair<128, SPLIT>(a, p, pairs, s);
        default: return launch_tc_pair<256, SPLIT>(a, p, pairs, s);
    }
}

// Pairs of SMs that can run the pair kernel at once on `dev` (one CTA per SM).
int max_pairs(int dev) {
    static int cache[64] = {0};
    if (dev < 0 || dev >= 64) return 0;
    if (cache[dev] == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * 512, 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = Cfg2<256, 1>::SMEM;
        int n = 0;
        auto kern = qgemm_tc_pair_kernel<256, 1>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Cfg2<256, 1>::SMEM) != cudaSuccess ||
            cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
            cudaGetLastError();
            n = sm_count(dev) / 2;
        }
        cache[dev] = n;
    }
    return cache[dev];
}

template <int SPLIT>
aem_status launch_bt(int bt, bool tsa, const GemmArgs& a, const TcParams& p, int grid,
                     cudaStream_t s) {
    if (tsa) {
        // issuers: as many as TMEM holds accumulators for (4 up to 32-row
        // tiles, 2 at 64 rows, 1 above)
        switch (bt) {
            case 16: return launch_tc<16, SPLIT, true, 4>(a, p, grid, s);
            case 32: return launch_tc<32, SPLIT, true, 4>(a, p, grid, s);
            case 64: return launch_tc<64, SPLIT, true, 2>(a, p, grid, s);
            case 128: return launch_tc<128, SPLIT, true>(a, p, grid, s);
            default: return launch_tc<192, SPLIT, true>(a, p, grid, s);
        }
    }
    switch (bt) {
        case 16: return launch_tc<16, SPLIT, false>(a, p, grid, s);
        case 32: return launch_tc<32, SPLIT, false>(a, p, grid, s);
        case 64: return launch_tc<64, SPLIT, false>(a, p, grid, s);
        case 128: return launch_tc<128, SPLIT, false>(a, p, grid, s);
        default: return launch_tc<256, SPLIT, false>(a, p, grid, s);
    }
}

int64_t tiles_estimate(int64_t M, int G, int bt, int64_t nch, int ks) {
    const int64_t avg = G > 0 ? (M + G - 1) / G : M;
    const int64_t per = (avg + bt - 1) / bt;
    return std::max<int64_t>(1, per * G) * nch * ks;
}

}  // namespace

namespace {
std::atomic<int> g_pair_mode{-1};
std::atomic<int> g_tmem_a_mode{-1};
}  // namespace

int gemm_pair_mode() { return g_pair_mode.load(std::memory_order_relaxed); }
int gemm_tmem_a_mode() { return g_tmem_a_mode.load(std::memory_order_relaxed); }

aem_status launch_qgemm(const GemmArgs& a, cudaStream_t s) {
    AEM_REQUIRE(a.w != nullptr, "qgemm: weight handle is NULL");
    const QWeight& w = *a.w;
    AEM_REQUIRE(a.G >= 1 && a.G <= kMaxGroups, "qgemm: G=%d outside [1, %d]", a.G, kMaxGroups);
    AEM_REQUIRE(a.group_base >= 0 && a.group_base + (a.wmod ? a.wmod : a.G) <= w.G,
                "qgemm: weight group out of range");
    AEM_REQUIRE(!(a.atomic_add && a.out_bf16), "qgemm: split-K needs float32 output");
    if (a.M == 0) return AEM_OK;
    if (a.x_f32_relu) {
        AEM_REQUIRE(a.M <= gemv_max_rows(), "qgemm: float32 pre-activation input takes at most %d rows",
                    gemv_max_rows());
        return launch_qgemm_gemv(a, s);
    }
    const int tmode = gemm_tmem_a_mode();
    // one row: the CUDA-core decode kernel (measured 5% ahead of the weight
    // stream there); few rows (so few per group): the weight stream on warp MMAs
    if (a.M == 1 && a.token_tile == 0 && tmode != 1) return launch_qgemm_decode(a, s);
    if (a.M <= gemv_max_rows() && a.token_tile == 0 && tmode != 1) return launch_qgemm_gemv(a, s);
    if (w.K % 8 != 0) return launch_qgemm_simt(a, s);
    AEM_REQUIRE(a.M < (1ll << 31) && w.G * w.N < (1ll << 31), "qgemm: too many rows");
    const int dev = current_device();
    const int sms = sm_count(dev);
    const int64_t nch = (w.N + kCh - 1) / kCh;
    const int64_t nkt = (w.K + kKT - 1) / kKT;

    int bt = a.token_tile;
    if (bt == 0) {
        const int64_t m = a.rows_hint > 0 ? a.rows_hint : a.M;
        const int64_t avg = (m + a.G - 1) / a.G;
        bt = avg <= 16 ? 16 : avg <= 32 ? 32 : avg <= 64 ? 64 : avg <= 128 ? 128 : 256;
        while (bt > 64 && tiles_estimate(m, a.G, bt, nch, 1) < 2 * sms) bt >>= 1;
    }
    // converted weights in TMEM (A from tensor memory): token tiles up to 192
    const bool tsa = tmode == 1 || (tmode < 0 && bt <= 64);
    if (tsa && bt > 192) bt = 192;
    int ks = a.ksplit < 1 ? 1 : a.ksplit;
    if (ks > nkt) ks = static_cast<int>(nkt);
    const int kper = static_cast<int>((nkt + ks - 1) / ks);
    ks = static_cast<int>((nkt + kper - 1) / kper);

    int* err = device_error_word(dev);
    AEM_REQUIRE(err != nullptr, "qgemm: no device error word");
    TcParams p;
    p.G = a.G;
    p.group_base = a.group_base;
    p.wmod = a.wmod;
    p.group_rows = a.group_rows;
    p.M = a.M;
    p.K = static_cast<int>(w.K);
    p.N = static_cast<int>(w.N);
    p.ksplit = ks;
    p.scale = w.scale;
    p.wq = w.q;
    p.NT = w.NT;
    p.KT = w.KT;
    p.out = a.out;
    p.out_lo = a.out_bf16 ? a.out_lo : nullptr;
    p.ldo = a.ldo;
    p.out_bf16 = a.out_bf16 ? 1 : 0;
    p.relu = a.relu ? 1 : 0;
    p.atomic_add = (a.atomic_add || ks > 1) ? 1 : 0;
    p.red_v4 = (p.atomic_add && !a.relu && w.N % 4 == 0 && a.ldo % 4 == 0 &&
                (reinterpret_cast<uintptr_t>(a.out) & 15) == 0)
                   ? 1
                   : 0;
    p.rowmap = a.rowmap;
    p.rowscale = a.rowscale;
    p.err = err;
    p.stream_k = (a.stream_k && a.atomic_add && !a.relu && !a.out_bf16) ? 1 : 0;
    if (p.stream_k) {
        ks = 1;
        p.ksplit = 1;
    }
    AEM_REQUIRE(!(ks > 1 && (a.relu || a.out_bf16)), "qgemm: split-K is float32 without ReLU only");

    // Upper bound of the tiles of all groups: sum_g ceil(rows_g / bt) <= ceil(M / bt) + (#non-empty groups).
    const int64_t rows = a.max_rows > 0 ? a.max_rows : a.M;
    const int64_t tiles_ub = ((rows + bt - 1) / bt + std::min<int64_t>(a.G, rows)) * nch * ks;
    // SM pairs (cta_group::2) for large token tiles: half the activation bytes
    // per SM and half the MMA issue per FLOP
    // automatic: 128/256-row tiles over an even number of 128-channel blocks,
    // or at least 11 (an odd count leaves the last pair's second block idle:
    // 1/12 of the MMAs at 11 blocks, which the halved activation traffic
    // still beats -- measured 5% ahead of single SMs on the 1408-channel up
    // projection of the layer bench)
    const int mode = gemm_pair_mode();
    if (!tsa && !p.stream_k && bt >= 64 &&
        (mode == 1 || (mode < 0 && bt >= 128 && (nch % 2 == 0 || nch >= 11)))) {
        const int64_t ptiles = ((rows + bt - 1) / bt + std::min<int64_t>(a.G, rows)) *
                               ((nch + 1) / 2) * ks;
        const int pairs =
            static_cast<int>(std::min<int64_t>(max_pairs(dev), std::max<int64_t>(1, ptiles)));
        if (a.x_lo) return launch_pair_bt<2>(bt, a, p, pairs, s);
        return launch_pair_bt<1>(bt, a, p, pairs, s);
    }
    const int grid = p.stream_k ? sms
                                : static_cast<int>(std::min<int64_t>(sms, std::max<int64_t>(1, tiles_ub)));
    if (a.x_lo) return launch_bt<2>(bt, tsa, a, p, grid, s);
    return launch_bt<1>(bt, tsa, a, p, grid, s);
}

}  // namespace aem

extern "C" aem_status aem_set_gemm_tmem_a(int mode) {
    AEM_REQUIRE(mode == -1 || mode == 0 || mode == 1,
                "aem_set_gemm_tmem_a: mode %d is not -1, 0 or 1", mode);
    aem::g_tmem_a_mode.store(mode, std::memory_order_relaxed);
    return AEM_OK;
}

extern "C" aem_status aem_set_gemm_pairs(int mode) {
    AEM_REQUIRE(mode == -1 || mode == 0 || mode == 1,
                "aem_set_gemm_pairs: mode %d is not -1, 0 or 1", mode);
    aem::g_pair_mode.store(mode, std::memory_order_relaxed);
    return AEM_OK;
}
