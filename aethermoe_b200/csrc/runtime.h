// Internal host-side declarations shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "aem.h"

#include <functional>
#include <utility>
#include <vector>

namespace aem {

const char* last_error_cstr();

// Counts kernel launches made by this library (aem_kernel_launches()).
void count_launches(int n);

// Per-phase device-time accounting with CUDA events on the step's stream.
// Telemetry of one layer step (telemetry.cu): when telemetry is on, records
// a CUDA event on `s` at construction and at destruction, and hands the pair
// to the process-wide recorder.  No cost beyond one atomic load when off.
class StepTimer {
public:
    StepTimer(int metric, cudaStream_t s);
    ~StepTimer();
    StepTimer(const StepTimer&) = delete;
    StepTimer& operator=(const StepTimer&) = delete;

private:
    int metric_;
    cudaStream_t stream_;
    int device_ = 0;
    cudaEvent_t a_ = nullptr, b_ = nullptr;
};

struct PhaseProfiler {
    bool on = false;
    int64_t steps = 0;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending[AEM_NUM_PHASES];
    double acc_ms[AEM_NUM_PHASES] = {0};
    std::vector<cudaEvent_t> pool;
    cudaEvent_t open_ev[AEM_NUM_PHASES] = {nullptr};
    cudaEvent_t take();
    void begin(int phase, cudaStream_t s);
    void end(int phase, cudaStream_t s);
    void step() {
        if (on) ++steps;
    }
    void enable(bool e);
    aem_status read(double* ms, int64_t* nsteps);
    ~PhaseProfiler();
};

struct HostPipe;  // asynchronous host-buffer steps (pipeline.cu)

// Host-staging context behind aem_context_t: one stream plus grow-only
// device and pinned-host buffers for the *_host entry points.
struct Context {
    int device = 0;
    cudaStream_t stream = nullptr;
    HostPipe* pipe = nullptr;  // created by the first asynchronous submit
    void* dev = nullptr;
    size_t dev_bytes = 0;
    void* host = nullptr;
    size_t host_bytes = 0;
    aem_status reserve_device(size_t bytes);
    aem_status reserve_host(size_t bytes);
};

// Asynchronous host-buffer steps on a context (pipeline.cu): copies x
// (xb bytes) in on an upload stream, runs compute(device in, device out,
// context stream), copies ob bytes out on a download stream; two steps in
// flight per context.  pipe_wait reports the step's in-kernel errors.
aem_status pipe_submit(Context* c, const void* x, size_t xb, void* out, size_t ob,
                       const std::function<aem_status(const void*, void*, cudaStream_t)>& compute,
                       uint64_t* ticket);
aem_status pipe_wait(Context* c, uint64_t ticket);
void pipe_free(Context* c);

// Packed gating weight (device).  The [D, E] weight is stored as
// [Dpad/4][Epad][4] float32: for every group of 4 consecutive d, the 4
// values of each expert are contiguous and experts follow each other, so a
// chunk of d is one contiguous block that lands in shared memory as is.
// Epad is E rounded up to the kernel's lane-group width (8/16/32/64/128/256),
// Dpad is D rounded up to 256 (the widest chunk a gating kernel reads);
// padding is zero.  bias [Epad], zero padded.
struct Gate {
    int device = 0;
    int64_t D = 0, E = 0, Dpad = 0, Epad = 0;
    float* wt = nullptr;
    float* bias = nullptr;
    // The same weights in expert blocks for the small-batch kernel:
    // [Epad/eb][Dpad/4][eb][4] float32 -- block b holds experts
    // [b*eb, (b+1)*eb), and one chunk of d of one block is contiguous.
    float* wblk = nullptr;
    int eb = 0;
    // Certified mode: squared norms of the weights per 16-wide block of d,
    // [Dpad/16][Epad] (the error bound of the fast logits), and the rows of a
    // call whose selection was not certified (cert_rows[0] = count, then the
    // row ids; room for cert_cap rows) with the running total of such rows.
    float* wsq16 = nullptr;
    float* wn64 = nullptr;  // norms of the weights per 64-wide block of d, [Dpad/64][Epad]
    mutable int* cert_rows = nullptr;
    mutable int64_t cert_cap = 0;
    unsigned long long* cert_total = nullptr;
};
int gate_epad(int64_t E);
int gate_small_eb(int64_t Epad);  // experts per CTA of the small-batch kernel

// Packed INT8 weight (device), pre-tiled for the GEMM's weight stream:
// [G][NT][KT][128][64] int8 with NT = ceil(N/128), KT = ceil(K/64): every
// 128-output-channel x 64-K tile is one contiguous 8 KB block of 64-byte
// channel rows, zero padded.  Inside a row, the 16-byte chunk c (K offsets
// 16c .. 16c+15) sits at chunk position c ^ ((row >> 1) & 3), so 32 threads
// reading the same chunk of 32 consecutive rows from shared memory touch
// every bank group evenly (4 wavefronts per 512 bytes).  scale [G][N] float32.
constexpr int64_t kWTileN = 128, kWTileK = 64, kWTileBytes = kWTileN * kWTileK;
struct QWeight {
    int device = 0;
    int64_t G = 0, K = 0, N = 0, NT = 0, KT = 0;
    int8_t* q = nullptr;
    float* scale = nullptr;
};
// Chunk position of the 16-byte chunk c of channel row r inside a tile.
__host__ __device__ inline int wtile_chunk(int r, int c) { return c ^ ((r >> 1) & 3); }
// Byte offset of element (g, n, k) in the tiled layout.
__host__ __device__ inline int64_t wtile_offset(int64_t g, int64_t n, int64_t k, int64_t NT,
                                                int64_t KT) {
    const int r = static_cast<int>(n % kWTileN), kk = static_cast<int>(k % kWTileK);
    return ((g * NT + n / kWTileN) * KT + k / kWTileK) * kWTileBytes + r * kWTileK +
           wtile_chunk(r, kk >> 4) * 16 + (kk & 15);
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ---- kernels' host launchers (defined in the .cu files)
aem_status launch_gating(const Gate& g, const void* x, aem_dtype xd, int64_t N, int k, int ksel,
                         aem_gating_mode mode, int32_t* idx, float* val, cudaStream_t s);

// Grouped INT8 GEMM on the tcgen05 tensor cores (or the CUDA-core fallback
// when K % 16 != 0).  Row group g owns activation rows
// [group_rows[g], group_rows[g+1]) (device array of G+1 ints; nullptr means
// one group of M rows) and weight group (group_base + g).
struct GemmArgs {
    const QWeight* w = nullptr;
    int64_t group_base = 0;    // first weight group used
    int G = 1;                 // number of row groups
    int wmod = 0;              // weight group of row group g: group_base + (wmod ? g % wmod : g)
    const int* group_rows = nullptr;
    int64_t M = 0;             // total activation rows (for the TMA map)
    int64_t max_rows = 0;      // upper bound of sum_g ceil(rows_g / BT) * BT (grid sizing)
    const void* x_hi = nullptr;  // bf16 [M, K]
    const void* x_lo = nullptr;  // bf16 [M, K] or nullptr (split float32 activations)
    // weight-stream kernel only (at most gemv_max_rows() rows): float32 [M, K]
    // pre-activations instead of x_hi / x_lo, taken as bf16(relu(v)) -- and
    // with x_f32_lo the pair hi + lo, lo = bf16(relu(v) - hi) -- as they are staged
    const float* x_f32_relu = nullptr;
    bool x_f32_lo = false;
    void* out = nullptr;
    bool out_bf16 = false;
    // bf16 output only: when set, the output is written as a bf16 pair,
    // out = bf16(v) and out_lo = bf16(v - out) (same layout and stride), so
    // out + out_lo carries v to about 16 significant bits -- the split form a
    // following GEMM takes as x_hi / x_lo
    void* out_lo = nullptr;
    int64_t ldo = 0;           // output row stride (elements)
    bool relu = false;
    bool atomic_add = false;   // float32 out only: red.add partial sums (split-K)
    int ksplit = 1;
    // atomic_add only: every CTA takes an equal share of the (tile, K step)
    // space (partial tiles add into the output, which must start at zero)
    bool stream_k = false;
    const int* rowmap = nullptr;    // output row of activation row r (nullable)
    const float* rowscale = nullptr;  // per-activation-row multiplier (nullable)
    int token_tile = 0;        // 0 = choose from average rows per group
    int64_t rows_hint = 0;     // expected rows when the group sizes live only on the
                               // device (0 = use M); only picks the token tile
};
aem_status launch_qgemm(const GemmArgs& a, cudaStream_t s);
int gemv_max_rows();  // rows up to which launch_qgemm takes the weight-stream kernel
int gemm_pair_mode();  // aem_set_gemm_pairs: -1 automatic, 0 never, 1 from 64-row tiles

// float32 [M, K] -> bf16 hi [M, K] + bf16 lo [M, K] (lo may be nullptr), or
// bf16 copy when the input is already bf16 (hi only).
aem_status launch_split_bf16(const void* x, aem_dtype xd, int64_t count, void* hi, void* lo,
                             cudaStream_t s);

}  // namespace aem
