// Scheduler -> MoE-layer seam: one continuous-batching iteration
// (ContinuousBatchingScheduler::step, src/core/scheduler.hpp:75-146) runs
// through the MoE layer as one batch.  Each sequence's slice of hidden rows
// is gathered into contiguous staging rows in the scheduler's result order
// (which is the batch_position order the capacity rule ranks by), the layer
// runs once, and the output rows are scattered back to each slice.
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "moe.h"
#include "runtime.h"

namespace aem {

namespace {

struct SliceRow {
    const char* x;
    char* out;
    int64_t row0;  // first staging row of the slice
};

constexpr int kSeamThreads = 256;

// Staging row r belongs to the slice with the largest row0 <= r.
__device__ __forceinline__ int find_slice(const SliceRow* t, int n, int64_t r) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (t[mid].row0 <= r) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// One warp per row: rows of `bytes` bytes (16-byte vectors when every row
// start is 16-byte aligned, else bytes one at a time).
__global__ void __launch_bounds__(kSeamThreads)
    seam_copy_kernel(const SliceRow* __restrict__ table, int n, int64_t rows, int64_t bytes,
                     char* __restrict__ stage, int to_stage, int vec) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
         r < rows; r += nw) {
        const SliceRow sl = table[find_slice(table, n, r)];
        const int64_t i = r - sl.row0;
        const char* src = to_stage ? sl.x + i * bytes : stage + r * bytes;
        char* dst = to_stage ? stage + r * bytes : sl.out + i * bytes;
        if (vec) {
            const uint4* s4 = reinterpret_cast<const uint4*>(src);
            uint4* d4 = reinterpret_cast<uint4*>(dst);
            for (int64_t j = lane; j < bytes / 16; j += 32) d4[j] = s4[j];
        } else {
            for (int64_t j = lane; j < bytes; j += 32) dst[j] = src[j];
        }
    }
}

}  // namespace

struct SeamStage {
    int device = 0;
    char* rows_in = nullptr;   // staged x rows
    char* rows_out = nullptr;  // staged output rows
    int64_t row_cap = 0;       // rows of each
    int64_t in_bytes = 0, out_bytes = 0;
    SliceRow* d_table = nullptr;
    SliceRow* h_table[2] = {nullptr, nullptr};  // pinned, alternating between calls
    cudaEvent_t table_done[2] = {nullptr, nullptr};
    int table_cap = 0;
    int flip = 0;
};

void seam_free(Moe* m) {
    SeamStage* st = m->seam;
    if (!st) return;
    cudaFree(st->rows_in);
    cudaFree(st->rows_out);
    cudaFree(st->d_table);
    for (int i = 0; i < 2; ++i) {
        cudaFreeHost(st->h_table[i]);
        if (st->table_done[i]) cudaEventDestroy(st->table_done[i]);
    }
    delete st;
    m->seam = nullptr;
}

namespace {

aem_status seam_reserve(Moe* m, int64_t rows, int64_t in_row, int64_t out_row, int n,
                        cudaStream_t s) {
    if (!m->seam) {
        m->seam = new SeamStage();
        m->seam->device = m->gate->device;
        for (int i = 0; i < 2; ++i)
            AEM_TRY_CUDA(cudaEventCreateWithFlags(&m->seam->table_done[i], cudaEventDisableTiming));
    }
    SeamStage* st = m->seam;
    if (rows > st->row_cap || in_row > st->in_bytes || out_row > st->out_bytes) {
        AEM_TRY_CUDA(cudaStreamSynchronize(s));
        cudaFree(st->rows_in);
        cudaFree(st->rows_out);
        st->rows_in = st->rows_out = nullptr;
        st->row_cap = std::max(rows, st->row_cap);
        st->in_bytes = std::max(in_row, st->in_bytes);
        st->out_bytes = std::max(out_row, st->out_bytes);
        AEM_TRY_CUDA(cudaMalloc(&st->rows_in, st->row_cap * st->in_bytes));
        AEM_TRY_CUDA(cudaMalloc(&st->rows_out, st->row_cap * st->out_bytes));
    }
    if (n > st->table_cap) {
        AEM_TRY_CUDA(cudaStreamSynchronize(s));
        cudaFree(st->d_table);
        for (int i = 0; i < 2; ++i) cudaFreeHost(st->h_table[i]);
        st->d_table = nullptr;
        st->h_table[0] = st->h_table[1] = nullptr;
        const int cap = std::max(n, 256);
        AEM_TRY_CUDA(cudaMalloc(&st->d_table, sizeof(SliceRow) * cap));
        for (int i = 0; i < 2; ++i)
            AEM_TRY_CUDA(cudaMallocHost(&st->h_table[i], sizeof(SliceRow) * cap));
        st->table_cap = cap;
    }
    return AEM_OK;
}

}  // namespace

}  // namespace aem

using aem::set_error;

extern "C" aem_status aem_moe_forward_slices(aem_moe_t moe, const aem_seq_slice* slices,
                                             int n_slices, aem_dtype x_dtype, aem_dtype out_dtype,
                                             void* stream) {
    AEM_REQUIRE(moe != nullptr, "aem_moe_forward_slices: NULL layer");
    AEM_REQUIRE(n_slices >= 0 && (n_slices == 0 || slices != nullptr),
                "aem_moe_forward_slices: bad slice list");
    AEM_REQUIRE(x_dtype == AEM_F32 || x_dtype == AEM_BF16, "aem_moe_forward_slices: bad x dtype");
    AEM_REQUIRE(out_dtype == AEM_F32 || out_dtype == AEM_BF16,
                "aem_moe_forward_slices: bad out dtype");
    auto* m = reinterpret_cast<aem::Moe*>(moe);
    auto s = static_cast<cudaStream_t>(stream);
    const int64_t d = m->cfg.d_model;
    const int64_t in_row = d * (x_dtype == AEM_F32 ? 4 : 2);
    const int64_t out_row = d * (out_dtype == AEM_F32 ? 4 : 2);
    // the slice table in iteration order; empty slices dropped
    std::vector<aem::SliceRow> rows;
    rows.reserve(n_slices);
    int64_t T = 0;
    bool aligned = (in_row % 16 == 0) && (out_row % 16 == 0);
    for (int i = 0; i < n_slices; ++i) {
        AEM_REQUIRE(slices[i].tokens >= 0, "aem_moe_forward_slices: slice %d has %lld tokens", i,
                    (long long)slices[i].tokens);
        if (slices[i].tokens == 0) continue;
        AEM_REQUIRE(slices[i].x && slices[i].out, "aem_moe_forward_slices: slice %d (seq %llu) "
                    "has a NULL buffer", i, (unsigned long long)slices[i].seq_id);
        aligned = aligned && (reinterpret_cast<uintptr_t>(slices[i].x) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(slices[i].out) & 15) == 0;
        rows.push_back({static_cast<const char*>(slices[i].x), static_cast<char*>(slices[i].out), T});
        T += slices[i].tokens;
    }
    AEM_REQUIRE(T < (1ll << 28), "aem_moe_forward_slices: %lld tokens in one iteration",
                (long long)T);
    if (T == 0) return AEM_OK;
    AEM_TRY_CUDA(cudaSetDevice(m->gate->device));
    const int n = static_cast<int>(rows.size());
    AEM_TRY(aem::seam_reserve(m, T, in_row, out_row, n, s));
    aem::SeamStage* st = m->seam;
    // the pinned table this call fills was last read by a copy two calls ago
    const int b = st->flip;
    st->flip ^= 1;
    AEM_TRY_CUDA(cudaEventSynchronize(st->table_done[b]));
    std::copy(rows.begin(), rows.end(), st->h_table[b]);
    AEM_TRY_CUDA(cudaMemcpyAsync(st->d_table, st->h_table[b], sizeof(aem::SliceRow) * n,
                                 cudaMemcpyHostToDevice, s));
    AEM_TRY_CUDA(cudaEventRecord(st->table_done[b], s));
    const int sms = aem::sm_count(st->device);
    const unsigned g = static_cast<unsigned>(
        std::min<int64_t>((T + 7) / 8, static_cast<int64_t>(sms) * 8));
    aem::seam_copy_kernel<<<g, aem::kSeamThreads, 0, s>>>(st->d_table, n, T, in_row, st->rows_in,
                                                          1, aligned ? 1 : 0);
    AEM_CHECK_LAUNCH();
    aem::count_launches(1);
    AEM_TRY(m->forward(st->rows_in, x_dtype, T, st->rows_out, out_dtype, s));
    aem::seam_copy_kernel<<<g, aem::kSeamThreads, 0, s>>>(st->d_table, n, T, out_row,
                                                          st->rows_out, 0, aligned ? 1 : 0);
    AEM_CHECK_LAUNCH();
    aem::count_launches(1);
    return AEM_OK;
}
