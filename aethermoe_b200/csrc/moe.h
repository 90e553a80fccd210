// Internal interface of the single-GPU MoE layer (moe.cu), reused by the
// expert-parallel layer for its local expert FFN.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "aem.h"
#include "runtime.h"

namespace aem {

// X[r] = x[src[r]] as bf16 (lo: the float32 pair's low half); also zeroes
// zero1[0, zero1_n) and zero2[0, zero2_n) (float counts, multiples of 4,
// 16-byte aligned) in the same launch.
aem_status gather_rows(const void* x, aem_dtype xd, const int32_t* src, int64_t rows, int64_t d,
                       void* out, cudaStream_t s, void* out_lo = nullptr,
                       float* zero1 = nullptr, int64_t zero1_n = 0, float* zero2 = nullptr,
                       int64_t zero2_n = 0);
aem_status combine_rows(const float* y, int64_t T, int k, int64_t d, void* out, aem_dtype od,
                        cudaStream_t s);

struct Moe {
    aem_moe_config cfg{};
    Gate* gate = nullptr;
    QWeight* up = nullptr;
    QWeight* down = nullptr;
    int64_t T_cap = 0;
    int64_t last_T = 0;
    void* buf = nullptr;
    int32_t* idx = nullptr;
    float* val = nullptr;
    void* route_ws = nullptr;
    uint32_t* eff = nullptr;
    int* starts = nullptr;
    int32_t* src_token = nullptr;
    int32_t* rowmap = nullptr;
    float* rowscale = nullptr;
    void* xperm = nullptr;  // bf16 [U, d]
    void* h = nullptr;      // bf16 [U, ffn]
    float* y = nullptr;     // f32 [T*k, d]
    // split-precision operands (float32 x, float32-class hidden activation):
    // the low halves of the bf16 pairs, allocated on the first step that needs them
    int hidden_dtype = -1;  // -1: follow x's dtype; AEM_F32: bf16 pair; AEM_BF16: bf16
    void* split_buf = nullptr;
    int64_t split_cap = 0;
    void* xperm_lo = nullptr;  // bf16 [U, d]
    void* h_lo = nullptr;      // bf16 [U, ffn]
    // decode steps (at most gemv_max_rows() units): the up projection's
    // float32 pre-activations [U, ffn], summed over K ranges
    float* h32 = nullptr;
    PhaseProfiler prof;
    // scheduler seam (seam.cu): staged rows of one iteration and its slice table
    struct SeamStage* seam = nullptr;

    // Routing buffers for T tokens, plus the expert-FFN buffers (xperm, h, y)
    // unless expert_buffers is false (the expert-parallel layer has its own).
    aem_status reserve(int64_t T, bool expert_buffers = true);
    aem_status reserve_split(int64_t T);
    aem_status forward(const void* x, aem_dtype xd, int64_t T, void* out, aem_dtype od,
                       cudaStream_t s);
    // Grouped up GEMM + ReLU, grouped down GEMM (scaled by the gate weight,
    // scattered to row t*k+j), combine -- on xperm/starts/rowmap/rowscale.
    // acc_zeroed / h32_zeroed: the float32 output rows / decode pre-activations
    // were zeroed already (by the gather's launch)
    aem_status expert_ffn(int64_t T, int64_t U, void* out, aem_dtype od, cudaStream_t s,
                          bool split_x = false, bool split_h = false, bool acc_zeroed = false,
                          bool h32_zeroed = false);
};

void seam_free(Moe* m);  // releases the scheduler seam's buffers (seam.cu)

}  // namespace aem
