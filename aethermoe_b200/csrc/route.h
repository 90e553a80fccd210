// Internal interface of the routing kernels (route.cu) used by the MoE layer
// and the expert-parallel layer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "aem.h"

namespace aem {

// Slot-major MoE routing of T tokens x k slots (see route.cu):
// capacity assignment (pass 1) and the expert-grouped permutation (pass 2).
struct MoeRouteArgs {
    const int32_t* idx = nullptr;  // gating output [T][ldi], ldi = k or k+1
    int64_t T = 0;
    int ldi = 0;
    int k = 0;
    int E = 0;
    uint64_t capacity = AEM_CAPACITY_UNLIMITED;
    const float* val = nullptr;     // gate weights [T][k]
    const int64_t* corr = nullptr;  // expert-parallel rank correction [k][E] (nullable)
    void* workspace = nullptr;      // moe_route_workspace(T, k, E) bytes
    uint32_t* eff_out = nullptr;    // effective expert per unit [T*k] (nullable)
    int* starts_out = nullptr;      // [E+1] first grouped row of each expert
    int32_t* src_token = nullptr;   // [T*k] grouped row -> token
    int32_t* rowmap = nullptr;      // [T*k] grouped row -> t*k + j
    float* rowscale = nullptr;      // [T*k] grouped row -> gate weight
    int32_t* dest_of = nullptr;     // [T*k] unit -> grouped row (nullable)
    // > 0: inside every expert's group, the units of tokens [0, half_T) come
    // first (each part in unit order); the capacity rule is unchanged
    int64_t half_T = 0;
};

int64_t route_chunks(int64_t n);
size_t moe_route_workspace(int64_t T, int k, int E);
aem_status route_moe(const MoeRouteArgs& a, cudaStream_t s);

}  // namespace aem
