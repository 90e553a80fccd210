// Library runtime: error reporting, per-device error words, device queries,
// TMA descriptor encoding and the host-staging context of the *_host calls.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "runtime.h"

namespace aem {

namespace {
thread_local std::string g_last_error;
std::mutex g_dev_mutex;
int* g_err_words[64] = {nullptr};
int g_sm_counts[64] = {0};
int g_is_sm100[64] = {-1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1,
                      -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1,
                      -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1,
                      -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
}  // namespace

void set_error(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

const char* last_error_cstr() { return g_last_error.c_str(); }

int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

static void query_device(int device) {
    if (device < 0 || device >= 64) return;
    if (g_is_sm100[device] >= 0) return;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
        g_is_sm100[device] = 0;
        g_sm_counts[device] = 0;
        return;
    }
    g_sm_counts[device] = prop.multiProcessorCount;
    g_is_sm100[device] = (prop.major == 10 && prop.minor == 0) ? 1 : 0;
}

int sm_count(int device) {
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    query_device(device);
    return device >= 0 && device < 64 ? g_sm_counts[device] : 0;
}

bool is_sm100(int device) {
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    query_device(device);
    return device >= 0 && device < 64 && g_is_sm100[device] == 1;
}

int* device_error_word(int device) {
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    if (device < 0 || device >= 64) return nullptr;
    if (!g_err_words[device]) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        int* p = nullptr;
        if (cudaMalloc(&p, sizeof(int)) == cudaSuccess) {
            cudaMemset(p, 0, sizeof(int));
            cudaDeviceSynchronize();
            g_err_words[device] = p;
        }
        cudaSetDevice(prev);
    }
    return g_err_words[device];
}

aem_status check_device_errors(cudaStream_t stream, const char* what) {
    AEM_TRY_CUDA(cudaStreamSynchronize(stream));
    int* w = device_error_word(current_device());
    if (!w) {
        set_error("%s: no device error word", what);
        return AEM_ENOMEM;
    }
    int bits = 0;
    AEM_TRY_CUDA(cudaMemcpyAsync(&bits, w, sizeof(int), cudaMemcpyDeviceToHost, stream));
    AEM_TRY_CUDA(cudaStreamSynchronize(stream));
    if (bits == 0) return AEM_OK;
    AEM_TRY_CUDA(cudaMemsetAsync(w, 0, sizeof(int), stream));
    AEM_TRY_CUDA(cudaStreamSynchronize(stream));
    if (bits & ERR_GEMM_TIMEOUT) {
        set_error("%s: a bounded device wait timed out (error bits 0x%x)", what, bits);
        return AEM_ETIMEOUT;
    }
    if (bits & (ERR_EP_PEER_TIMEOUT | ERR_EP_PEER_FAILED)) {
        set_error("%s: an expert-parallel peer %s (error bits 0x%x)", what,
                  (bits & ERR_EP_PEER_TIMEOUT) ? "did not signal within the deadline"
                                               : "reported a failed step",
                  bits);
        return AEM_ETIMEOUT;
    }
    if (bits & ERR_ROUTE_POSITION) {
        set_error("%s: batch_position is not a permutation of [0, n) (error bits 0x%x)", what,
                  bits);
        return AEM_EDEVICE;
    }
    if (bits & ERR_ROUTE_EXPERT) {
        set_error("%s: expert id out of range (error bits 0x%x)", what, bits);
        return AEM_EDEVICE;
    }
    if (bits & ERR_EP_PLAN) {
        set_error("%s: expert-parallel step exceeds the receive capacity (error bits 0x%x)",
                  what, bits);
        return AEM_EDEVICE;
    }
    set_error("%s: in-kernel check failed (error bits 0x%x)", what, bits);
    return AEM_EDEVICE;
}

aem_status make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                        int elem_bytes, uint64_t cols, uint64_t rows, uint32_t box_cols,
                        uint32_t box_rows, CUtensorMapSwizzle swizzle) {
    {
        std::lock_guard<std::mutex> lk(g_dev_mutex);
        if (!g_encode) {
            void* fn = nullptr;
            cudaDriverEntryPointQueryResult q;
            cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn,
                                                    cudaEnableDefault, &q);
            if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
                set_error("cuTensorMapEncodeTiled unavailable");
                return AEM_EUNSUPPORTED;
            }
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        }
    }
    AEM_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0,
                "TMA base address must be 16-byte aligned");
    AEM_REQUIRE((cols * elem_bytes) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * static_cast<cuuint64_t>(elem_bytes)};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d): cols=%llu rows=%llu box=%ux%u", (int)r,
                  (unsigned long long)cols, (unsigned long long)rows, box_cols, box_rows);
        return AEM_ECUDA;
    }
    return AEM_OK;
}

// ------------------------------------------------------------------ launch counter
namespace {
std::atomic<uint64_t> g_launches{0};
}
void count_launches(int n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }

// ------------------------------------------------------------------ profiler
cudaEvent_t PhaseProfiler::take() {
    if (!pool.empty()) {
        cudaEvent_t e = pool.back();
        pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void PhaseProfiler::begin(int phase, cudaStream_t s) {
    if (!on) return;
    cudaEvent_t e = take();
    cudaEventRecord(e, s);
    open_ev[phase] = e;
}

void PhaseProfiler::end(int phase, cudaStream_t s) {
    if (!on || !open_ev[phase]) return;
    cudaEvent_t e = take();
    cudaEventRecord(e, s);
    pending[phase].emplace_back(open_ev[phase], e);
    open_ev[phase] = nullptr;
}

void PhaseProfiler::enable(bool e) {
    on = e;
    steps = 0;
    for (int p = 0; p < AEM_NUM_PHASES; ++p) {
        acc_ms[p] = 0;
        for (auto& pr : pending[p]) {
            pool.push_back(pr.first);
            pool.push_back(pr.second);
        }
        pending[p].clear();
    }
}

aem_status PhaseProfiler::read(double* ms, int64_t* nsteps) {
    for (int p = 0; p < AEM_NUM_PHASES; ++p) {
        for (auto& pr : pending[p]) {
            AEM_TRY_CUDA(cudaEventSynchronize(pr.second));
            float t = 0.0f;
            AEM_TRY_CUDA(cudaEventElapsedTime(&t, pr.first, pr.second));
            acc_ms[p] += t;
            pool.push_back(pr.first);
            pool.push_back(pr.second);
        }
        pending[p].clear();
        if (ms) ms[p] = acc_ms[p];
    }
    if (nsteps) *nsteps = steps;
    return AEM_OK;
}

PhaseProfiler::~PhaseProfiler() {
    for (int p = 0; p < AEM_NUM_PHASES; ++p)
        for (auto& pr : pending[p]) {
            cudaEventDestroy(pr.first);
            cudaEventDestroy(pr.second);
        }
    for (auto e : pool) cudaEventDestroy(e);
}

// ------------------------------------------------------------------ context
aem_status Context::reserve_device(size_t bytes) {
    if (bytes <= dev_bytes) return AEM_OK;
    if (dev) {
        AEM_TRY_CUDA(cudaStreamSynchronize(stream));
        cudaFree(dev);
        dev = nullptr;
        dev_bytes = 0;
    }
    size_t want = bytes + bytes / 4 + 4096;
    AEM_TRY_CUDA(cudaMalloc(&dev, want));
    dev_bytes = want;
    return AEM_OK;
}

aem_status Context::reserve_host(size_t bytes) {
    if (bytes <= host_bytes) return AEM_OK;
    if (host) {
        AEM_TRY_CUDA(cudaStreamSynchronize(stream));
        cudaFreeHost(host);
        host = nullptr;
        host_bytes = 0;
    }
    size_t want = bytes + bytes / 4 + 4096;
    AEM_TRY_CUDA(cudaMallocHost(&host, want));
    host_bytes = want;
    return AEM_OK;
}

}  // namespace aem

using aem::set_error;

extern "C" {

const char* aem_last_error(void) { return aem::last_error_cstr(); }

const char* aem_version(void) { return "aethermoe-b200 0.1.0 (sm_100a)"; }

uint64_t aem_kernel_launches(void) { return aem::g_launches.load(std::memory_order_relaxed); }

int aem_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int c = 0;
    for (int d = 0; d < n; ++d)
        if (aem::is_sm100(d)) ++c;
    return c;
}

aem_status aem_context_create(int device, aem_context_t* out) {
    AEM_REQUIRE(out != nullptr, "aem_context_create: out is NULL");
    *out = nullptr;
    if (!aem::is_sm100(device)) {
        set_error("aem_context_create: device %d is not an sm_100 (B200) GPU", device);
        return AEM_EUNSUPPORTED;
    }
    AEM_TRY_CUDA(cudaSetDevice(device));
    auto* c = new aem::Context();
    c->device = device;
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete c;
        set_error("aem_context_create: cudaStreamCreate failed: %s", cudaGetErrorString(e));
        return AEM_ECUDA;
    }
    *out = reinterpret_cast<aem_context_t>(c);
    return AEM_OK;
}

aem_status aem_context_destroy(aem_context_t ctx) {
    if (!ctx) return AEM_OK;
    auto* c = reinterpret_cast<aem::Context*>(ctx);
    cudaSetDevice(c->device);
    aem::pipe_free(c);
    cudaStreamSynchronize(c->stream);
    if (c->dev) cudaFree(c->dev);
    if (c->host) cudaFreeHost(c->host);
    cudaStreamDestroy(c->stream);
    delete c;
    return AEM_OK;
}

void* aem_context_stream(aem_context_t ctx) {
    return ctx ? reinterpret_cast<aem::Context*>(ctx)->stream : nullptr;
}

aem_status aem_device_status(void* stream) {
    return aem::check_device_errors(static_cast<cudaStream_t>(stream), "aem_device_status");
}

}  // extern "C"
