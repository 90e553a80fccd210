// Asynchronous host-buffer layer steps: the next step's host -> device copy
// and the previous step's device -> host copy run on their own streams (the
// GPU's two copy engines) while the current step computes.
//
// A context owns three slots, each a device input and output buffer and three
// events.  submit(step i) takes slot i % 3:
//   1. waits on the host until the slot's previous step (i - 3) has been
//      copied back -- then nothing reads or writes the slot any more;
//   2. copies the step's input in on the upload stream;
//   3. computes on the context's stream once the upload is done;
//   4. copies the output back on the download stream once the compute is done,
//      and the device error word beside it (so a wait need not synchronise
//      the compute stream, which is already busy with the next step).
// wait(ticket) waits for step's download and reports what its kernels
// recorded.  With pinned host buffers a step's copies overlap the
// neighbouring steps' compute; pageable buffers still work, serialised.
// Three slots, not two: with two, step i + 1's upload could only start once
// step i - 1's download had finished (they share a slot), so a step cost a
// download plus an upload (2.2-2.4 ms for 64 MiB each way at the bench
// size) instead of its 1.7 ms of compute; with three, a caller that waits
// for step i - 2 after submitting step i keeps the compute stream busy.
#include <cuda_runtime.h>

#include "common.cuh"
#include "moe.h"
#include "runtime.h"

namespace aem {

constexpr int kPipeSlots = 3;

struct HostPipe {
    cudaStream_t up = nullptr, down = nullptr;
    struct Slot {
        void* din = nullptr;
        void* dout = nullptr;
        size_t din_bytes = 0, dout_bytes = 0;
        cudaEvent_t uploaded = nullptr, computed = nullptr, downloaded = nullptr;
        uint64_t ticket = 0;
        bool busy = false;
    } slot[kPipeSlots];
    int* err_host = nullptr;  // pinned [kPipeSlots]: the error word after each slot's step
    uint64_t next = 1;
};

void pipe_free(Context* c) {
    HostPipe* p = c->pipe;
    if (!p) return;
    cudaSetDevice(c->device);
    if (p->up) cudaStreamSynchronize(p->up);
    if (p->down) cudaStreamSynchronize(p->down);
    cudaStreamSynchronize(c->stream);
    for (auto& s : p->slot) {
        cudaFree(s.din);
        cudaFree(s.dout);
        if (s.uploaded) cudaEventDestroy(s.uploaded);
        if (s.computed) cudaEventDestroy(s.computed);
        if (s.downloaded) cudaEventDestroy(s.downloaded);
    }
    if (p->err_host) cudaFreeHost(p->err_host);
    if (p->up) cudaStreamDestroy(p->up);
    if (p->down) cudaStreamDestroy(p->down);
    delete p;
    c->pipe = nullptr;
}

namespace {

aem_status pipe_get(Context* c, HostPipe** out) {
    if (!c->pipe) {
        auto* p = new HostPipe();
        c->pipe = p;  // pipe_free releases whatever was created if a step below fails
        AEM_TRY_CUDA(cudaStreamCreateWithFlags(&p->up, cudaStreamNonBlocking));
        AEM_TRY_CUDA(cudaStreamCreateWithFlags(&p->down, cudaStreamNonBlocking));
        for (auto& s : p->slot) {
            AEM_TRY_CUDA(cudaEventCreateWithFlags(&s.uploaded, cudaEventDisableTiming));
            AEM_TRY_CUDA(cudaEventCreateWithFlags(&s.computed, cudaEventDisableTiming));
            AEM_TRY_CUDA(cudaEventCreateWithFlags(&s.downloaded, cudaEventDisableTiming));
        }
        AEM_TRY_CUDA(cudaMallocHost(&p->err_host, kPipeSlots * sizeof(int)));
        for (int i = 0; i < kPipeSlots; ++i) p->err_host[i] = 0;
    }
    *out = c->pipe;
    return AEM_OK;
}

aem_status grow(void** buf, size_t* have, size_t want) {
    if (want <= *have) return AEM_OK;
    cudaFree(*buf);
    *buf = nullptr;
    *have = 0;
    AEM_TRY_CUDA(cudaMalloc(buf, want));
    *have = want;
    return AEM_OK;
}

}  // namespace

aem_status pipe_submit(Context* c, const void* x, size_t xb, void* out, size_t ob,
                       const std::function<aem_status(const void*, void*, cudaStream_t)>& compute,
                       uint64_t* ticket) {
    AEM_TRY_CUDA(cudaSetDevice(c->device));
    HostPipe* p = nullptr;
    AEM_TRY(pipe_get(c, &p));
    const int si = static_cast<int>(p->next % kPipeSlots);
    auto& s = p->slot[si];
    if (s.busy) {
        // the slot's previous step: downloaded, so its buffers are free
        AEM_TRY_CUDA(cudaEventSynchronize(s.downloaded));
        s.busy = false;
    }
    AEM_TRY(grow(&s.din, &s.din_bytes, xb));
    AEM_TRY(grow(&s.dout, &s.dout_bytes, ob));
    int* err = device_error_word(c->device);
    AEM_REQUIRE(err != nullptr, "pipelined step: no device error word");
    if (xb) AEM_TRY_CUDA(cudaMemcpyAsync(s.din, x, xb, cudaMemcpyHostToDevice, p->up));
    AEM_TRY_CUDA(cudaEventRecord(s.uploaded, p->up));
    AEM_TRY_CUDA(cudaStreamWaitEvent(c->stream, s.uploaded, 0));
    AEM_TRY(compute(s.din, s.dout, c->stream));
    AEM_TRY_CUDA(cudaMemcpyAsync(&p->err_host[si], err, sizeof(int), cudaMemcpyDeviceToHost,
                                 c->stream));
    AEM_TRY_CUDA(cudaEventRecord(s.computed, c->stream));
    AEM_TRY_CUDA(cudaStreamWaitEvent(p->down, s.computed, 0));
    if (ob) AEM_TRY_CUDA(cudaMemcpyAsync(out, s.dout, ob, cudaMemcpyDeviceToHost, p->down));
    AEM_TRY_CUDA(cudaEventRecord(s.downloaded, p->down));
    s.ticket = p->next;
    s.busy = true;
    *ticket = p->next++;
    return AEM_OK;
}

aem_status pipe_wait(Context* c, uint64_t ticket) {
    HostPipe* p = c->pipe;
    AEM_REQUIRE(p != nullptr && ticket != 0 && ticket < p->next,
                "pipelined wait: ticket %llu was never submitted on this context",
                (unsigned long long)ticket);
    const int si = static_cast<int>(ticket % kPipeSlots);
    auto& s = p->slot[si];
    if (s.ticket != ticket) return AEM_OK;  // slot reused: that step was waited for already
    AEM_TRY_CUDA(cudaSetDevice(c->device));
    AEM_TRY_CUDA(cudaEventSynchronize(s.downloaded));
    s.busy = false;
    if (p->err_host[si] != 0) {
        p->err_host[si] = 0;
        return check_device_errors(c->stream, "pipelined step");
    }
    return AEM_OK;
}

}  // namespace aem

using aem::set_error;

extern "C" {

aem_status aem_moe_submit_host(aem_context_t ctx, aem_moe_t moe, const void* x, aem_dtype x_dtype,
                               int64_t T, void* out, aem_dtype out_dtype, uint64_t* ticket) {
    AEM_REQUIRE(ctx != nullptr && moe != nullptr && ticket != nullptr,
                "aem_moe_submit_host: NULL argument");
    AEM_REQUIRE(T >= 1 && T < (1ll << 28), "aem_moe_submit_host: T=%lld out of range",
                (long long)T);
    AEM_REQUIRE(x && out, "aem_moe_submit_host: NULL buffer");
    AEM_REQUIRE(x_dtype == AEM_F32 || x_dtype == AEM_BF16, "aem_moe_submit_host: bad x dtype");
    AEM_REQUIRE(out_dtype == AEM_F32 || out_dtype == AEM_BF16,
                "aem_moe_submit_host: bad out dtype");
    auto* c = reinterpret_cast<aem::Context*>(ctx);
    auto* m = reinterpret_cast<aem::Moe*>(moe);
    const size_t xb = static_cast<size_t>(T) * m->cfg.d_model * (x_dtype == AEM_F32 ? 4 : 2);
    const size_t ob = static_cast<size_t>(T) * m->cfg.d_model * (out_dtype == AEM_F32 ? 4 : 2);
    return aem::pipe_submit(
        c, x, xb, out, ob,
        [&](const void* din, void* dout, cudaStream_t s) {
            return m->forward(din, x_dtype, T, dout, out_dtype, s);
        },
        ticket);
}

aem_status aem_context_wait(aem_context_t ctx, uint64_t ticket) {
    AEM_REQUIRE(ctx != nullptr, "aem_context_wait: NULL context");
    return aem::pipe_wait(reinterpret_cast<aem::Context*>(ctx), ticket);
}

}  // extern "C"
