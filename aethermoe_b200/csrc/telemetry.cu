// Per-step telemetry of the MoE layers, in the pattern of the reference's
// TelemetryRecorder / TelemetryFlusher (src/core/telemetry.hpp:131-250): a
// process-wide switch read once per step (one relaxed atomic load when off),
// samples pushed without waiting, statistics computed only when a snapshot is
// asked for.  A step's latency is its device time: a CUDA event pair around
// the step's launches on its stream, harvested once the end event completed
// (never waiting on an unfinished step).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <deque>
#include <map>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "runtime.h"

namespace aem {

namespace {

struct Pending {
    cudaEvent_t a, b;
    int metric;
    int device;
};

constexpr size_t kMaxPending = 65536;     // steps in flight before samples are dropped
constexpr size_t kMaxSamples = 1u << 22;  // kept per metric

struct Telemetry {
    std::atomic<bool> enabled{false};
    std::atomic<uint64_t> dropped{0};
    std::mutex mu;
    std::deque<Pending> pending;
    std::map<int, std::vector<cudaEvent_t>> pool;  // events are per device
    std::vector<uint64_t> samples[AEM_NUM_METRICS];

    cudaEvent_t take(int device) {
        auto& v = pool[device];
        if (!v.empty()) {
            cudaEvent_t e = v.back();
            v.pop_back();
            return e;
        }
        cudaEvent_t e = nullptr;
        if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
        return e;
    }

    // Moves every completed step into the samples (lock held).
    void harvest_locked() {
        for (auto it = pending.begin(); it != pending.end();) {
            const cudaError_t q = cudaEventQuery(it->b);
            if (q == cudaErrorNotReady) {
                ++it;
                continue;
            }
            float ms = 0.0f;
            if (q == cudaSuccess && cudaEventElapsedTime(&ms, it->a, it->b) == cudaSuccess) {
                auto& s = samples[it->metric];
                if (s.size() < kMaxSamples)
                    s.push_back(static_cast<uint64_t>(std::llround(static_cast<double>(ms) * 1e6)));
                else
                    dropped.fetch_add(1, std::memory_order_relaxed);
            } else {
                cudaGetLastError();  // a failed step is not a sample
            }
            pool[it->device].push_back(it->a);
            pool[it->device].push_back(it->b);
            it = pending.erase(it);
        }
    }
};

Telemetry& tel() {
    static Telemetry* t = new Telemetry();  // lives for the process (events outlive statics)
    return *t;
}

// Nearest-rank statistics (compute_stats, telemetry.hpp:88-113).
aem_metric_stats stats_of(std::vector<uint64_t>& v) {
    aem_metric_stats s{};
    s.count = v.size();
    if (s.count == 0) return s;
    std::sort(v.begin(), v.end());
    double sum = 0.0;
    for (uint64_t x : v) sum += static_cast<double>(x);
    s.mean_ns = sum / static_cast<double>(s.count);
    s.max_ns = static_cast<double>(v.back());
    auto pct = [&](double p) {
        size_t idx = static_cast<size_t>(std::ceil(p * static_cast<double>(s.count)));
        if (idx == 0) idx = 1;
        if (idx > s.count) idx = s.count;
        return static_cast<double>(v[idx - 1]);
    };
    s.p50_ns = pct(0.50);
    s.p95_ns = pct(0.95);
    s.p99_ns = pct(0.99);
    return s;
}

}  // namespace

StepTimer::StepTimer(int metric, cudaStream_t s) : metric_(metric), stream_(s) {
    Telemetry& t = tel();
    if (!t.enabled.load(std::memory_order_relaxed)) return;
    device_ = current_device();
    std::lock_guard<std::mutex> lk(t.mu);
    if (t.pending.size() >= kMaxPending) {
        t.harvest_locked();
        if (t.pending.size() >= kMaxPending) {
            t.dropped.fetch_add(1, std::memory_order_relaxed);
            return;
        }
    }
    a_ = t.take(device_);
    b_ = t.take(device_);
    if (!a_ || !b_ || cudaEventRecord(a_, s) != cudaSuccess) {
        if (a_) t.pool[device_].push_back(a_);
        if (b_) t.pool[device_].push_back(b_);
        a_ = b_ = nullptr;
        cudaGetLastError();
    }
}

StepTimer::~StepTimer() {
    if (!a_) return;
    Telemetry& t = tel();
    std::lock_guard<std::mutex> lk(t.mu);
    if (cudaEventRecord(b_, stream_) != cudaSuccess) {
        cudaGetLastError();
        t.pool[device_].push_back(a_);
        t.pool[device_].push_back(b_);
        return;
    }
    t.pending.push_back({a_, b_, metric_, device_});
    if (t.pending.size() > 64) t.harvest_locked();  // keep the queue short, never wait
}

}  // namespace aem

using aem::set_error;

extern "C" {

void aem_telemetry_enable(int enabled) {
    aem::tel().enabled.store(enabled != 0, std::memory_order_relaxed);
}

int aem_telemetry_enabled(void) { return aem::tel().enabled.load(std::memory_order_relaxed); }

aem_status aem_telemetry_snapshot(int metric, aem_metric_stats* out, uint64_t* dropped) {
    AEM_REQUIRE(out != nullptr, "aem_telemetry_snapshot: out is NULL");
    AEM_REQUIRE(metric >= 0 && metric < AEM_NUM_METRICS, "aem_telemetry_snapshot: bad metric %d",
                metric);
    aem::Telemetry& t = aem::tel();
    std::vector<uint64_t> copy;
    {
        std::lock_guard<std::mutex> lk(t.mu);
        t.harvest_locked();
        copy = t.samples[metric];
    }
    *out = aem::stats_of(copy);
    if (dropped) *dropped = t.dropped.load(std::memory_order_relaxed);
    return AEM_OK;
}

aem_status aem_telemetry_reset(void) {
    aem::Telemetry& t = aem::tel();
    std::lock_guard<std::mutex> lk(t.mu);
    t.harvest_locked();
    for (auto& s : t.samples) s.clear();
    t.dropped.store(0, std::memory_order_relaxed);
    return AEM_OK;
}

aem_status aem_metric_stats_of(const uint64_t* latencies_ns, int64_t n, aem_metric_stats* out) {
    AEM_REQUIRE(out != nullptr && (n == 0 || latencies_ns != nullptr),
                "aem_metric_stats_of: NULL argument");
    AEM_REQUIRE(n >= 0, "aem_metric_stats_of: n < 0");
    std::vector<uint64_t> v(latencies_ns, latencies_ns + n);
    *out = aem::stats_of(v);
    return AEM_OK;
}

}  // extern "C"
