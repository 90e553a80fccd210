// Runs the reference's own C++ Router (src/orchestration/router.hpp, header-only)
// in-process -- TEST INFRASTRUCTURE ONLY, built into oracle/_ref by oracle/Makefile
// from the reference sources where they lie; no reference source is copied.
//
// A loopback ICollectiveTransport (collective_transport.hpp:37-51) answers each
// send() with the reference worker's placeholder compute
// (process_token_placeholder, worker_shard.hpp) so that Router::route_batch
// (router.hpp:67-100) runs unmodified: capacity assignment, scatter by shard,
// wire encode/decode (serialization.hpp), gather and reassembly.
#include <cstdint>
#include <deque>
#include <limits>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "orchestration/router.hpp"
#include "orchestration/worker_shard.hpp"

namespace ao = aether::orchestration;

namespace {

class LoopbackShard : public ao::ICollectiveTransport {
public:
    explicit LoopbackShard(uint32_t id) : id_(id) {}
    void send(const std::vector<uint8_t>& message) override {
        auto tokens = ao::decode_token_batch(message);
        std::vector<ao::RoutedResult> results;
        results.reserve(tokens.size());
        for (const auto& t : tokens) results.push_back(ao::process_token_placeholder(t, id_));
        pending_.push_back(ao::encode_result_batch(results));
    }
    std::vector<uint8_t> receive() override {
        if (pending_.empty()) throw ao::PeerClosedError();
        auto m = std::move(pending_.front());
        pending_.pop_front();
        return m;
    }
private:
    uint32_t id_;
    std::deque<std::vector<uint8_t>> pending_;
};

thread_local std::string g_err;

}  // namespace

extern "C" const char* ref_last_error() { return g_err.c_str(); }

// Routes n tokens through Router::route_batch with a contiguous expert->shard
// map (tests/test_orchestration.cpp:25-33).  capacity == UINT64_MAX: unlimited.
// Outputs effective_expert and processed_by_shard per batch position, and the
// negated first payload float (proves the payload crossed the wire intact).
extern "C" int ref_route_batch(const uint32_t* primary, const uint32_t* secondary,
                               const uint32_t* batch_position, const float* payload,
                               uint64_t n, uint64_t capacity, uint32_t num_experts,
                               uint32_t num_shards, uint32_t* effective_out,
                               uint32_t* shard_out, float* payload_out) {
    try {
        std::unordered_map<uint32_t, uint32_t> e2s;
        uint32_t per = num_experts / num_shards;
        for (uint32_t e = 0; e < num_experts; ++e) e2s[e] = e / per;
        std::vector<std::unique_ptr<LoopbackShard>> shards;
        std::unordered_map<uint32_t, ao::ICollectiveTransport*> tr;
        for (uint32_t s = 0; s < num_shards; ++s) {
            shards.emplace_back(new LoopbackShard(s));
            tr[s] = shards.back().get();
        }
        ao::RouterConfig cfg;
        cfg.expert_capacity = capacity == std::numeric_limits<uint64_t>::max()
                                  ? std::numeric_limits<size_t>::max()
                                  : static_cast<size_t>(capacity);
        ao::Router router(e2s, tr, cfg);
        std::vector<ao::RoutedToken> batch;
        batch.reserve(n);
        for (uint64_t i = 0; i < n; ++i)
            batch.emplace_back(i + 1, batch_position[i], primary[i], secondary[i],
                               std::vector<float>{payload ? payload[i] : 0.0f});
        auto results = router.route_batch(batch);
        for (uint64_t i = 0; i < results.size(); ++i) {
            effective_out[i] = results[i].effective_expert;
            shard_out[i] = results[i].processed_by_shard;
            if (payload_out) payload_out[i] = results[i].payload.empty() ? 0.0f : results[i].payload[0];
        }
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}
