// Generator: the reference's continuous-batching engine loop
// (ContinuousBatchingEngine::engine_loop, src/engine.cpp:163-246) on one GPU:
// schedule_step -> forward_batch over running() -> process_step_outputs, with
// the KV arena, the block allocator and the metadata upload of the
// AttentionEngine and the forward pass of the DeviceModel. Per step the host
// does the scheduling and one metadata + token upload; the device does the
// whole forward; the sampled ids come back in one download (the scheduler
// needs them before the next step, as in the reference).
//
// Telemetry follows the reference's AtomicEngineMetrics / MetricsSnapshot
// (include/nano_vllm/engine.hpp:29-60, src/engine.cpp:8-38, :119-161).
#pragma once

#include <cstdint>
#include <cstdio>
#include <expected>
#include <functional>
#include <optional>
#include <string>
#include <unordered_map>
#include <vector>

#include "engine.hpp"
#include "model.hpp"
#include "scheduler.hpp"

namespace nvllm {

struct Metrics {
    double uptime_secs = 0.0;
    uint64_t total_requests_received = 0;
    uint64_t total_requests_completed = 0;
    uint64_t total_tokens_generated = 0;
    double throughput_tokens_per_sec = 0.0;
    std::size_t active_batch_size = 0;
    std::size_t waiting_queue_depth = 0;
    std::size_t kv_cache_used_blocks = 0;
    std::size_t kv_cache_total_blocks = 0;
    double kv_cache_utilization_pct = 0.0;
    double avg_ttft_ms = 0.0;
    double avg_iteration_latency_ms = 0.0;
    uint64_t total_preemptions = 0;
    uint64_t total_iterations = 0;
    uint64_t total_tokens_computed = 0;  // flattened rows through the forward pass
    uint64_t h2d_bytes = 0, d2h_bytes = 0, kernel_launches = 0;

    // The reference's MetricsSnapshot::to_json layout (src/engine.cpp:8-38).
    std::string to_json() const;
};

// The running batch in the trace record layout:
//   -1, step, n, then per sequence in running() order
//   seq_id, num_computed, total_len, last token, table_len, table..., n_uncomputed, uncomputed...
void append_batch_record(const Scheduler& s, int64_t step, std::vector<int64_t>& out);

// One sampled token of one sequence, as the reference streams it to its client
// (TokenStreamEvent, include/nano_vllm/scheduler.hpp:24-30): finished on the
// sequence's last token, the time to first token (from arrival) on its first.
struct TokenEvent {
    SeqId seq_id = 0;
    int64_t token = 0;
    bool finished = false;
    std::optional<uint64_t> ttft_us{};
};
using TokenSink = std::function<void(const TokenEvent&)>;

class Generator {
public:
    Generator(AttentionEngine& eng, DeviceModel& model, const SchedulerConfig& cfg,
              int32_t precision);
    ~Generator();

    void add_request(SeqId id, std::vector<int64_t> prompt, std::size_t max_new_tokens);
    // One iteration. batch_size 0 with work pending means nothing could be
    // admitted (a request larger than the arena).
    std::expected<StepSummary, EngineError> step();
    // Steps until no work is pending (or max_steps > 0 steps ran).
    std::expected<int64_t, EngineError> run(int64_t max_steps);
    bool has_pending_work() const noexcept { return sched_.has_pending_work(); }
    // Rows still to run through the forward pass for the sequences it holds:
    // their uncomputed tokens plus the tokens still to generate (the router's
    // load measure).
    std::size_t outstanding_tokens() const noexcept;
    int32_t device() const noexcept { return eng_.config().device; }

    // Token list (prompt + generated) of a finished sequence, or nullptr.
    const std::vector<int64_t>* output(SeqId id) const;
    Metrics metrics() const;
    // Records every following step to `path` in the reference trace format
    // (the batch record, then -2, the sampled ids and per sequence the top-2
    // margin and the 8 largest logits as (index, float bits)); "" stops.
    bool set_trace(const std::string& path);
    const Scheduler& scheduler() const noexcept { return sched_; }
    // Called after every step with each sampled token, in batch order (the
    // reference pushes them from process_step_outputs, src/scheduler.cpp:132-165).
    void set_token_sink(TokenSink sink) { sink_ = std::move(sink); }

private:
    AttentionEngine& eng_;
    DeviceModel& model_;
    Scheduler sched_;
    int32_t precision_;
    Clock::time_point start_;
    std::unordered_map<SeqId, std::vector<int64_t>> done_;
    // per-step scratch
    std::vector<SequenceView> views_;
    std::vector<int64_t> tokens_, prev_, sampled_;
    std::vector<float> margins_, top_val_;
    std::vector<int32_t> top_idx_;
    std::vector<Sequence> retired_;
    std::vector<int64_t> record_;
    std::FILE* trace_ = nullptr;
    TokenSink sink_;
    std::vector<SeqId> ev_ids_;
    std::vector<uint8_t> ev_first_;
    int64_t step_index_ = 0;
    // telemetry
    uint64_t received_ = 0, tokens_generated_ = 0, iterations_ = 0, ttft_samples_ = 0;
    uint64_t tokens_computed_ = 0;
    uint64_t launches0_ = 0, h2d0_ = 0, d2h0_ = 0;  // model counters at construction
    double step_us_ = 0.0, ttft_us_ = 0.0;
};

}  // namespace nvllm
