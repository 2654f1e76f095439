#include "generator.hpp"

#include <algorithm>
#include <bit>
#include <cstring>
#include <format>

namespace nvllm {

namespace {
constexpr int32_t kTraceTopK = 8;

int64_t float_bits(float x) { return int64_t(std::bit_cast<uint32_t>(x)); }

// the power of two at or above x (x >= 1), at most cap
int32_t bucket(std::size_t x, int32_t cap) {
    const std::size_t b = std::bit_ceil(std::max<std::size_t>(x, 1));
    return int32_t(std::min<std::size_t>(b, std::size_t(cap)));
}
}  // namespace

std::string Metrics::to_json() const {
    return std::format(
        "{{\n"
        "  \"uptime_secs\": {:.3f},\n"
        "  \"total_requests_received\": {},\n"
        "  \"total_requests_completed\": {},\n"
        "  \"total_tokens_generated\": {},\n"
        "  \"throughput_tokens_per_sec\": {:.2f},\n"
        "  \"active_batch_size\": {},\n"
        "  \"waiting_queue_depth\": {},\n"
        "  \"kv_cache_used_blocks\": {},\n"
        "  \"kv_cache_total_blocks\": {},\n"
        "  \"kv_cache_utilization_pct\": {:.2f},\n"
        "  \"avg_ttft_ms\": {:.3f},\n"
        "  \"avg_iteration_latency_ms\": {:.3f},\n"
        "  \"total_preemptions\": {}\n"
        "}}",
        uptime_secs, total_requests_received, total_requests_completed, total_tokens_generated,
        throughput_tokens_per_sec, active_batch_size, waiting_queue_depth, kv_cache_used_blocks,
        kv_cache_total_blocks, kv_cache_utilization_pct, avg_ttft_ms, avg_iteration_latency_ms,
        total_preemptions);
}

void append_batch_record(const Scheduler& s, int64_t step, std::vector<int64_t>& out) {
    const auto& run = s.running();
    out.push_back(-1);
    out.push_back(step);
    out.push_back(int64_t(run.size()));
    for (const Sequence& seq : run) {
        out.push_back(int64_t(seq.id));
        out.push_back(int64_t(seq.num_computed));
        out.push_back(int64_t(seq.total_len()));
        out.push_back(seq.tokens.empty() ? 0 : seq.tokens.back());
        out.push_back(int64_t(seq.table.size()));
        for (const BlockId b : seq.table) out.push_back(int64_t(b));
        const auto unc = seq.uncomputed();
        out.push_back(int64_t(unc.size()));
        out.insert(out.end(), unc.begin(), unc.end());
    }
}

Generator::Generator(AttentionEngine& eng, DeviceModel& model, const SchedulerConfig& cfg,
                     int32_t precision)
    : eng_(eng),
      model_(model),
      sched_(cfg, std::size_t(eng.config().layout.block_size)),
      precision_(precision),
      start_(Clock::now()),
      launches0_(model.kernel_launches()),
      h2d0_(model.h2d_bytes()),
      d2h0_(model.d2h_bytes()) {}

Generator::~Generator() {
    if (trace_ != nullptr) std::fclose(trace_);
}

void Generator::add_request(SeqId id, std::vector<int64_t> prompt, std::size_t max_new_tokens) {
    sched_.add_request(Sequence(id, std::move(prompt), max_new_tokens));
    ++received_;
}

std::size_t Generator::outstanding_tokens() const noexcept {
    auto rows = [](const Sequence& q) {
        const std::size_t left = q.max_new_tokens > q.generated_len()
                                     ? q.max_new_tokens - q.generated_len() : 0;
        return (q.total_len() - q.num_computed) + left;
    };
    std::size_t n = 0;
    for (const Sequence& q : sched_.running()) n += rows(q);
    for (const Sequence& q : sched_.waiting()) n += rows(q);
    return n;
}

bool Generator::set_trace(const std::string& path) {
    if (trace_ != nullptr) {
        std::fclose(trace_);
        trace_ = nullptr;
    }
    if (path.empty()) return true;
    trace_ = std::fopen(path.c_str(), "wb");
    step_index_ = 0;
    return trace_ != nullptr;
}

std::expected<StepSummary, EngineError> Generator::step() {
    const auto t0 = Clock::now();
    BlockAllocator& blocks = eng_.allocator();
    StepSummary sum = sched_.schedule_step(blocks);
    if (sum.batch_size == 0) return sum;

    const auto& run = sched_.running();
    const std::size_t n = run.size();
    views_.clear();
    tokens_.clear();
    prev_.resize(n);
    for (std::size_t i = 0; i < n; ++i) {
        const Sequence& seq = run[i];
        views_.push_back(SequenceView{int32_t(seq.num_computed), int32_t(seq.total_len()),
                                      std::span<const BlockId>(seq.table)});
        const auto unc = seq.uncomputed();
        tokens_.insert(tokens_.end(), unc.begin(), unc.end());
        prev_[i] = seq.tokens.back();  // tokens is never empty
    }
    // small steps are padded to a (sequences, tokens) bucket so that the model
    // replays one captured CUDA graph per bucket
    int32_t pad_seqs = 0, pad_tokens = 0;
    const int32_t graph_max = model_.config().graph_max_tokens;
    if (graph_max > 0 && tokens_.size() <= std::size_t(graph_max)) {
        pad_seqs = bucket(n, eng_.config().max_seqs);
        pad_tokens = bucket(tokens_.size(), eng_.config().max_tokens);
    }
    if (auto r = eng_.begin_step(views_, pad_seqs, pad_tokens); !r) {
        return std::unexpected(r.error());
    }
    sampled_.resize(n);
    const int32_t top_k = trace_ != nullptr ? kTraceTopK : 0;
    if (top_k > 0) {
        margins_.resize(n);
        top_idx_.resize(n * top_k);
        top_val_.resize(n * top_k);
    }
    if (auto r = model_.forward(tokens_, prev_, sampled_.data(), precision_,
                                top_k ? margins_.data() : nullptr,
                                top_k ? top_idx_.data() : nullptr,
                                top_k ? top_val_.data() : nullptr, top_k);
        !r) {
        return std::unexpected(r.error());
    }
    if (trace_ != nullptr) {
        record_.clear();
        append_batch_record(sched_, step_index_, record_);
        record_.push_back(-2);
        record_.insert(record_.end(), sampled_.begin(), sampled_.end());
        for (std::size_t i = 0; i < n; ++i) {
            record_.push_back(float_bits(margins_[i]));
            for (int32_t j = 0; j < top_k; ++j) {
                record_.push_back(top_idx_[i * top_k + j]);
                record_.push_back(float_bits(top_val_[i * top_k + j]));
            }
        }
        std::fwrite(record_.data(), sizeof(int64_t), record_.size(), trace_);
    }
    ++step_index_;

    if (sink_) {
        ev_ids_.resize(n);
        ev_first_.resize(n);
        for (std::size_t i = 0; i < n; ++i) {
            ev_ids_[i] = run[i].id;
            ev_first_[i] = run[i].first_token.has_value() ? 0 : 1;
        }
    }
    retired_.clear();
    std::vector<uint64_t> ttfts;
    sum.retired = sched_.process_step_outputs(sampled_, blocks, &retired_, &ttfts);
    if (sink_) {
        std::size_t k = 0;
        for (std::size_t i = 0; i < n; ++i) {
            TokenEvent ev;
            ev.seq_id = ev_ids_[i];
            ev.token = sampled_[i];
            for (const Sequence& r : retired_) {
                if (r.id == ev.seq_id) ev.finished = true;
            }
            if (ev_first_[i] && k < ttfts.size()) ev.ttft_us = ttfts[k++];
            sink_(ev);
        }
    }
    for (Sequence& seq : retired_) done_[seq.id] = std::move(seq.tokens);
    for (const uint64_t t : ttfts) {
        ttft_us_ += double(t);
        ++ttft_samples_;
    }
    tokens_generated_ += n;
    tokens_computed_ += tokens_.size();
    ++iterations_;
    step_us_ += std::chrono::duration<double, std::micro>(Clock::now() - t0).count();
    return sum;
}

std::expected<int64_t, EngineError> Generator::run(int64_t max_steps) {
    int64_t steps = 0;
    while (sched_.has_pending_work() && (max_steps <= 0 || steps < max_steps)) {
        auto r = step();
        if (!r) return std::unexpected(r.error());
        if (r->batch_size == 0) {
            // nothing running and the queue head cannot be admitted
            return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
        }
        ++steps;
    }
    if (trace_ != nullptr) std::fflush(trace_);
    return steps;
}

const std::vector<int64_t>* Generator::output(SeqId id) const {
    auto it = done_.find(id);
    return it == done_.end() ? nullptr : &it->second;
}

Metrics Generator::metrics() const {
    Metrics m;
    m.uptime_secs = std::max(1e-6, std::chrono::duration<double>(Clock::now() - start_).count());
    m.total_requests_received = received_;
    m.total_requests_completed = sched_.total_completed();
    m.total_tokens_generated = tokens_generated_;
    m.throughput_tokens_per_sec = double(tokens_generated_) / m.uptime_secs;
    m.active_batch_size = sched_.running().size();
    m.waiting_queue_depth = sched_.waiting().size();
    const BlockAllocator& blocks = eng_.allocator();
    m.kv_cache_total_blocks = blocks.num_total_blocks();
    m.kv_cache_used_blocks = m.kv_cache_total_blocks - blocks.num_free_blocks();
    m.kv_cache_utilization_pct =
        m.kv_cache_total_blocks > 0
            ? 100.0 * double(m.kv_cache_used_blocks) / double(m.kv_cache_total_blocks)
            : 0.0;
    m.avg_ttft_ms = ttft_samples_ > 0 ? ttft_us_ / double(ttft_samples_) / 1000.0 : 0.0;
    m.avg_iteration_latency_ms = iterations_ > 0 ? step_us_ / double(iterations_) / 1000.0 : 0.0;
    m.total_preemptions = sched_.total_preemptions();
    m.total_iterations = iterations_;
    m.total_tokens_computed = tokens_computed_;
    m.h2d_bytes = model_.h2d_bytes() - h2d0_;
    m.d2h_bytes = model_.d2h_bytes() - d2h0_;
    m.kernel_launches = model_.kernel_launches() - launches0_;
    return m;
}

}  // namespace nvllm
