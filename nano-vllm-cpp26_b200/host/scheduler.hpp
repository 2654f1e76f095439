// Iteration-level continuous-batching scheduler with recompute preemption, the
// reference ContinuousScheduler's policy (src/scheduler.cpp:8-198,
// include/nano_vllm/scheduler.hpp:83-170) on this library's BlockAllocator.
//
// Per step:
//   1. every running sequence gets the one extra block its newest token may
//      need; when none is free the youngest running sequences are preempted
//      (blocks freed, progress dropped, back to the FRONT of the waiting queue),
//      and a sequence that still cannot grow preempts itself (its slot taken by
//      the last running sequence);
//   2. waiting sequences are admitted in queue order while the batch has room,
//      the step's token budget holds (the first admission into an empty batch
//      is exempt) and the arena keeps `watermark` blocks spare after giving the
//      candidate all the blocks of its current length.
// After the forward pass, process_step_outputs appends each sampled token,
// marks sequences that reached max_new_tokens (or sampled EOS) finished, and
// retires them by swapping the last running sequence into their slot.
//
// The order of `running()` is the order the forward pass flattens, and every
// decision above depends on it, so it is kept exactly as the reference keeps it.
#pragma once

#include <chrono>
#include <cstddef>
#include <cstdint>
#include <deque>
#include <optional>
#include <span>
#include <vector>

#include "block_allocator.hpp"

namespace nvllm {

using SeqId = uint64_t;
using Clock = std::chrono::steady_clock;

enum class SeqStatus { Waiting, Running, Finished };

struct Sequence {
    SeqId id = 0;
    SeqStatus status = SeqStatus::Waiting;
    std::vector<int64_t> tokens;  // prompt followed by generated tokens
    std::size_t prompt_len = 0;
    std::size_t num_computed = 0;  // tokens whose K/V are in the arena
    std::size_t max_new_tokens = 1;
    std::vector<BlockId> table;
    Clock::time_point arrival{};
    std::optional<Clock::time_point> first_token{};

    // An empty prompt becomes {1}; max_new_tokens is at least 1
    // (src/scheduler.cpp:8-20).
    Sequence(SeqId seq_id, std::vector<int64_t> prompt, std::size_t max_new);

    std::size_t total_len() const noexcept { return tokens.size(); }
    std::size_t generated_len() const noexcept {
        return tokens.size() > prompt_len ? tokens.size() - prompt_len : 0;
    }
    std::span<const int64_t> uncomputed() const noexcept {
        return std::span<const int64_t>(tokens).subspan(num_computed);
    }
    bool finished(std::optional<int64_t> eos) const noexcept;
};

struct SchedulerConfig {
    std::size_t max_batch_size = 32;
    std::size_t max_tokens_per_step = 512;
    std::size_t watermark_blocks = 4;
    std::optional<int64_t> eos_token_id{};
};

struct StepSummary {
    std::size_t admitted = 0;
    std::size_t preempted = 0;
    std::size_t retired = 0;
    std::size_t batch_size = 0;
    std::size_t scheduled_tokens = 0;
};

class Scheduler {
public:
    Scheduler(SchedulerConfig cfg, std::size_t block_size);

    void add_request(Sequence seq);
    StepSummary schedule_step(BlockAllocator& blocks);
    // One sampled token per running sequence, in running() order. Returns the
    // number of sequences retired; their final token lists go to `finished`,
    // the time to first token of every sequence that produced its first token
    // in this step to `ttft_us` (src/scheduler.cpp:123-166).
    std::size_t process_step_outputs(std::span<const int64_t> sampled, BlockAllocator& blocks,
                                     std::vector<Sequence>* finished = nullptr,
                                     std::vector<uint64_t>* ttft_us = nullptr);

    const std::vector<Sequence>& running() const noexcept { return running_; }
    const std::deque<Sequence>& waiting() const noexcept { return waiting_; }
    bool has_pending_work() const noexcept { return !running_.empty() || !waiting_.empty(); }
    uint64_t total_preemptions() const noexcept { return preemptions_; }
    uint64_t total_completed() const noexcept { return completed_; }
    const SchedulerConfig& config() const noexcept { return cfg_; }
    std::size_t block_size() const noexcept { return block_size_; }

private:
    std::size_t blocks_for(std::size_t len) const noexcept {
        return (len + block_size_ - 1) / block_size_;
    }
    void preempt(Sequence&& victim, BlockAllocator& blocks);

    SchedulerConfig cfg_;
    std::size_t block_size_;
    std::vector<Sequence> running_;
    std::deque<Sequence> waiting_;
    uint64_t preemptions_ = 0;
    uint64_t completed_ = 0;
};

}  // namespace nvllm
