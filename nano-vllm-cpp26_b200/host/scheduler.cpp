#include "scheduler.hpp"

#include <algorithm>
#include <utility>

namespace nvllm {

Sequence::Sequence(SeqId seq_id, std::vector<int64_t> prompt, std::size_t max_new)
    : id(seq_id),
      tokens(prompt.empty() ? std::vector<int64_t>{1} : std::move(prompt)),
      max_new_tokens(std::max<std::size_t>(max_new, 1)),
      arrival(Clock::now()) {
    prompt_len = tokens.size();
}

bool Sequence::finished(std::optional<int64_t> eos) const noexcept {
    if (generated_len() >= max_new_tokens) return true;
    return eos.has_value() && generated_len() > 0 && tokens.back() == *eos;
}

Scheduler::Scheduler(SchedulerConfig cfg, std::size_t block_size)
    : cfg_(cfg), block_size_(block_size == 0 ? 1 : block_size) {
    running_.reserve(cfg_.max_batch_size);
}

void Scheduler::add_request(Sequence seq) {
    seq.status = SeqStatus::Waiting;
    waiting_.push_back(std::move(seq));
}

// Recompute preemption: the victim keeps its tokens, loses its blocks and its
// computed prefix, and waits at the head of the queue.
void Scheduler::preempt(Sequence&& victim, BlockAllocator& blocks) {
    (void)blocks.free_blocks(victim.table);
    victim.table.clear();
    victim.num_computed = 0;
    victim.status = SeqStatus::Waiting;
    waiting_.push_front(std::move(victim));
    ++preemptions_;
}

StepSummary Scheduler::schedule_step(BlockAllocator& blocks) {
    StepSummary sum{};
    // Phase 1: one more block for any running sequence whose newest token
    // starts a block (src/scheduler.cpp:30-76).
    std::size_t i = 0;
    while (i < running_.size()) {
        Sequence& seq = running_[i];
        if (seq.table.size() >= blocks_for(seq.total_len())) {
            ++i;
            continue;
        }
        while (blocks.num_free_blocks() == 0 && running_.size() > i + 1) {
            Sequence victim = std::move(running_.back());
            running_.pop_back();
            preempt(std::move(victim), blocks);
            ++sum.preempted;
        }
        if (auto b = blocks.allocate_block(); b.has_value()) {
            running_[i].table.push_back(*b);
            ++i;
        } else {
            Sequence victim = std::move(running_[i]);
            running_[i] = std::move(running_.back());
            running_.pop_back();
            preempt(std::move(victim), blocks);
            ++sum.preempted;
        }
    }

    std::size_t scheduled = 0;
    for (const Sequence& s : running_) scheduled += s.uncomputed().size();

    // Phase 2: admission in queue order (src/scheduler.cpp:84-114).
    while (running_.size() < cfg_.max_batch_size && !waiting_.empty()) {
        const Sequence& cand = waiting_.front();
        const std::size_t need_tokens = cand.uncomputed().size();
        if (scheduled + need_tokens > cfg_.max_tokens_per_step && !running_.empty()) break;
        const std::size_t need_blocks = blocks_for(cand.total_len());
        if (blocks.num_free_blocks() < need_blocks + cfg_.watermark_blocks) break;
        auto got = blocks.allocate_blocks(need_blocks);
        if (!got.has_value()) break;
        Sequence seq = std::move(waiting_.front());
        waiting_.pop_front();
        seq.table = std::move(*got);
        seq.status = SeqStatus::Running;
        scheduled += need_tokens;
        running_.push_back(std::move(seq));
        ++sum.admitted;
    }
    sum.batch_size = running_.size();
    sum.scheduled_tokens = scheduled;
    return sum;
}

std::size_t Scheduler::process_step_outputs(std::span<const int64_t> sampled,
                                            BlockAllocator& blocks,
                                            std::vector<Sequence>* finished,
                                            std::vector<uint64_t>* ttft_us) {
    const auto now = Clock::now();
    const std::size_t n = std::min(sampled.size(), running_.size());
    for (std::size_t i = 0; i < n; ++i) {
        Sequence& seq = running_[i];
        seq.num_computed = seq.tokens.size();
        seq.tokens.push_back(sampled[i]);
        if (!seq.first_token.has_value()) {
            seq.first_token = now;
            if (ttft_us != nullptr) {
                ttft_us->push_back(uint64_t(
                    std::chrono::duration_cast<std::chrono::microseconds>(now - seq.arrival)
                        .count()));
            }
        }
        if (seq.finished(cfg_.eos_token_id)) seq.status = SeqStatus::Finished;
    }
    // retire in place: the last running sequence takes the finished one's slot
    // (src/scheduler.cpp:168-183)
    std::size_t retired = 0;
    std::size_t i = 0;
    while (i < running_.size()) {
        if (running_[i].status != SeqStatus::Finished) {
            ++i;
            continue;
        }
        (void)blocks.free_blocks(running_[i].table);
        if (finished != nullptr) finished->push_back(std::move(running_[i]));
        if (i + 1 != running_.size()) running_[i] = std::move(running_.back());
        running_.pop_back();
        ++retired;
        ++completed_;
    }
    return retired;
}

}  // namespace nvllm
