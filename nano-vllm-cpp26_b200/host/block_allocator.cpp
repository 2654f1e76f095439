#include "block_allocator.hpp"

namespace nvllm {

BlockAllocator::BlockAllocator(std::size_t num_blocks) : allocated_(num_blocks, false) {
    for (BlockId id = 0; id < num_blocks; ++id) free_.push_back(id);
}

double BlockAllocator::utilization() const noexcept {
    if (allocated_.empty()) return 0.0;
    return static_cast<double>(allocated_.size() - free_.size()) /
           static_cast<double>(allocated_.size());
}

std::expected<BlockId, KVError> BlockAllocator::allocate_block() noexcept {
    if (free_.empty()) return std::unexpected(KVError::OutOfPhysicalBlocks);
    const BlockId id = free_.front();
    free_.pop_front();
    allocated_[id] = true;
    return id;
}

std::expected<std::vector<BlockId>, KVError> BlockAllocator::allocate_blocks(std::size_t count) {
    if (free_.size() < count) return std::unexpected(KVError::OutOfPhysicalBlocks);
    std::vector<BlockId> out;
    out.reserve(count);
    for (std::size_t i = 0; i < count; ++i) {
        const BlockId id = free_.front();
        free_.pop_front();
        allocated_[id] = true;
        out.push_back(id);
    }
    return out;
}

std::expected<void, KVError> BlockAllocator::free_blocks(std::span<const BlockId> blocks) {
    // validate first (range, allocated, no duplicates within the span)
    std::vector<bool> seen;
    for (const BlockId id : blocks) {
        if (id >= allocated_.size() || !allocated_[id]) return std::unexpected(KVError::InvalidBlock);
        if (seen.empty()) seen.assign(allocated_.size(), false);
        if (seen[id]) return std::unexpected(KVError::InvalidBlock);
        seen[id] = true;
    }
    for (const BlockId id : blocks) {
        allocated_[id] = false;
        free_.push_back(id);
    }
    return {};
}

}  // namespace nvllm
