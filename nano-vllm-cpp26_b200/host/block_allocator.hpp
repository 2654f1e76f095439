// Physical KV-block allocator with the reference BlockManager's semantics
// (PagedKVCache::allocate_block / allocate_blocks / free_blocks,
// src/kv_cache.cpp:23-55, include/nano_vllm/kv_cache.hpp:48-55):
//   * free blocks form a FIFO queue, initially 0..num_blocks-1;
//   * allocate_block pops the front, allocate_blocks(count) pops `count` blocks
//     all-or-nothing, both reporting KVError::OutOfPhysicalBlocks through
//     std::expected;
//   * free_blocks appends to the back, in the order given.
// The reference asserts on out-of-range ids and double frees (debug builds
// only); here free_blocks checks the whole span first and rejects it unchanged.
#pragma once

#include <cstddef>
#include <cstdint>
#include <deque>
#include <expected>
#include <span>
#include <vector>

namespace nvllm {

using BlockId = std::size_t;

enum class KVError {
    OutOfPhysicalBlocks,
    InvalidBlock,  // out of range or not allocated (double free)
};

class BlockAllocator {
public:
    explicit BlockAllocator(std::size_t num_blocks);

    [[nodiscard]] std::size_t num_free_blocks() const noexcept { return free_.size(); }
    [[nodiscard]] std::size_t num_total_blocks() const noexcept { return allocated_.size(); }
    [[nodiscard]] double utilization() const noexcept;

    [[nodiscard]] std::expected<BlockId, KVError> allocate_block() noexcept;
    [[nodiscard]] std::expected<std::vector<BlockId>, KVError> allocate_blocks(std::size_t count);
    [[nodiscard]] std::expected<void, KVError> free_blocks(std::span<const BlockId> blocks);

private:
    std::deque<BlockId> free_;
    std::vector<bool> allocated_;
};

}  // namespace nvllm
