// Per-step attention metadata: selective token flattening
// (src/model.cpp:138-159) packed into one contiguous int32 buffer, the unit of
// the single host-to-device upload per engine iteration.
//
// Buffer layout (int32, each section 16-byte aligned):
//   cu_seqlens_q[S+1] | context_lens[S] | last_token_idx[S] |
//   slot_mapping[n_tokens] | block_tables[S * max_blocks]
// with, for sequence s holding total_len tokens of which num_computed are cached:
//   cu_seqlens_q[s+1] - cu_seqlens_q[s] = total_len - num_computed,
//   context_lens[s] = total_len,
//   last_token_idx[s] = cu_seqlens_q[s+1] - 1           (src/model.cpp:156),
//   slot_mapping[t] = table[pos / B] * B + pos % B      (src/model.cpp:192-194),
//   block_tables[s][b] = table[b] (int32), 0 past the table's end.
#pragma once

#include <cstddef>
#include <cstdint>
#include <expected>
#include <span>

#include "block_allocator.hpp"

namespace nvllm {

struct SequenceView {
    int32_t num_computed;              // tokens whose K/V are already cached
    int32_t total_len;                 // tokens after this step (context length)
    std::span<const BlockId> table;    // physical blocks, logical order
};

struct MetadataLayout {
    std::size_t cu_off = 0, ctx_off = 0, last_off = 0, slot_off = 0, table_off = 0, bytes = 0;
    int32_t num_seqs = 0, num_tokens = 0, max_blocks = 0;  // as laid out (padding included)
    int32_t max_query_len = 0, max_context_len = 0;
    int32_t real_seqs = 0, real_tokens = 0;  // the batch's own sequences and new tokens
    bool padded = false;
};

enum class PackError {
    Invalid,        // negative lengths, num_computed > total_len
    TableTooShort,  // fewer than ceil(total_len / B) blocks
    TooWide,        // more blocks than max_blocks, or an id beyond int32
    BufferTooSmall,
};

// Offsets and size for a batch of num_seqs sequences and num_tokens new tokens.
MetadataLayout metadata_layout(int32_t num_seqs, int32_t num_tokens, int32_t max_blocks);

// Packs the batch into buf; returns the layout actually used (max_blocks is the
// caller's table width). pad_seqs / pad_tokens (0: none) lay the batch out as
// pad_seqs sequences and pad_tokens token rows, so that every batch of a
// bucket has the same layout: the extra sequences are empty (no new tokens,
// context 0, zero table row, last_token_idx 0) and the extra token rows have
// slot -1, which the KV write skips.
std::expected<MetadataLayout, PackError> pack_metadata(std::span<const SequenceView> seqs,
                                                       int32_t block_size, int32_t max_blocks,
                                                       std::span<std::byte> buf,
                                                       int32_t pad_seqs = 0,
                                                       int32_t pad_tokens = 0);

}  // namespace nvllm
