#include "metadata.hpp"

#include <algorithm>
#include <cstring>
#include <limits>

namespace nvllm {

namespace {
constexpr std::size_t align16(std::size_t x) { return (x + 15) / 16 * 16; }
}  // namespace

MetadataLayout metadata_layout(int32_t num_seqs, int32_t num_tokens, int32_t max_blocks) {
    MetadataLayout m;
    const std::size_t S = static_cast<std::size_t>(num_seqs);
    std::size_t off = 0;
    m.cu_off = off;
    off = align16(off + (S + 1) * sizeof(int32_t));
    m.ctx_off = off;
    off = align16(off + S * sizeof(int32_t));
    m.last_off = off;
    off = align16(off + S * sizeof(int32_t));
    m.slot_off = off;
    off = align16(off + static_cast<std::size_t>(num_tokens) * sizeof(int32_t));
    m.table_off = off;
    off = align16(off + S * static_cast<std::size_t>(max_blocks) * sizeof(int32_t));
    m.bytes = off;
    m.num_seqs = num_seqs;
    m.num_tokens = num_tokens;
    m.max_blocks = max_blocks;
    return m;
}

std::expected<MetadataLayout, PackError> pack_metadata(std::span<const SequenceView> seqs,
                                                       int32_t block_size, int32_t max_blocks,
                                                       std::span<std::byte> buf,
                                                       int32_t pad_seqs, int32_t pad_tokens) {
    if (block_size <= 0 || max_blocks <= 0 || pad_seqs < 0 || pad_tokens < 0) {
        return std::unexpected(PackError::Invalid);
    }
    int64_t n_tokens = 0;
    int32_t max_q = 0, max_ctx = 0;
    for (const auto& sv : seqs) {
        if (sv.num_computed < 0 || sv.total_len < 0 || sv.num_computed > sv.total_len) {
            return std::unexpected(PackError::Invalid);
        }
        const int64_t need = (int64_t(sv.total_len) + block_size - 1) / block_size;
        if (int64_t(sv.table.size()) < need) return std::unexpected(PackError::TableTooShort);
        if (need > max_blocks) return std::unexpected(PackError::TooWide);
        n_tokens += sv.total_len - sv.num_computed;
        max_q = std::max(max_q, sv.total_len - sv.num_computed);
        max_ctx = std::max(max_ctx, sv.total_len);
    }
    if (n_tokens > std::numeric_limits<int32_t>::max()) return std::unexpected(PackError::TooWide);
    const bool padded = pad_seqs > 0 || pad_tokens > 0;
    const int32_t S = int32_t(seqs.size());
    const int32_t S_out = std::max(S, pad_seqs);
    const int32_t T_out = std::max(int32_t(n_tokens), pad_tokens);
    if (padded && (pad_seqs < S || pad_tokens < n_tokens)) return std::unexpected(PackError::Invalid);
    MetadataLayout m = metadata_layout(S_out, T_out, max_blocks);
    if (buf.size() < m.bytes) return std::unexpected(PackError::BufferTooSmall);
    m.max_query_len = max_q;
    m.max_context_len = max_ctx;
    m.real_seqs = S;
    m.real_tokens = int32_t(n_tokens);
    m.padded = padded;

    auto* base = reinterpret_cast<unsigned char*>(buf.data());
    auto* cu = reinterpret_cast<int32_t*>(base + m.cu_off);
    auto* ctx = reinterpret_cast<int32_t*>(base + m.ctx_off);
    auto* last = reinterpret_cast<int32_t*>(base + m.last_off);
    auto* slots = reinterpret_cast<int32_t*>(base + m.slot_off);
    auto* tables = reinterpret_cast<int32_t*>(base + m.table_off);

    constexpr BlockId kMaxId = BlockId(std::numeric_limits<int32_t>::max());
    int32_t t = 0;
    cu[0] = 0;
    for (std::size_t s = 0; s < seqs.size(); ++s) {
        const SequenceView& sv = seqs[s];
        int32_t* row = tables + s * static_cast<std::size_t>(max_blocks);
        const std::size_t nb = std::min<std::size_t>(sv.table.size(), std::size_t(max_blocks));
        for (std::size_t b = 0; b < nb; ++b) {
            if (sv.table[b] > kMaxId) return std::unexpected(PackError::TooWide);
            row[b] = int32_t(sv.table[b]);
        }
        std::fill(row + nb, row + max_blocks, 0);
        // flatten: one record per uncomputed token, positions num_computed.. (model.cpp:144-157)
        for (int32_t pos = sv.num_computed; pos < sv.total_len; ++pos, ++t) {
            const int64_t slot = int64_t(sv.table[pos / block_size]) * block_size + pos % block_size;
            if (slot > std::numeric_limits<int32_t>::max()) return std::unexpected(PackError::TooWide);
            slots[t] = int32_t(slot);
        }
        cu[s + 1] = t;
        ctx[s] = sv.total_len;
        last[s] = t - 1;
    }
    for (int32_t s = S; s < S_out; ++s) {
        std::fill(tables + std::size_t(s) * std::size_t(max_blocks),
                  tables + std::size_t(s + 1) * std::size_t(max_blocks), 0);
        cu[s + 1] = t;
        ctx[s] = 0;
        last[s] = 0;
    }
    std::fill(slots + t, slots + T_out, -1);
    return m;
}

}  // namespace nvllm
