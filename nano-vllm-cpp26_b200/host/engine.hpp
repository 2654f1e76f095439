// AttentionEngine: the per-device host object that replaces steps 3c/3d of
// TransformerModel::forward_batch (src/model.cpp:188-260) for an engine thread
// (src/engine.cpp:212-213).
//
// It owns, on one CUDA device:
//   * the K and V arenas in HBM, [num_blocks, num_layers, block_size, H*hd]
//     fp32 (the reference's PagedKVCache arena, include/nano_vllm/kv_cache.hpp:30-33),
//     and their BlockAllocator (the reference's allocator semantics);
//   * the int32 device mirror of the step's metadata, filled by ONE pinned
//     cudaMemcpyAsync per iteration from a double-buffered pinned staging area;
//   * pinned host buffers for the step's Q/K/V rows and the attention output,
//     a device workspace for nvllm_paged_attention, and a CUDA stream.
//
// Per iteration: begin_step(sequences) packs and uploads the metadata; then per
// layer attention(...) copies that layer's Q/K/V rows in, runs
// nvllm_reshape_and_cache + nvllm_paged_attention and copies the output back
// (synchronously, like the reference's loop), or attention_device(...) runs on
// caller-owned device rows asynchronously.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <expected>
#include <memory>
#include <span>

#include "../../include/nvllm.h"
#include "block_allocator.hpp"
#include "metadata.hpp"

namespace nvllm {

struct EngineConfig {
    nvllm_kv_layout layout{};
    int32_t max_seqs = 0;          // sequences per step
    int32_t max_tokens = 0;        // new tokens (flattened rows) per step
    int32_t max_blocks_per_seq = 0;
    int32_t device = 0;
};

struct EngineError {
    enum class Kind { Invalid, Cuda, Pack, Kernel, NoStep, Blas, Unsupported } kind;
    int code = 0;  // cudaError_t, PackError, nvllm status or cublasStatus_t, by kind
};

class AttentionEngine {
public:
    static std::expected<std::unique_ptr<AttentionEngine>, EngineError> create(
        const EngineConfig& cfg);
    ~AttentionEngine();
    AttentionEngine(const AttentionEngine&) = delete;
    AttentionEngine& operator=(const AttentionEngine&) = delete;

    BlockAllocator& allocator() noexcept { return allocator_; }
    const EngineConfig& config() const noexcept { return cfg_; }
    float* k_arena() noexcept { return d_k_; }
    float* v_arena() noexcept { return d_v_; }
    cudaStream_t stream() noexcept { return stream_; }
    // pinned staging for one layer's rows ([max_tokens, H*hd] each)
    float* host_query() noexcept { return h_q_[0]; }
    float* host_key() noexcept { return h_k_[0]; }
    float* host_value() noexcept { return h_v_[0]; }
    float* host_output() noexcept { return h_out_[0]; }
    const MetadataLayout& step() const noexcept { return step_; }
    bool has_step() const noexcept { return have_step_; }
    // the step's packed metadata on the device (offsets in step())
    const unsigned char* device_metadata() const noexcept { return d_meta_; }

    // Flattens the batch and uploads its metadata (one cudaMemcpyAsync). With
    // pad_seqs / pad_tokens the batch is laid out as that many sequences and
    // token rows (empty sequences, slot -1 rows) and the step's attention
    // bounds become those of the bucket: max_query_len 1 for decode-only
    // batches, else min(pad_tokens, max context); max_context_len the table
    // capacity. Every batch of a bucket then issues identical launches, which
    // is what lets the device model replay one captured CUDA graph per bucket.
    std::expected<void, EngineError> begin_step(std::span<const SequenceView> seqs,
                                                int32_t pad_seqs = 0, int32_t pad_tokens = 0);

    // One layer with host rows: H2D of Q/K/V, KV write, attention, D2H of the
    // output; returns once `out` holds the result. Rows that already live in
    // the engine's pinned buffers are not copied again.
    std::expected<void, EngineError> attention(int32_t layer, const float* q, const float* k,
                                               const float* v, float* out, int32_t precision);

    // One layer with device rows, asynchronous on stream().
    std::expected<void, EngineError> attention_device(int32_t layer, const float* d_q,
                                                      const float* d_k, const float* d_v,
                                                      float* d_out, int32_t precision);

    // Pipelined host rows, two slots. submit(layer, slot) queues, for the step
    // begun last, the H2D of the slot's pinned Q/K/V rows on an upload stream,
    // the KV write + attention on stream() once they have landed, and the D2H of
    // the output into the slot's pinned output buffer on a download stream once
    // the kernels are done; it returns without waiting. collect(slot) waits for that
    // output. While one slot's kernels run, the other slot's copies proceed, so
    // the copies of consecutive steps overlap the kernels. A slot must be
    // collected before it is submitted again (its pinned rows stay in use until
    // then); the synchronous attention() refuses while a slot is in flight.
    std::expected<void, EngineError> submit(int32_t layer, int32_t slot, int32_t precision);
    std::expected<void, EngineError> collect(int32_t slot);
    // pinned rows of a slot ([max_tokens, H*hd] each); slot 0's are host_query() etc.
    std::expected<void, EngineError> slot_buffers(int32_t slot, float** q, float** k, float** v,
                                                  float** out);

private:
    explicit AttentionEngine(const EngineConfig& cfg);
    std::expected<void, EngineError> init();
    std::expected<void, EngineError> init_slot(int slot);

    EngineConfig cfg_;
    BlockAllocator allocator_;
    MetadataLayout step_{};
    bool have_step_ = false;
    std::size_t meta_capacity_ = 0;
    std::size_t row_floats_ = 0;
    size_t ws_bytes_ = 0;
    int meta_slot_ = 0;

    cudaStream_t stream_ = nullptr;
    cudaEvent_t meta_done_[2] = {nullptr, nullptr};
    unsigned char* h_meta_[2] = {nullptr, nullptr};
    unsigned char* d_meta_ = nullptr;
    float* d_k_ = nullptr;
    float* d_v_ = nullptr;
    // per slot: Q, K, V, out rows on the device and their pinned host copies
    // (slot 1 is allocated on its first use)
    float* d_rows_[2] = {nullptr, nullptr};
    void* d_ws_ = nullptr;
    float* h_q_[2] = {nullptr, nullptr};
    float* h_k_[2] = {nullptr, nullptr};
    float* h_v_[2] = {nullptr, nullptr};
    float* h_out_[2] = {nullptr, nullptr};
    // the pipelined path's copies: H2D on one stream, D2H on another, so that a
    // step's uploads never queue behind the previous step's download (which
    // waits for that step's kernels)
    cudaStream_t h2d_stream_ = nullptr;
    cudaStream_t d2h_stream_ = nullptr;
    cudaEvent_t in_ready_[2] = {nullptr, nullptr};   // slot's rows landed
    cudaEvent_t out_ready_[2] = {nullptr, nullptr};  // slot's kernels done
    cudaEvent_t out_done_[2] = {nullptr, nullptr};   // slot's output back on the host
    bool in_flight_[2] = {false, false};
    bool slot_used_[2] = {false, false};  // out_done_ recorded at least once
};

}  // namespace nvllm
