#include "engine.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace nvllm {

namespace {

std::unexpected<EngineError> cuda_error(cudaError_t e) {
    return std::unexpected(EngineError{EngineError::Kind::Cuda, int(e)});
}

#define NVLLM_CUDA_TRY(expr)                        \
    do {                                            \
        const cudaError_t e_ = (expr);              \
        if (e_ != cudaSuccess) return cuda_error(e_); \
    } while (0)

}  // namespace

AttentionEngine::AttentionEngine(const EngineConfig& cfg)
    : cfg_(cfg), allocator_(static_cast<std::size_t>(cfg.layout.num_blocks)) {}

std::expected<std::unique_ptr<AttentionEngine>, EngineError> AttentionEngine::create(
    const EngineConfig& cfg) {
    const nvllm_kv_layout& L = cfg.layout;
    if (L.num_blocks <= 0 || L.num_layers <= 0 || L.block_size <= 0 || L.num_heads <= 0 ||
        L.head_dim <= 0 || cfg.max_seqs <= 0 || cfg.max_tokens <= 0 ||
        cfg.max_blocks_per_seq <= 0 || cfg.device < 0) {
        return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
    }
    std::unique_ptr<AttentionEngine> eng(new AttentionEngine(cfg));
    if (auto r = eng->init(); !r) return std::unexpected(r.error());
    return eng;
}

std::expected<void, EngineError> AttentionEngine::init() {
    const nvllm_kv_layout& L = cfg_.layout;
    NVLLM_CUDA_TRY(cudaSetDevice(cfg_.device));
    NVLLM_CUDA_TRY(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    row_floats_ = std::size_t(L.num_heads) * std::size_t(L.head_dim);
    const std::size_t arena_bytes = std::size_t(L.num_blocks) * std::size_t(L.num_layers) *
                                    std::size_t(L.block_size) * row_floats_ * sizeof(float);
    NVLLM_CUDA_TRY(cudaMalloc(&d_k_, arena_bytes));
    NVLLM_CUDA_TRY(cudaMalloc(&d_v_, arena_bytes));
    // the reference zero-fills its arenas (src/kv_cache.cpp:14-15)
    NVLLM_CUDA_TRY(cudaMemsetAsync(d_k_, 0, arena_bytes, stream_));
    NVLLM_CUDA_TRY(cudaMemsetAsync(d_v_, 0, arena_bytes, stream_));

    meta_capacity_ = metadata_layout(cfg_.max_seqs, cfg_.max_tokens, cfg_.max_blocks_per_seq).bytes;
    for (int i = 0; i < 2; ++i) {
        NVLLM_CUDA_TRY(cudaMallocHost(reinterpret_cast<void**>(&h_meta_[i]), meta_capacity_));
        NVLLM_CUDA_TRY(cudaEventCreateWithFlags(&meta_done_[i], cudaEventDisableTiming));
        NVLLM_CUDA_TRY(cudaEventRecord(meta_done_[i], stream_));
    }
    NVLLM_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&d_meta_), meta_capacity_));

    if (auto r = init_slot(0); !r) return r;

    const int32_t max_ctx = cfg_.max_blocks_per_seq * L.block_size;
    ws_bytes_ = nvllm_paged_attention_workspace_size(cfg_.max_seqs, cfg_.max_tokens, max_ctx, &L);
    if (ws_bytes_ == 0) return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
    NVLLM_CUDA_TRY(cudaMalloc(&d_ws_, ws_bytes_));
    NVLLM_CUDA_TRY(cudaStreamSynchronize(stream_));
    return {};
}

std::expected<void, EngineError> AttentionEngine::init_slot(int slot) {
    if (d_rows_[slot] != nullptr) return {};
    const std::size_t rows_bytes = std::size_t(cfg_.max_tokens) * row_floats_ * sizeof(float);
    NVLLM_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&d_rows_[slot]), 4 * rows_bytes));
    NVLLM_CUDA_TRY(cudaMallocHost(reinterpret_cast<void**>(&h_q_[slot]), rows_bytes));
    NVLLM_CUDA_TRY(cudaMallocHost(reinterpret_cast<void**>(&h_k_[slot]), rows_bytes));
    NVLLM_CUDA_TRY(cudaMallocHost(reinterpret_cast<void**>(&h_v_[slot]), rows_bytes));
    NVLLM_CUDA_TRY(cudaMallocHost(reinterpret_cast<void**>(&h_out_[slot]), rows_bytes));
    return {};
}

AttentionEngine::~AttentionEngine() {
    if (stream_ != nullptr) {
        cudaSetDevice(cfg_.device);
        cudaStreamSynchronize(stream_);
    }
    for (cudaStream_t cs : {h2d_stream_, d2h_stream_}) {
        if (cs != nullptr) cudaStreamSynchronize(cs);
    }
    for (int i = 0; i < 2; ++i) {
        if (meta_done_[i]) cudaEventDestroy(meta_done_[i]);
        if (h_meta_[i]) cudaFreeHost(h_meta_[i]);
        for (cudaEvent_t ev : {in_ready_[i], out_ready_[i], out_done_[i]}) {
            if (ev) cudaEventDestroy(ev);
        }
        for (float* p : {h_q_[i], h_k_[i], h_v_[i], h_out_[i]}) {
            if (p) cudaFreeHost(p);
        }
        if (d_rows_[i]) cudaFree(d_rows_[i]);
    }
    if (h2d_stream_) cudaStreamDestroy(h2d_stream_);
    if (d2h_stream_) cudaStreamDestroy(d2h_stream_);
    if (d_meta_) cudaFree(d_meta_);
    if (d_ws_) cudaFree(d_ws_);
    if (d_k_) cudaFree(d_k_);
    if (d_v_) cudaFree(d_v_);
    if (stream_) cudaStreamDestroy(stream_);
}

std::expected<void, EngineError> AttentionEngine::begin_step(std::span<const SequenceView> seqs,
                                                            int32_t pad_seqs, int32_t pad_tokens) {
    if (seqs.size() > std::size_t(cfg_.max_seqs) || pad_seqs > cfg_.max_seqs ||
        pad_tokens > cfg_.max_tokens) {
        return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
    }
    NVLLM_CUDA_TRY(cudaSetDevice(cfg_.device));
    // the staging buffer about to be refilled must have finished its last upload
    NVLLM_CUDA_TRY(cudaEventSynchronize(meta_done_[meta_slot_]));
    auto packed = pack_metadata(
        seqs, cfg_.layout.block_size, cfg_.max_blocks_per_seq,
        std::span<std::byte>(reinterpret_cast<std::byte*>(h_meta_[meta_slot_]), meta_capacity_),
        pad_seqs, pad_tokens);
    if (!packed) return std::unexpected(EngineError{EngineError::Kind::Pack, int(packed.error())});
    if (packed->num_tokens > cfg_.max_tokens) {
        return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
    }
    NVLLM_CUDA_TRY(cudaMemcpyAsync(d_meta_, h_meta_[meta_slot_], packed->bytes,
                                   cudaMemcpyHostToDevice, stream_));
    NVLLM_CUDA_TRY(cudaEventRecord(meta_done_[meta_slot_], stream_));
    meta_slot_ ^= 1;
    if (packed->padded) {
        const int32_t cap = cfg_.max_blocks_per_seq * cfg_.layout.block_size;
        packed->max_query_len = packed->max_query_len <= 1 ? 1 : std::min(packed->num_tokens, cap);
        packed->max_context_len = cap;
    }
    step_ = *packed;
    have_step_ = true;
    return {};
}

std::expected<void, EngineError> AttentionEngine::attention_device(int32_t layer, const float* d_q,
                                                                   const float* d_k,
                                                                   const float* d_v, float* d_out,
                                                                   int32_t precision) {
    if (!have_step_) return std::unexpected(EngineError{EngineError::Kind::NoStep, 0});
    if (step_.num_tokens == 0) return {};
    const nvllm_kv_layout& L = cfg_.layout;
    const auto* meta = d_meta_;
    const auto* cu = reinterpret_cast<const int32_t*>(meta + step_.cu_off);
    const auto* ctx = reinterpret_cast<const int32_t*>(meta + step_.ctx_off);
    const auto* slots = reinterpret_cast<const int32_t*>(meta + step_.slot_off);
    const auto* tables = reinterpret_cast<const int32_t*>(meta + step_.table_off);
    int rc = nvllm_reshape_and_cache(d_k, d_v, d_k_, d_v_, slots, step_.num_tokens, layer, &L,
                                     stream_);
    if (rc != NVLLM_OK) return std::unexpected(EngineError{EngineError::Kind::Kernel, rc});
    // softmax scale of the reference, src/model.cpp:205
    const float scale = 1.0f / std::sqrt(static_cast<float>(L.head_dim));
    rc = nvllm_paged_attention(d_out, d_q, d_k_, d_v_, tables, step_.max_blocks, cu, ctx,
                               step_.num_seqs, step_.max_query_len, step_.max_context_len, layer,
                               scale, precision, d_ws_, ws_bytes_, &L, stream_);
    if (rc != NVLLM_OK) return std::unexpected(EngineError{EngineError::Kind::Kernel, rc});
    return {};
}

std::expected<void, EngineError> AttentionEngine::attention(int32_t layer, const float* q,
                                                            const float* k, const float* v,
                                                            float* out, int32_t precision) {
    if (!have_step_) return std::unexpected(EngineError{EngineError::Kind::NoStep, 0});
    if (in_flight_[0] || in_flight_[1]) {
        return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
    }
    NVLLM_CUDA_TRY(cudaSetDevice(cfg_.device));
    const std::size_t n = std::size_t(step_.num_tokens);
    if (n == 0) return {};
    const std::size_t bytes = n * row_floats_ * sizeof(float);
    const std::size_t stride = std::size_t(cfg_.max_tokens) * row_floats_;
    float* dq = d_rows_[0];
    float* dk = d_rows_[0] + stride;
    float* dv = d_rows_[0] + 2 * stride;
    float* dout = d_rows_[0] + 3 * stride;
    const float* srcs[3] = {q, k, v};
    float* pinned[3] = {h_q_[0], h_k_[0], h_v_[0]};
    float* dsts[3] = {dq, dk, dv};
    for (int i = 0; i < 3; ++i) {
        if (srcs[i] != pinned[i]) std::memcpy(pinned[i], srcs[i], bytes);
        NVLLM_CUDA_TRY(cudaMemcpyAsync(dsts[i], pinned[i], bytes, cudaMemcpyHostToDevice, stream_));
    }
    if (auto r = attention_device(layer, dq, dk, dv, dout, precision); !r) return r;
    NVLLM_CUDA_TRY(cudaMemcpyAsync(h_out_[0], dout, bytes, cudaMemcpyDeviceToHost, stream_));
    NVLLM_CUDA_TRY(cudaStreamSynchronize(stream_));
    if (out != h_out_[0]) std::memcpy(out, h_out_[0], bytes);
    return {};
}

std::expected<void, EngineError> AttentionEngine::slot_buffers(int32_t slot, float** q, float** k,
                                                               float** v, float** out) {
    if (slot < 0 || slot > 1) return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
    NVLLM_CUDA_TRY(cudaSetDevice(cfg_.device));
    if (auto r = init_slot(slot); !r) return r;
    if (q) *q = h_q_[slot];
    if (k) *k = h_k_[slot];
    if (v) *v = h_v_[slot];
    if (out) *out = h_out_[slot];
    return {};
}

std::expected<void, EngineError> AttentionEngine::submit(int32_t layer, int32_t slot,
                                                         int32_t precision) {
    if (!have_step_) return std::unexpected(EngineError{EngineError::Kind::NoStep, 0});
    if (slot < 0 || slot > 1 || in_flight_[slot]) {
        return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
    }
    NVLLM_CUDA_TRY(cudaSetDevice(cfg_.device));
    if (auto r = init_slot(slot); !r) return r;
    if (h2d_stream_ == nullptr) {
        NVLLM_CUDA_TRY(cudaStreamCreateWithFlags(&h2d_stream_, cudaStreamNonBlocking));
        NVLLM_CUDA_TRY(cudaStreamCreateWithFlags(&d2h_stream_, cudaStreamNonBlocking));
        for (int i = 0; i < 2; ++i) {
            for (cudaEvent_t* ev : {&in_ready_[i], &out_ready_[i], &out_done_[i]}) {
                NVLLM_CUDA_TRY(cudaEventCreateWithFlags(ev, cudaEventDisableTiming));
            }
        }
    }
    const std::size_t n = std::size_t(step_.num_tokens);
    const std::size_t bytes = n * row_floats_ * sizeof(float);
    const std::size_t stride = std::size_t(cfg_.max_tokens) * row_floats_;
    float* dq = d_rows_[slot];
    float* dk = dq + stride;
    float* dv = dq + 2 * stride;
    float* dout = dq + 3 * stride;
    // The slot's device rows were last read by its previous kernels, and its
    // output copied out after them; the uploads wait for that download (already
    // complete when the slot was collected, as it must have been).
    if (slot_used_[slot]) NVLLM_CUDA_TRY(cudaStreamWaitEvent(h2d_stream_, out_done_[slot], 0));
    if (n > 0) {
        NVLLM_CUDA_TRY(cudaMemcpyAsync(dq, h_q_[slot], bytes, cudaMemcpyHostToDevice, h2d_stream_));
        NVLLM_CUDA_TRY(cudaMemcpyAsync(dk, h_k_[slot], bytes, cudaMemcpyHostToDevice, h2d_stream_));
        NVLLM_CUDA_TRY(cudaMemcpyAsync(dv, h_v_[slot], bytes, cudaMemcpyHostToDevice, h2d_stream_));
    }
    NVLLM_CUDA_TRY(cudaEventRecord(in_ready_[slot], h2d_stream_));
    NVLLM_CUDA_TRY(cudaStreamWaitEvent(stream_, in_ready_[slot], 0));
    if (n > 0) {
        if (auto r = attention_device(layer, dq, dk, dv, dout, precision); !r) return r;
    }
    NVLLM_CUDA_TRY(cudaEventRecord(out_ready_[slot], stream_));
    NVLLM_CUDA_TRY(cudaStreamWaitEvent(d2h_stream_, out_ready_[slot], 0));
    if (n > 0) {
        NVLLM_CUDA_TRY(cudaMemcpyAsync(h_out_[slot], dout, bytes, cudaMemcpyDeviceToHost,
                                       d2h_stream_));
    }
    NVLLM_CUDA_TRY(cudaEventRecord(out_done_[slot], d2h_stream_));
    slot_used_[slot] = true;
    in_flight_[slot] = true;
    return {};
}

std::expected<void, EngineError> AttentionEngine::collect(int32_t slot) {
    if (slot < 0 || slot > 1 || !in_flight_[slot]) {
        return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
    }
    in_flight_[slot] = false;
    NVLLM_CUDA_TRY(cudaEventSynchronize(out_done_[slot]));
    return {};
}

}  // namespace nvllm
