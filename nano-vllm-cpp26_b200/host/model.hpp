// DeviceModel: TransformerModel::forward_batch (src/model.cpp:124-312) on one
// GPU, around the AttentionEngine that holds the paged KV arenas.
//
// Weights are the reference's LCG weights (src/model.cpp:64-112), generated on
// the device in the constructor's draw order into one allocation laid out as
// that order: embedding [V, D]; per layer w_q, w_k, w_v, w_o [D, D], w_up
// [D, F], w_down [F, D]; LM head [D, V] (all row-major [k, n], the operand
// layout of matmul_batched). The RMSNorm weights are all ones and are not
// stored (src/model.cpp:88-89).
//
// One forward per engine step, all on the engine's stream: embedding gather,
// per layer RMSNorm, one strided-batched GEMM for Q/K/V (w_q, w_k, w_v are
// adjacent), KV write + paged attention (the engine), W_o GEMM accumulating
// into the residual, RMSNorm, up GEMM, SiLU, down GEMM accumulating into the
// residual; then the last-token gather, the LM-head GEMM and the penalised
// argmax. The projections run on fp32 data: cuBLAS SGEMMs (FFMA on the CUDA
// cores, or with gemm_math 1 cuBLAS's bf16x9 emulation of fp32 on the tensor
// cores), or with gemm_math 2 nvllm_gemm_tf32x3 (tcgen05, 3xTF32 at fp32
// quality, weights kept transposed and pre-split into tf32 hi / lo parts) for
// every projection of more than 32 rows, its epilogue doing the residual add
// (W_o, down), the SiLU (up) and the Q/K/V split; never single-pass TF32.
#pragma once

#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <expected>
#include <map>
#include <memory>
#include <span>
#include <tuple>

#include "engine.hpp"

namespace nvllm {

struct ModelConfig {
    int64_t vocab = 0, hidden = 0, layers = 0, heads = 0, head_dim = 0, ffn = 0;
    // weight scales of src/model.cpp:81-82; 0 = 1/sqrt(hidden), 1/sqrt(ffn)
    float emb_scale = 0.0f, ffn_scale = 0.0f;
    // 0: fp32 FFMA (cuBLAS); 1: fp32 emulated with bf16x9 (cuBLAS); 2: this
    // library's tcgen05 3xTF32 GEMM for projections of more than 32 rows (with
    // the residual add, SiLU and Q/K/V split in its epilogue), cuBLAS FFMA below
    int32_t gemm_math = 0;
    // Steps of at most this many new tokens run as one CUDA graph per padded
    // (tokens, sequences) bucket, captured on first use (0: always eager).
    int32_t graph_max_tokens = 0;
    // Head parallelism over this many GPUs (one process each, <= 8): the engine
    // holds heads / head_ranks heads; set_head_group() names this rank and the
    // gather buffers before the first forward. 1: single GPU.
    int32_t head_ranks = 1;
};

// The peers of a head-parallel model: gather buffers [max_tokens, hidden] on
// every rank by epoch parity, and every rank's flag word (device pointers valid
// in this process: the peers' through CUDA IPC).
struct HeadGroup {
    int32_t rank = 0, world = 1;
    float* outs[2][8] = {};
    uint32_t* flags[8] = {};
};

class DeviceModel {
public:
    // The engine's layout must match the model (layers, heads, head_dim); the
    // model keeps a reference to it.
    static std::expected<std::unique_ptr<DeviceModel>, EngineError> create(const ModelConfig& cfg,
                                                                           AttentionEngine& eng);
    ~DeviceModel();
    DeviceModel(const DeviceModel&) = delete;
    DeviceModel& operator=(const DeviceModel&) = delete;

    const ModelConfig& config() const noexcept { return cfg_; }
    const float* weights() const noexcept { return d_w_; }
    std::size_t weight_floats() const noexcept { return w_floats_; }

    // forward_batch over the step begun with AttentionEngine::begin_step:
    // token_ids = the uncomputed tokens of every sequence in flatten order
    // (taken modulo the vocabulary, src/model.cpp:152), prev_tokens[s] = the
    // sequence's last token (src/model.cpp:297-298). Writes sampled[s]; with
    // top_k > 0 also the top-2 margin of the penalised logits and the top_k
    // largest raw logits of every row. Returns once the results are on the host.
    // A step begun padded (begin_step with pad_seqs / pad_tokens) runs the
    // padded shapes; with graph_max_tokens > 0 it replays the bucket's CUDA
    // graph (captured the first time the bucket is seen). Padded rows compute
    // values nobody reads; they never reach the arena or the results.
    std::expected<void, EngineError> forward(std::span<const int64_t> token_ids,
                                             std::span<const int64_t> prev_tokens,
                                             int64_t* sampled, int32_t precision,
                                             float* margins = nullptr, int32_t* top_idx = nullptr,
                                             float* top_val = nullptr, int32_t top_k = 0);

    // Asynchronous half of forward(): enqueues the whole step on the engine's
    // stream, with the sampled ids left in device memory (device_sampled()).
    std::expected<void, EngineError> enqueue(std::span<const int64_t> token_ids,
                                             std::span<const int64_t> prev_tokens,
                                             int32_t precision, int32_t top_k = 0);
    const int32_t* device_sampled() const noexcept { return d_sampled_; }

    // Head parallelism (config head_ranks > 1): QKV for this rank's heads only
    // (column slices of w_q, w_k, w_v), attention on the engine's head slice,
    // nvllm_head_gather of every rank's attention rows into the gather buffer of
    // the call's epoch parity, then W_o, the FFN and the LM head on the full
    // rows, replicated on every rank (all ranks then sample the same tokens).
    std::expected<void, EngineError> set_head_group(const HeadGroup& g);

    // Totals over every forward so far: launches of this library's kernels
    // (cuBLAS GEMMs not counted) and bytes copied host->device (token ids,
    // previous tokens, the engine's metadata) and device->host (results).
    uint64_t kernel_launches() const noexcept { return launches_; }
    uint64_t graph_launches() const noexcept { return graph_launches_; }
    std::size_t graphs_captured() const noexcept { return graphs_.size(); }
    uint64_t h2d_bytes() const noexcept { return h2d_bytes_; }
    uint64_t d2h_bytes() const noexcept { return d2h_bytes_; }

private:
    DeviceModel(const ModelConfig& cfg, AttentionEngine& eng) : cfg_(cfg), eng_(eng) {}
    std::expected<void, EngineError> init();
    std::expected<void, EngineError> gemm(const float* a, const float* w, float* c, int64_t m,
                                          int64_t k, int64_t n, float beta);
    // the tcgen05 GEMM on the transposed hi / lo weights at draw offset w_off
    std::expected<void, EngineError> gemm_tc(const float* a, int64_t m, int64_t k,
                                             std::size_t w_off, int64_t n, float* const* outs,
                                             int32_t n_outs, int64_t out_block, int64_t ldc,
                                             int32_t epilogue);
    // nvllm_gemm_skinny (rows <= 16) or nvllm_gemm_decode_tc (17-32) on the
    // row-major weights (row stride ldw; batch matrices at stride w_stride)
    std::expected<void, EngineError> gemm_small(const float* a, int64_t m, int64_t k,
                                                const float* w, int64_t ldw, int64_t n,
                                                int32_t batch, int64_t w_stride,
                                                float* const* outs, int32_t epilogue);
    bool use_small(int64_t rows) const noexcept { return use_skinny(rows) || use_decode_tc(rows); }
    std::size_t small_workspace(int64_t m, int64_t n, int64_t k, int32_t batch) const;
    bool use_tc(int64_t rows) const noexcept { return cfg_.gemm_math == 2 && rows > 32; }
    // decode-size projections (<= 32 rows): the FFMA skinny GEMM up to 16 rows,
    // the tcgen05 decode GEMM above (measured crossover on the 4096-wide shapes)
    bool use_skinny(int64_t rows) const noexcept { return cfg_.gemm_math == 2 && rows <= 16; }
    bool use_decode_tc(int64_t rows) const noexcept {
        return cfg_.gemm_math == 2 && rows > 16 && rows <= 32;
    }
    uint64_t step_launches(const MetadataLayout& step) const;
    // the device work of one step (everything after the input upload)
    std::expected<void, EngineError> body(const MetadataLayout& step, int32_t precision,
                                          int32_t top_k);

    ModelConfig cfg_;
    AttentionEngine& eng_;
    HeadGroup heads_;
    bool have_heads_ = false;
    uint32_t gather_epoch_ = 0;
    cublasHandle_t blas_ = nullptr;
    float* d_w_ = nullptr;
    std::size_t w_floats_ = 0;
    // gemm_math 2: every projection and the LM head transposed ([n, k]) and split
    // into tf32 hi / lo parts, at their draw offsets minus the embedding's
    float* d_wt_hi_ = nullptr;
    float* d_wt_lo_ = nullptr;
    void* d_gemm_ws_ = nullptr;
    std::size_t gemm_ws_bytes_ = 0;
    std::size_t layer_floats_ = 0;
    // activations, sized for the engine's max_tokens (T) and max_seqs (S)
    float* d_act_ = nullptr;
    float* d_hidden_ = nullptr;  // [T, D]
    float* d_norm_ = nullptr;    // [T, D]
    float* d_qkv_ = nullptr;     // [3, T, D]
    float* d_attn_ = nullptr;    // [T, D]
    float* d_up_ = nullptr;      // [T, F]
    float* d_last_ = nullptr;    // [S, D]
    float* d_logits_ = nullptr;  // [S, V]
    // per-step inputs (one upload) and results (one download)
    unsigned char* d_io_ = nullptr;
    unsigned char* h_io_ = nullptr;
    std::size_t io_in_bytes_ = 0, io_out_bytes_ = 0;
    int32_t* d_tokens_ = nullptr;   // [T]
    int64_t* d_prev_ = nullptr;     // [S]
    int32_t* d_sampled_ = nullptr;  // [S]
    float* d_margin_ = nullptr;     // [S]
    int32_t* d_top_idx_ = nullptr;  // [S, 32]
    float* d_top_val_ = nullptr;    // [S, 32]
    cudaEvent_t io_done_ = nullptr;
    int32_t last_rows_ = 0;
    uint64_t launches_ = 0, h2d_bytes_ = 0, d2h_bytes_ = 0, graph_launches_ = 0;
    void* d_blas_ws_ = nullptr;           // cuBLAS workspace (graph capture needs a fixed one)
    const uint32_t* d_status_ = nullptr;  // libnvllm's device status word
    // (tokens, sequences, max query rows, precision, top_k) -> instantiated graph
    std::map<std::tuple<int32_t, int32_t, int32_t, int32_t, int32_t>, cudaGraphExec_t> graphs_;
};

}  // namespace nvllm
