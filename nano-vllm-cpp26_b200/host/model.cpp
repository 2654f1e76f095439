#include "model.hpp"

#include <dlfcn.h>

#include <algorithm>
#include <climits>
#include <tuple>
#include <utility>
#include <cmath>

#include "../../include/nvllm_ops.h"

namespace nvllm {

namespace {

constexpr float kRmsEps = 1e-5f;        // src/model.cpp:33
constexpr float kRepeatPenalty = 1.5f;  // src/model.cpp:301
constexpr int32_t kMaxTopK = 32;

std::unexpected<EngineError> cuda_error(cudaError_t e) {
    return std::unexpected(EngineError{EngineError::Kind::Cuda, int(e)});
}
std::unexpected<EngineError> blas_error(cublasStatus_t s) {
    return std::unexpected(EngineError{EngineError::Kind::Blas, int(s)});
}
std::unexpected<EngineError> kernel_error(int rc) {
    return std::unexpected(EngineError{EngineError::Kind::Kernel, rc});
}
std::unexpected<EngineError> invalid() {
    return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
}

#define NVLLM_CUDA_TRY(expr)                          \
    do {                                              \
        const cudaError_t e_ = (expr);                \
        if (e_ != cudaSuccess) return cuda_error(e_); \
    } while (0)
#define NVLLM_BLAS_TRY(expr)                                    \
    do {                                                        \
        const cublasStatus_t s_ = (expr);                       \
        if (s_ != CUBLAS_STATUS_SUCCESS) return blas_error(s_); \
    } while (0)
#define NVLLM_OP_TRY(expr)                           \
    do {                                             \
        const int rc_ = (expr);                      \
        if (rc_ != NVLLM_OK) return kernel_error(rc_); \
    } while (0)

constexpr std::size_t align16(std::size_t x) { return (x + 15) & ~std::size_t(15); }

}  // namespace

std::expected<std::unique_ptr<DeviceModel>, EngineError> DeviceModel::create(
    const ModelConfig& cfg, AttentionEngine& eng) {
    const nvllm_kv_layout& L = eng.config().layout;
    if (cfg.vocab <= 0 || cfg.vocab > INT32_MAX || cfg.hidden <= 0 || cfg.layers <= 0 ||
        cfg.heads <= 0 || cfg.head_dim <= 0 || cfg.ffn <= 0 ||
        cfg.hidden != cfg.heads * cfg.head_dim || cfg.hidden > INT32_MAX ||
        cfg.ffn > INT32_MAX || cfg.head_ranks < 1 || cfg.head_ranks > 8 ||
        cfg.heads % cfg.head_ranks != 0 || L.num_layers != cfg.layers ||
        L.num_heads * cfg.head_ranks != cfg.heads ||
        (cfg.head_ranks > 1 && cfg.graph_max_tokens != 0) ||
        (cfg.head_ranks > 1 && cfg.gemm_math == 2 && (cfg.hidden / cfg.head_ranks) % 128 != 0) ||
        L.head_dim != cfg.head_dim || cfg.emb_scale < 0.0f || cfg.ffn_scale < 0.0f ||
        cfg.gemm_math < 0 || cfg.gemm_math > 2 || cfg.graph_max_tokens < 0 ||
        (cfg.gemm_math == 2 &&
         (cfg.hidden % 128 != 0 || cfg.ffn % 128 != 0 || cfg.vocab % 128 != 0))) {
        return invalid();
    }
    std::unique_ptr<DeviceModel> m(new DeviceModel(cfg, eng));
    if (auto r = m->init(); !r) return std::unexpected(r.error());
    return m;
}

std::expected<void, EngineError> DeviceModel::init() {
    const int64_t V = cfg_.vocab, D = cfg_.hidden, F = cfg_.ffn;
    const int64_t T = eng_.config().max_tokens, S = eng_.config().max_seqs;
    cudaStream_t st = eng_.stream();
    NVLLM_CUDA_TRY(cudaSetDevice(eng_.config().device));
    NVLLM_BLAS_TRY(cublasCreate(&blas_));
    NVLLM_BLAS_TRY(cublasSetStream(blas_, st));
    // fp32 arithmetic: FFMA, or the bf16x9 emulation of fp32 on the tensor
    // cores; never a TF32 down-conversion
    if (cfg_.gemm_math == 1) {
        // the bf16x9 mode needs the cuBLAS of CUDA 12.9 or later in the process
        if (cublasSetMathMode(blas_, CUBLAS_FP32_EMULATED_BF16X9_MATH) != CUBLAS_STATUS_SUCCESS) {
            return std::unexpected(EngineError{EngineError::Kind::Unsupported, 0});
        }
        // Prefer the emulation for every shape where the loaded cuBLAS lets us
        // choose (the setter is absent from some 12.9 builds, which then pick
        // per shape by their own heuristics).
        using SetStrategy = cublasStatus_t (*)(cublasHandle_t, cublasEmulationStrategy_t);
        if (auto fn = reinterpret_cast<SetStrategy>(dlsym(RTLD_DEFAULT, "cublasSetEmulationStrategy"))) {
            NVLLM_BLAS_TRY(fn(blas_, CUBLAS_EMULATION_STRATEGY_EAGER));
        }
    } else {
        NVLLM_BLAS_TRY(cublasSetMathMode(blas_, CUBLAS_DEFAULT_MATH));
    }

    // weights, in the reference constructor's draw order
    layer_floats_ = std::size_t(4 * D * D + 2 * D * F);
    w_floats_ = std::size_t(V * D) + std::size_t(cfg_.layers) * layer_floats_ + std::size_t(D * V);
    NVLLM_CUDA_TRY(cudaMalloc(&d_w_, w_floats_ * sizeof(float)));
    const float emb_scale =
        cfg_.emb_scale > 0.0f ? cfg_.emb_scale : 1.0f / std::sqrt(static_cast<float>(D));
    const float ffn_scale =
        cfg_.ffn_scale > 0.0f ? cfg_.ffn_scale : 1.0f / std::sqrt(static_cast<float>(F));
    uint64_t draw = 0;
    auto fill = [&](int64_t rows, int64_t cols, float scale) -> int {
        const int rc = nvllm_lcg_fill(d_w_ + draw, rows, cols, cols, draw, scale, st);
        draw += uint64_t(rows * cols);
        return rc;
    };
    NVLLM_OP_TRY(fill(V, D, emb_scale));
    for (int64_t l = 0; l < cfg_.layers; ++l) {
        for (int i = 0; i < 4; ++i) NVLLM_OP_TRY(fill(D, D, emb_scale));  // w_q, w_k, w_v, w_o
        NVLLM_OP_TRY(fill(D, F, emb_scale));                               // w_up
        NVLLM_OP_TRY(fill(F, D, ffn_scale));                               // w_down
    }
    NVLLM_OP_TRY(fill(D, V, emb_scale));  // LM head
    if (draw != w_floats_) return invalid();

    if (cfg_.gemm_math == 2) {
        // transposed, tf32-split copies of every [k, n] weight after the embedding
        const std::size_t t_floats = w_floats_ - std::size_t(V * D);
        NVLLM_CUDA_TRY(cudaMalloc(&d_wt_hi_, t_floats * sizeof(float)));
        NVLLM_CUDA_TRY(cudaMalloc(&d_wt_lo_, t_floats * sizeof(float)));
        float* scratch = nullptr;
        NVLLM_CUDA_TRY(cudaMalloc(&scratch, std::size_t(std::max(D * V, D * F)) * sizeof(float)));
        std::size_t off = std::size_t(V * D);
        auto prep = [&](int64_t rows, int64_t cols) -> int {
            int rc = nvllm_transpose(d_w_ + off, rows, cols, scratch, st);
            const std::size_t t = off - std::size_t(V * D);
            if (rc == NVLLM_OK) {
                rc = nvllm_tf32_split(scratch, d_wt_hi_ + t, d_wt_lo_ + t, rows * cols, st);
            }
            off += std::size_t(rows * cols);
            return rc;
        };
        int rc = NVLLM_OK;
        for (int64_t l = 0; l < cfg_.layers && rc == NVLLM_OK; ++l) {
            for (int i = 0; i < 4 && rc == NVLLM_OK; ++i) rc = prep(D, D);
            if (rc == NVLLM_OK) rc = prep(D, F);
            if (rc == NVLLM_OK) rc = prep(F, D);
        }
        if (rc == NVLLM_OK) rc = prep(D, V);
        cudaStreamSynchronize(st);
        cudaFree(scratch);
        if (rc != NVLLM_OK) return kernel_error(rc);
        // split-K partials: the largest any projection of more than 32 rows asks for
        const int64_t tmax = eng_.config().max_tokens;
        for (int64_t m = 33; m <= tmax; ++m) {
            for (const auto& [k, n] : {std::pair{D, 3 * D}, std::pair{D, D}, std::pair{D, F},
                                       std::pair{F, D}, std::pair{D, V},
                                       std::pair{D, D / cfg_.head_ranks}}) {
                gemm_ws_bytes_ = std::max(gemm_ws_bytes_, nvllm_gemm_workspace_size(m, n, k));
            }
        }
        // and what the decode-size GEMMs ask for at <= 32 rows
        for (int64_t m = 1; m <= std::min<int64_t>(tmax, 32); ++m) {
            for (const auto& [k, n, b] : {std::tuple{D, D, 3}, std::tuple{D, D, 1},
                                          std::tuple{D, F, 1}, std::tuple{F, D, 1},
                                          std::tuple{D, V, 1},
                                          std::tuple{D, D / cfg_.head_ranks, 3}}) {
                gemm_ws_bytes_ = std::max(
                    {gemm_ws_bytes_, nvllm_gemm_skinny_workspace_size(m, n, k, int32_t(b)),
                     nvllm_gemm_decode_tc_workspace_size(m, n, k, int32_t(b))});
            }
        }
        if (gemm_ws_bytes_ > 0) NVLLM_CUDA_TRY(cudaMalloc(&d_gemm_ws_, gemm_ws_bytes_));
    }

    const std::size_t act = std::size_t(T * D * 6 + T * F + S * D + S * V);
    NVLLM_CUDA_TRY(cudaMalloc(&d_act_, act * sizeof(float)));
    d_hidden_ = d_act_;
    d_norm_ = d_hidden_ + T * D;
    d_qkv_ = d_norm_ + T * D;
    d_attn_ = d_qkv_ + 3 * T * D;
    d_up_ = d_attn_ + T * D;
    d_last_ = d_up_ + T * F;
    d_logits_ = d_last_ + S * D;

    io_in_bytes_ = align16(std::size_t(T) * 4) + align16(std::size_t(S) * 8);
    // sampled ids, margins, top-k indices and values, then 16 bytes for the
    // status word
    io_out_bytes_ = 2 * align16(std::size_t(S) * 4) + 2 * std::size_t(S) * kMaxTopK * 4 + 16;
    NVLLM_CUDA_TRY(cudaMalloc(&d_io_, io_in_bytes_ + io_out_bytes_));
    NVLLM_CUDA_TRY(cudaMallocHost(&h_io_, io_in_bytes_ + io_out_bytes_));
    d_tokens_ = reinterpret_cast<int32_t*>(d_io_);
    d_prev_ = reinterpret_cast<int64_t*>(d_io_ + align16(std::size_t(T) * 4));
    unsigned char* out = d_io_ + io_in_bytes_;
    d_sampled_ = reinterpret_cast<int32_t*>(out);
    d_margin_ = reinterpret_cast<float*>(out + align16(std::size_t(S) * 4));
    d_top_idx_ = reinterpret_cast<int32_t*>(out + 2 * align16(std::size_t(S) * 4));
    d_top_val_ = reinterpret_cast<float*>(d_top_idx_ + S * kMaxTopK);
    // a fixed cuBLAS workspace: captured GEMMs must not allocate
    constexpr std::size_t kBlasWorkspace = std::size_t(32) << 20;
    NVLLM_CUDA_TRY(cudaMalloc(&d_blas_ws_, kBlasWorkspace));
    NVLLM_BLAS_TRY(cublasSetWorkspace(blas_, d_blas_ws_, kBlasWorkspace));
    NVLLM_OP_TRY(nvllm_device_status_word(&d_status_));
    // activations start finite: padded rows of a bucket read rows no step wrote
    NVLLM_CUDA_TRY(cudaMemsetAsync(d_act_, 0, act * sizeof(float), st));
    NVLLM_CUDA_TRY(cudaEventCreateWithFlags(&io_done_, cudaEventDisableTiming));
    NVLLM_CUDA_TRY(cudaEventRecord(io_done_, st));
    NVLLM_CUDA_TRY(cudaStreamSynchronize(st));
    return {};
}

DeviceModel::~DeviceModel() {
    cudaSetDevice(eng_.config().device);
    cudaStreamSynchronize(eng_.stream());
    for (auto& [key, exec] : graphs_) cudaGraphExecDestroy(exec);
    if (blas_) cublasDestroy(blas_);
    if (d_blas_ws_) cudaFree(d_blas_ws_);
    if (io_done_) cudaEventDestroy(io_done_);
    if (h_io_) cudaFreeHost(h_io_);
    if (d_io_) cudaFree(d_io_);
    if (d_act_) cudaFree(d_act_);
    if (d_w_) cudaFree(d_w_);
    if (d_wt_hi_) cudaFree(d_wt_hi_);
    if (d_wt_lo_) cudaFree(d_wt_lo_);
    if (d_gemm_ws_) cudaFree(d_gemm_ws_);
}

// Row-major C[m, n] = A[m, k] . W[k, n] + beta * C: the column-major product
// C^T = W^T A^T, with W^T and A^T being the row-major buffers read as
// column-major.
std::expected<void, EngineError> DeviceModel::gemm(const float* a, const float* w, float* c,
                                                   int64_t m, int64_t k, int64_t n, float beta) {
    const float one = 1.0f;
    NVLLM_BLAS_TRY(cublasSgemm(blas_, CUBLAS_OP_N, CUBLAS_OP_N, int(n), int(m), int(k), &one, w,
                               int(n), a, int(k), &beta, c, int(n)));
    return {};
}

std::expected<void, EngineError> DeviceModel::gemm_tc(const float* a, int64_t m, int64_t k,
                                                      std::size_t w_off, int64_t n,
                                                      float* const* outs, int32_t n_outs,
                                                      int64_t out_block, int64_t ldc,
                                                      int32_t epilogue) {
    const std::size_t t = w_off - std::size_t(cfg_.vocab * cfg_.hidden);
    NVLLM_OP_TRY(nvllm_gemm_tf32x3(a, k, m, k, d_wt_hi_ + t, d_wt_lo_ + t, n, outs, n_outs,
                                   out_block, ldc, epilogue, d_gemm_ws_, gemm_ws_bytes_,
                                   eng_.stream()));
    return {};
}

std::expected<void, EngineError> DeviceModel::gemm_small(const float* a, int64_t m, int64_t k,
                                                         const float* w, int64_t ldw, int64_t n,
                                                         int32_t batch, int64_t w_stride,
                                                         float* const* outs, int32_t epilogue) {
    if (use_decode_tc(m)) {
        NVLLM_OP_TRY(nvllm_gemm_decode_tc(a, k, m, k, w, ldw, n, batch, w_stride, outs, n,
                                          epilogue, d_gemm_ws_, gemm_ws_bytes_, eng_.stream()));
    } else {
        NVLLM_OP_TRY(nvllm_gemm_skinny(a, k, m, k, w, ldw, n, batch, w_stride, outs, n, epilogue,
                                       d_gemm_ws_, gemm_ws_bytes_, eng_.stream()));
    }
    return {};
}

std::expected<void, EngineError> DeviceModel::set_head_group(const HeadGroup& g) {
    if (g.world != cfg_.head_ranks || g.world < 2 || g.rank < 0 || g.rank >= g.world) {
        return invalid();
    }
    for (int r = 0; r < g.world; ++r) {
        if (g.outs[0][r] == nullptr || g.outs[1][r] == nullptr || g.flags[r] == nullptr) {
            return invalid();
        }
    }
    heads_ = g;
    have_heads_ = true;
    return {};
}

// The workspace of the decode-size GEMM that gemm_small picks for m rows (a
// second, summing kernel runs when it is not 0).
std::size_t DeviceModel::small_workspace(int64_t m, int64_t n, int64_t k, int32_t batch) const {
    return use_decode_tc(m) ? nvllm_gemm_decode_tc_workspace_size(m, n, k, batch)
                            : nvllm_gemm_skinny_workspace_size(m, n, k, batch);
}

// Launches of this library's kernels in one step: embedding, last-token gather
// and sampler; per layer two RMSNorms, the KV write and the attention's plan,
// decode and merge (+ prefill), and either the SiLU (cuBLAS projections) or the
// four tcgen05 / skinny GEMMs (+ their split-K sums); the LM head's own GEMM
// (+ its split-K sum) unless cuBLAS runs it.
uint64_t DeviceModel::step_launches(const MetadataLayout& step) const {
    const int64_t D = cfg_.hidden, F = cfg_.ffn, V = cfg_.vocab;
    const int64_t T = step.num_tokens, S = step.num_seqs;
    const int64_t hr = cfg_.head_ranks, Dl = D / hr;
    // + the head gather (copy, signal, wait) of a head-parallel model
    uint64_t per_layer = 2 + 4 + (step.max_query_len > 1 ? 1 : 0) + (hr > 1 ? 3 : 0);
    if (use_tc(T)) {
        // Q, K, V as one three-way GEMM, or one GEMM each for a head slice
        const int64_t qkv_calls = hr > 1 ? 3 : 1, qkv_n = hr > 1 ? Dl : 3 * D;
        per_layer += uint64_t(qkv_calls) * (1 + (nvllm_gemm_workspace_size(T, qkv_n, D) > 0 ? 1 : 0));
        for (const auto& [k, n] : {std::pair{D, D}, std::pair{D, F}, std::pair{F, D}}) {
            per_layer += 1 + (nvllm_gemm_workspace_size(T, n, k) > 0 ? 1 : 0);
        }
    } else if (use_small(T)) {
        for (const auto& [k, n, b] : {std::tuple{D, Dl, 3}, std::tuple{D, D, 1},
                                      std::tuple{D, F, 1}, std::tuple{F, D, 1}}) {
            per_layer += 1 + (small_workspace(T, n, k, int32_t(b)) > 0 ? 1 : 0);
        }
    } else {
        per_layer += 1;
    }
    uint64_t total = 3 + uint64_t(cfg_.layers) * per_layer;
    if (use_tc(S)) {
        total += 1 + (nvllm_gemm_workspace_size(S, V, D) > 0 ? 1 : 0);
    } else if (use_small(S)) {
        total += 1 + (small_workspace(S, V, D, 1) > 0 ? 1 : 0);
    }
    return total;
}

std::expected<void, EngineError> DeviceModel::enqueue(std::span<const int64_t> token_ids,
                                                      std::span<const int64_t> prev_tokens,
                                                      int32_t precision, int32_t top_k) {
    const MetadataLayout& step = eng_.step();
    if (!eng_.has_step() || token_ids.size() != std::size_t(step.real_tokens) ||
        prev_tokens.size() != std::size_t(step.real_seqs) || top_k < 0 || top_k > kMaxTopK) {
        return invalid();
    }
    const int64_t V = cfg_.vocab;
    const int64_t T = step.num_tokens, S = step.num_seqs;  // as laid out (padded or not)
    last_rows_ = step.real_seqs;
    if (step.real_seqs == 0) return {};
    cudaStream_t st = eng_.stream();
    NVLLM_CUDA_TRY(cudaSetDevice(eng_.config().device));

    // inputs: token ids modulo the vocabulary (src/model.cpp:152) and the
    // previous tokens, one upload from pinned staging; padded rows get token 0
    NVLLM_CUDA_TRY(cudaEventSynchronize(io_done_));
    auto* h_tok = reinterpret_cast<int32_t*>(h_io_);
    auto* h_prev = reinterpret_cast<int64_t*>(h_io_ + align16(std::size_t(eng_.config().max_tokens) * 4));
    for (std::size_t t = 0; t < token_ids.size(); ++t) {
        if (token_ids[t] < 0) return invalid();
        h_tok[t] = int32_t(token_ids[t] % V);
    }
    for (int64_t t = int64_t(token_ids.size()); t < T; ++t) h_tok[t] = 0;
    for (std::size_t s = 0; s < prev_tokens.size(); ++s) h_prev[s] = prev_tokens[s];
    for (int64_t s = int64_t(prev_tokens.size()); s < S; ++s) h_prev[s] = 0;
    NVLLM_CUDA_TRY(cudaMemcpyAsync(d_io_, h_io_, io_in_bytes_, cudaMemcpyHostToDevice, st));
    NVLLM_CUDA_TRY(cudaEventRecord(io_done_, st));
    launches_ += step_launches(step);
    h2d_bytes_ += io_in_bytes_ + step.bytes;

    if (!(step.padded && cfg_.graph_max_tokens > 0)) return body(step, precision, top_k);
    const auto key = std::make_tuple(int32_t(T), int32_t(S), step.max_query_len, precision, top_k);
    auto it = graphs_.find(key);
    if (it == graphs_.end()) {
        NVLLM_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        auto r = body(step, precision, top_k);
        cudaGraph_t graph = nullptr;
        const cudaError_t e = cudaStreamEndCapture(st, &graph);
        if (!r || e != cudaSuccess) {
            if (graph != nullptr) cudaGraphDestroy(graph);
            if (!r) return r;
            return cuda_error(e);
        }
        cudaGraphExec_t exec = nullptr;
        const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ie != cudaSuccess) return cuda_error(ie);
        it = graphs_.emplace(key, exec).first;
    }
    NVLLM_CUDA_TRY(cudaGraphLaunch(it->second, st));
    ++graph_launches_;
    return {};
}

std::expected<void, EngineError> DeviceModel::body(const MetadataLayout& step, int32_t precision,
                                                   int32_t top_k) {
    const int64_t V = cfg_.vocab, D = cfg_.hidden, F = cfg_.ffn;
    const int64_t T = step.num_tokens, S = step.num_seqs;
    const int32_t hr = cfg_.head_ranks;
    if (hr > 1 && !have_heads_) return invalid();
    cudaStream_t st = eng_.stream();
    const float* emb = d_w_;
    NVLLM_OP_TRY(nvllm_embedding_gather(d_hidden_, emb, d_tokens_, T, V, D, st));
    const float one = 1.0f, zero = 0.0f;
    for (int64_t l = 0; l < cfg_.layers; ++l) {
        const float* lw = d_w_ + V * D + std::size_t(l) * layer_floats_;
        const float* w_q = lw;  // w_q, w_k, w_v: three adjacent [D, D]
        const float* w_o = lw + 3 * D * D;
        const float* w_up = lw + 4 * D * D;
        const float* w_down = w_up + D * F;
        const std::size_t l_off = std::size_t(V * D) + std::size_t(l) * layer_floats_;
        // this rank's heads: columns [c0, c0 + Dl) of w_q, w_k, w_v (all of them on
        // one GPU)
        const int64_t Dl = D / hr, c0 = int64_t(heads_.rank) * Dl;
        float* q = d_qkv_;
        float* k = d_qkv_ + T * Dl;
        float* v = d_qkv_ + 2 * T * Dl;
        NVLLM_OP_TRY(nvllm_rms_norm(d_norm_, d_hidden_, nullptr, T, D, kRmsEps, st));
        // Q, K, V = norm . {w_q, w_k, w_v} (src/model.cpp:184-186): one GEMM over the
        // stacked transposed weights with a three-way output (one per matrix for a
        // head slice), or one batched GEMM
        if (use_tc(T)) {
            if (hr == 1) {
                float* const outs[3] = {q, k, v};
                if (auto r = gemm_tc(d_norm_, T, D, l_off, 3 * D, outs, 3, D, D, NVLLM_GEMM_STORE);
                    !r) {
                    return r;
                }
            } else {
                float* const qkv[3] = {q, k, v};
                for (int i = 0; i < 3; ++i) {
                    float* const outs[1] = {qkv[i]};
                    // rows c0.. of the transposed matrix i
                    if (auto r = gemm_tc(d_norm_, T, D, l_off + std::size_t(i * D * D + c0 * D), Dl,
                                         outs, 1, Dl, Dl, NVLLM_GEMM_STORE);
                        !r) {
                        return r;
                    }
                }
            }
        } else if (use_small(T)) {
            float* const outs[3] = {q, k, v};
            if (auto r = gemm_small(d_norm_, T, D, w_q + c0, D, Dl, 3, D * D, outs, NVLLM_GEMM_STORE);
                !r) {
                return r;
            }
        } else {
            NVLLM_BLAS_TRY(cublasSgemmStridedBatched(blas_, CUBLAS_OP_N, CUBLAS_OP_N, int(Dl),
                                                     int(T), int(D), &one, w_q + c0, int(D), D * D,
                                                     d_norm_, int(D), 0, &zero, d_qkv_, int(Dl),
                                                     T * Dl, 3));
        }
        if (auto r = eng_.attention_device(int32_t(l), q, k, v, d_attn_, precision); !r) return r;
        const float* attn = d_attn_;
        if (hr > 1) {
            // every rank's heads into the gather buffer of this call's epoch parity
            nvllm_head_split hs{};
            hs.rank = heads_.rank;
            hs.world = hr;
            hs.epoch = ++gather_epoch_;
            for (int r = 0; r < hr; ++r) {
                hs.outs[r] = heads_.outs[hs.epoch & 1u][r];
                hs.flags[r] = heads_.flags[r];
            }
            NVLLM_OP_TRY(nvllm_head_gather(d_attn_, T, Dl, &hs, st));
            attn = heads_.outs[hs.epoch & 1u][heads_.rank];
        }
        // hidden += attn . w_o (src/model.cpp:263-266)
        if (use_tc(T)) {
            float* const outs[1] = {d_hidden_};
            if (auto r = gemm_tc(attn, T, D, l_off + 3 * D * D, D, outs, 1, D, D,
                                 NVLLM_GEMM_ACCUMULATE);
                !r) {
                return r;
            }
        } else if (use_small(T)) {
            float* const outs[1] = {d_hidden_};
            if (auto r = gemm_small(attn, T, D, w_o, D, D, 1, 0, outs, NVLLM_GEMM_ACCUMULATE); !r) {
                return r;
            }
        } else if (auto r = gemm(attn, w_o, d_hidden_, T, D, D, 1.0f); !r) {
            return r;
        }
        NVLLM_OP_TRY(nvllm_rms_norm(d_norm_, d_hidden_, nullptr, T, D, kRmsEps, st));
        // up = silu(norm . w_up) (src/model.cpp:270-273)
        if (use_tc(T)) {
            float* const outs[1] = {d_up_};
            if (auto r = gemm_tc(d_norm_, T, D, l_off + 4 * D * D, F, outs, 1, F, F,
                                 NVLLM_GEMM_SILU);
                !r) {
                return r;
            }
        } else if (use_small(T)) {
            float* const outs[1] = {d_up_};
            if (auto r = gemm_small(d_norm_, T, D, w_up, F, F, 1, 0, outs, NVLLM_GEMM_SILU); !r) {
                return r;
            }
        } else {
            if (auto r = gemm(d_norm_, w_up, d_up_, T, D, F, 0.0f); !r) return r;
            NVLLM_OP_TRY(nvllm_silu(d_up_, T * F, st));
        }
        // hidden += up . w_down (src/model.cpp:274-277)
        if (use_tc(T)) {
            float* const outs[1] = {d_hidden_};
            if (auto r = gemm_tc(d_up_, T, F, l_off + 4 * D * D + D * F, D, outs, 1, D, D,
                                 NVLLM_GEMM_ACCUMULATE);
                !r) {
                return r;
            }
        } else if (use_small(T)) {
            float* const outs[1] = {d_hidden_};
            if (auto r = gemm_small(d_up_, T, F, w_down, D, D, 1, 0, outs, NVLLM_GEMM_ACCUMULATE); !r) {
                return r;
            }
        } else if (auto r = gemm(d_up_, w_down, d_hidden_, T, F, D, 1.0f); !r) {
            return r;
        }
    }
    const auto* last_idx = reinterpret_cast<const int32_t*>(eng_.device_metadata() + step.last_off);
    NVLLM_OP_TRY(nvllm_gather_rows(d_last_, d_hidden_, last_idx, S, T, D, st));
    const std::size_t lm_off = std::size_t(V * D) + std::size_t(cfg_.layers) * layer_floats_;
    if (use_tc(S)) {
        float* const outs[1] = {d_logits_};
        if (auto r = gemm_tc(d_last_, S, D, lm_off, V, outs, 1, V, V, NVLLM_GEMM_STORE); !r) {
            return r;
        }
    } else if (use_small(S)) {
        float* const outs[1] = {d_logits_};
        if (auto r = gemm_small(d_last_, S, D, d_w_ + lm_off, V, V, 1, 0, outs, NVLLM_GEMM_STORE); !r) {
            return r;
        }
    } else if (auto r = gemm(d_last_, d_w_ + lm_off, d_logits_, S, D, V, 0.0f); !r) {
        return r;
    }
    NVLLM_OP_TRY(nvllm_penalized_argmax(d_logits_, d_prev_, S, V, kRepeatPenalty, d_sampled_,
                                        top_k > 0 ? d_margin_ : nullptr,
                                        top_k > 0 ? d_top_idx_ : nullptr,
                                        top_k > 0 ? d_top_val_ : nullptr, top_k, st));
    return {};
}

std::expected<void, EngineError> DeviceModel::forward(std::span<const int64_t> token_ids,
                                                      std::span<const int64_t> prev_tokens,
                                                      int64_t* sampled, int32_t precision,
                                                      float* margins, int32_t* top_idx,
                                                      float* top_val, int32_t top_k) {
    if (auto r = enqueue(token_ids, prev_tokens, precision, top_k); !r) return r;
    const int64_t S = last_rows_;
    if (S == 0) return {};
    if (sampled == nullptr) return invalid();
    cudaStream_t st = eng_.stream();
    unsigned char* h_out = h_io_ + io_in_bytes_;
    const std::size_t bytes = top_k > 0 ? io_out_bytes_ - 16 : std::size_t(S) * 4;
    NVLLM_CUDA_TRY(cudaMemcpyAsync(h_out, d_io_ + io_in_bytes_, bytes, cudaMemcpyDeviceToHost, st));
    // the kernels' status word rides along with the results (4 bytes)
    auto* h_status = reinterpret_cast<uint32_t*>(h_out + io_out_bytes_ - 16);
    NVLLM_CUDA_TRY(cudaMemcpyAsync(h_status, d_status_, 4, cudaMemcpyDeviceToHost, st));
    d2h_bytes_ += bytes + 4;
    NVLLM_CUDA_TRY(cudaStreamSynchronize(st));
    if (*h_status != 0) {
        const int32_t status = nvllm_get_last_error(st);  // decodes and clears it
        if (status != NVLLM_OK) return kernel_error(status);
    }
    const int64_t S_cap = eng_.config().max_seqs;
    const auto* h_sampled = reinterpret_cast<const int32_t*>(h_out);
    for (int64_t s = 0; s < S; ++s) sampled[s] = h_sampled[s];
    if (top_k > 0) {
        const auto* h_margin = reinterpret_cast<const float*>(h_out + align16(std::size_t(S_cap) * 4));
        const auto* h_ti = reinterpret_cast<const int32_t*>(h_out + 2 * align16(std::size_t(S_cap) * 4));
        const auto* h_tv = reinterpret_cast<const float*>(h_ti + S_cap * kMaxTopK);
        for (int64_t s = 0; s < S; ++s) {
            if (margins) margins[s] = h_margin[s];
            for (int32_t j = 0; j < top_k; ++j) {
                if (top_idx) top_idx[s * top_k + j] = h_ti[s * top_k + j];
                if (top_val) top_val[s * top_k + j] = h_tv[s * top_k + j];
            }
        }
    }
    return {};
}

}  // namespace nvllm
