// Test infrastructure: a C entry layer over the reference's OWN C++ code for the
// paged-KV write + paged attention path. It is the checker that pins the C
// restatement in nvllm_oracle.c and generates the golden fixtures; nothing in
// the product links or loads it.
//
// What runs here is unmodified reference code:
//   - nano_vllm::PagedKVCache (src/kv_cache.cpp) for the block allocator, the
//     arena, write_kv and read_head_kv;
//   - nano_vllm::TransformerModel::forward_batch (src/model.cpp:124-312), whose
//     step 3c (KV write, :188-202) and step 3d (paged online-softmax attention,
//     :204-260) are the path under test;
//   - nano_vllm::ThreadPool (include/nano_vllm/thread_pool.hpp) as its CPU grid.
//
// The harness defines nano_vllm::matmul_batched (declared at
// include/nano_vllm/model.hpp:57-64). Because the reference core is a separate
// -fPIC shared object, forward_batch's calls to it bind to this definition. Per
// layer forward_batch calls it six times in a fixed order (model.cpp:184-186 Q,
// K, V; :263 W_o; :270 up; :274 down) and once more for the LM head (:291). The
// harness answers the Q/K/V calls with caller-supplied projections, records the
// attention output that arrives as the A operand of the W_o call, and returns
// zeros for the rest. The attention outputs are therefore exactly what the
// reference's own loop computes for the given Q/K/V and KV history. With no
// capture active the definition forwards to the reference's own matmul_batched,
// so ref_generate runs the unmodified model end to end.

#include "nano_vllm/kv_cache.hpp"
#include "nano_vllm/model.hpp"
#include "nano_vllm/scheduler.hpp"
#include "nano_vllm/thread_pool.hpp"

#include <dlfcn.h>

#include <algorithm>
#include <array>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <vector>

namespace {

struct MatmulPlan {
    std::size_t call = 0;
    std::size_t num_layers = 0;
    std::size_t n_tokens = 0;
    std::size_t hidden = 0;
    const float* q = nullptr;  // [L][n_tokens][hidden]
    const float* k = nullptr;
    const float* v = nullptr;
    float* attn_out = nullptr;  // [L][n_tokens][hidden]
    bool active = false;
};

MatmulPlan g_plan;

// LM-head capture for ref_generate: the (6 * layers)-th matmul_batched call of a
// forward_batch is the LM head (src/model.cpp:291); its output is kept.
struct LogitsCapture {
    bool active = false;
    std::size_t call = 0;
    std::size_t target = 0;
    std::vector<float> logits;
};
LogitsCapture g_lm;

// Operand capture for ref_model_operands: every matmul_batched call of one
// forward_batch keeps copies of its A and W operands and its (batch, k, n).
// The W operands are the model's LCG weights (src/model.cpp:71-112) in the
// order forward_batch uses them.
struct OperandCapture {
    bool active = false;
    std::vector<std::vector<float>> a, w;
    std::vector<std::array<std::size_t, 3>> dims;
};
OperandCapture g_ops;

using MatmulFn = void (*)(std::span<const float>, std::span<const float>, std::span<float>,
                          std::size_t, std::size_t, std::size_t, nano_vllm::ThreadPool&);

// The reference's own matmul_batched (src/model.cpp:42-62), found behind the
// harness's interposing definition; used whenever no attention capture is active.
MatmulFn reference_matmul();

struct RefEngine {
    std::unique_ptr<nano_vllm::TransformerModel> model;
    std::unique_ptr<nano_vllm::ThreadPool> pool;
    std::size_t num_layers = 0;
    std::size_t hidden = 0;
};

}  // namespace

namespace nano_vllm {

void matmul_batched(
    std::span<const float> a,
    std::span<const float> w,
    std::span<float> c,
    std::size_t batch_size,
    std::size_t k_dim,
    std::size_t n_dim,
    ThreadPool& pool) {
    const std::size_t count = batch_size * n_dim;
    if (!g_plan.active) {
        if (MatmulFn f = reference_matmul()) {
            f(a, w, c, batch_size, k_dim, n_dim, pool);
        } else {
            std::fill_n(c.data(), count, 0.0f);
        }
        if (g_lm.active && g_lm.call++ == g_lm.target) g_lm.logits.assign(c.begin(), c.begin() + count);
        if (g_ops.active) {
            g_ops.a.emplace_back(a.begin(), a.begin() + batch_size * k_dim);
            g_ops.w.emplace_back(w.begin(), w.begin() + k_dim * n_dim);
            g_ops.dims.push_back({batch_size, k_dim, n_dim});
        }
        return;
    }
    const std::size_t call = g_plan.call++;
    const std::size_t layer = call / 6;
    const std::size_t which = call % 6;
    const std::size_t per_layer = g_plan.n_tokens * g_plan.hidden;
    if (layer < g_plan.num_layers && which <= 2) {
        const float* src = which == 0 ? g_plan.q : (which == 1 ? g_plan.k : g_plan.v);
        std::copy_n(src + layer * per_layer, count, c.data());
        return;
    }
    if (layer < g_plan.num_layers && which == 3 && g_plan.attn_out != nullptr) {
        std::copy_n(a.data(), per_layer, g_plan.attn_out + layer * per_layer);
    }
    std::fill_n(c.data(), count, 0.0f);
}

}  // namespace nano_vllm

namespace {
MatmulFn reference_matmul() {
    static MatmulFn fn = [] {
        Dl_info info{};
        if (dladdr(reinterpret_cast<void*>(&nano_vllm::matmul_batched), &info) == 0 ||
            info.dli_sname == nullptr) {
            return MatmulFn{nullptr};
        }
        return reinterpret_cast<MatmulFn>(dlsym(RTLD_NEXT, info.dli_sname));
    }();
    return fn;
}
}  // namespace

using nano_vllm::BlockId;
using nano_vllm::PagedKVCache;

extern "C" {

void* ref_cache_create(int64_t num_blocks, int32_t block_size, int32_t num_layers,
                       int32_t num_heads, int32_t head_dim) {
    nano_vllm::KVCacheConfig cfg{
        .num_blocks = static_cast<std::size_t>(num_blocks),
        .block_size = static_cast<std::size_t>(block_size),
        .num_layers = static_cast<std::size_t>(num_layers),
        .num_heads = static_cast<std::size_t>(num_heads),
        .head_dim = static_cast<std::size_t>(head_dim),
    };
    return new PagedKVCache(cfg);
}

void ref_cache_destroy(void* cache) { delete static_cast<PagedKVCache*>(cache); }

int64_t ref_cache_num_free(void* cache) {
    return static_cast<int64_t>(static_cast<PagedKVCache*>(cache)->num_free_blocks());
}

double ref_cache_utilization(void* cache) {
    return static_cast<PagedKVCache*>(cache)->utilization();
}

// 0 = ok, 1 = KVError::OutOfPhysicalBlocks.
int ref_cache_allocate_block(void* cache, int64_t* out) {
    auto r = static_cast<PagedKVCache*>(cache)->allocate_block();
    if (!r.has_value()) return 1;
    *out = static_cast<int64_t>(*r);
    return 0;
}

int ref_cache_allocate_blocks(void* cache, int64_t count, int64_t* out) {
    auto r = static_cast<PagedKVCache*>(cache)->allocate_blocks(static_cast<std::size_t>(count));
    if (!r.has_value()) return 1;
    for (std::size_t i = 0; i < r->size(); ++i) out[i] = static_cast<int64_t>((*r)[i]);
    return 0;
}

void ref_cache_free_blocks(void* cache, const int64_t* ids, int64_t n) {
    std::vector<BlockId> v(ids, ids + n);
    static_cast<PagedKVCache*>(cache)->free_blocks(v);
}

void ref_cache_write_kv(void* cache, int64_t block, int32_t layer, int32_t slot,
                        const float* k, const float* v) {
    auto* c = static_cast<PagedKVCache*>(cache);
    const std::size_t d = c->config().hidden_dim();
    c->write_kv(static_cast<BlockId>(block), static_cast<std::size_t>(layer),
                static_cast<std::size_t>(slot), std::span<const float>{k, d},
                std::span<const float>{v, d});
}

void ref_cache_read_head_kv(void* cache, int64_t block, int32_t layer, int32_t slot,
                            int32_t head, float* k_out, float* v_out) {
    auto* c = static_cast<PagedKVCache*>(cache);
    auto [k, v] = c->read_head_kv(static_cast<BlockId>(block), static_cast<std::size_t>(layer),
                                  static_cast<std::size_t>(slot), static_cast<std::size_t>(head));
    std::memcpy(k_out, k.data(), k.size() * sizeof(float));
    std::memcpy(v_out, v.data(), v.size() * sizeof(float));
}

// Writes the KV history of a batch: for sequence s, positions [0, n_prior[s])
// of every layer, rows taken in order from k/v laid out [L][sum n_prior][D],
// through PagedKVCache::write_kv at (block_table[pos / B], layer, pos % B), the
// same addressing forward_batch uses (src/model.cpp:192-194).
void ref_cache_write_history(void* cache, int32_t num_seqs, const int32_t* n_prior,
                             const int64_t* block_tables, int32_t max_blocks,
                             const float* k, const float* v) {
    auto* c = static_cast<PagedKVCache*>(cache);
    const std::size_t d = c->config().hidden_dim();
    const std::size_t bs = c->block_size();
    const std::size_t L = c->config().num_layers;
    std::size_t total = 0;
    for (int32_t s = 0; s < num_seqs; ++s) total += static_cast<std::size_t>(n_prior[s]);
    for (std::size_t layer = 0; layer < L; ++layer) {
        std::size_t row = 0;
        for (int32_t s = 0; s < num_seqs; ++s) {
            for (int32_t p = 0; p < n_prior[s]; ++p, ++row) {
                const BlockId blk = static_cast<BlockId>(
                    block_tables[static_cast<std::size_t>(s) * max_blocks + p / bs]);
                const std::size_t off = (layer * total + row) * d;
                c->write_kv(blk, layer, p % bs, std::span<const float>{k + off, d},
                            std::span<const float>{v + off, d});
            }
        }
    }
}

void* ref_engine_create(int32_t num_layers, int32_t num_heads, int32_t head_dim,
                        int32_t num_threads) {
    auto* e = new RefEngine;
    nano_vllm::ModelConfig mc{
        .vocab_size = 2,
        .hidden_dim = static_cast<std::size_t>(num_heads) * head_dim,
        .num_layers = static_cast<std::size_t>(num_layers),
        .num_heads = static_cast<std::size_t>(num_heads),
        .head_dim = static_cast<std::size_t>(head_dim),
        .ffn_dim = 1,
    };
    e->model = std::make_unique<nano_vllm::TransformerModel>(mc);
    e->pool = std::make_unique<nano_vllm::ThreadPool>(
        num_threads > 0 ? static_cast<std::size_t>(num_threads)
                        : std::thread::hardware_concurrency());
    e->num_layers = mc.num_layers;
    e->hidden = mc.hidden_dim;
    return e;
}

// Runs the reference forward_batch over num_seqs sequences. Sequence s has
// ctx_lens[s] tokens of which the last q_lens[s] are uncomputed (the reference's
// SequenceState::num_computed_tokens = ctx - q_len); its block table is the
// first ceil(ctx/B) entries of row s of block_tables. q/k/v are the per-layer
// projections of the flattened uncomputed tokens ([L][n_tok][D], flatten order
// of src/model.cpp:144-157); attn_out receives the reference attention output
// in the same layout. Returns the number of flattened tokens, or -1.
int64_t ref_forward_attention(void* engine, void* cache, int32_t num_seqs,
                              const int32_t* q_lens, const int32_t* ctx_lens,
                              const int64_t* block_tables, int32_t max_blocks,
                              const float* q, const float* k, const float* v,
                              float* attn_out) {
    auto* e = static_cast<RefEngine*>(engine);
    auto* c = static_cast<PagedKVCache*>(cache);
    const std::size_t bs = c->block_size();
    std::vector<nano_vllm::SequenceState> seqs;
    seqs.reserve(static_cast<std::size_t>(num_seqs));
    std::size_t n_tok = 0;
    for (int32_t s = 0; s < num_seqs; ++s) {
        if (ctx_lens[s] < 1 || q_lens[s] < 1 || q_lens[s] > ctx_lens[s]) return -1;
        std::vector<std::size_t> toks(static_cast<std::size_t>(ctx_lens[s]), 1);
        nano_vllm::SequenceState st(static_cast<nano_vllm::SeqId>(s + 1), std::move(toks), 1);
        st.num_computed_tokens = static_cast<std::size_t>(ctx_lens[s] - q_lens[s]);
        const std::size_t nb = (static_cast<std::size_t>(ctx_lens[s]) + bs - 1) / bs;
        if (nb > static_cast<std::size_t>(max_blocks)) return -1;
        for (std::size_t b = 0; b < nb; ++b) {
            st.block_table.push_back(
                static_cast<BlockId>(block_tables[static_cast<std::size_t>(s) * max_blocks + b]));
        }
        n_tok += static_cast<std::size_t>(q_lens[s]);
        seqs.push_back(std::move(st));
    }
    g_plan = MatmulPlan{.call = 0, .num_layers = e->num_layers, .n_tokens = n_tok,
                        .hidden = e->hidden, .q = q, .k = k, .v = v, .attn_out = attn_out,
                        .active = true};
    auto sampled = e->model->forward_batch(seqs, *c, *e->pool);
    g_plan.active = false;
    (void)sampled;
    return static_cast<int64_t>(n_tok);
}

// Runs the reference's continuous-batching loop (src/benchmark.cpp:163-229:
// schedule_step -> forward_batch over running() -> process_step_outputs) with
// the reference TransformerModel (real matmuls, LCG weights of
// src/model.cpp:64-122) on `num_requests` requests, and writes a trace of every
// step to `path` as little-endian int64 records:
//   step header:  -1, step index, n_running
//   per running sequence, in running() order:
//     seq_id, num_computed, total_len, prev_token (tokens.back()),
//     table_len, table[table_len], n_uncomputed, uncomputed tokens[n_uncomputed]
//   step footer:  -2, then n_running sampled token ids, then per sequence the
//     top-2 margin of the penalised logits (src/model.cpp:294-309) and the 8
//     largest raw logits as (index, value) pairs; float values are stored as
//     their 32-bit patterns
// path NULL: no trace (timing runs). loop_seconds (may be NULL) receives the
// wall time of the scheduling loop alone, model construction excluded.
// Returns the number of steps, or -1 (cannot open path / bad arguments).
int64_t ref_generate(int64_t vocab, int64_t hidden, int64_t layers, int64_t heads, int64_t head_dim,
                     int64_t ffn, int64_t num_blocks, int64_t block_size, int64_t max_batch,
                     int64_t max_tokens_per_step, int64_t watermark, int64_t num_requests,
                     const int64_t* prompt_lens, const int64_t* prompt_tokens,
                     const int64_t* max_new_tokens, int32_t num_threads, int64_t max_steps,
                     const char* path, double* loop_seconds) {
    if (num_requests < 0 || hidden != heads * head_dim) return -1;
    std::FILE* f = path != nullptr ? std::fopen(path, "wb") : nullptr;
    if (path != nullptr && f == nullptr) return -1;
    const bool tracing = f != nullptr;
    auto put = [f](int64_t v) {
        if (f != nullptr) std::fwrite(&v, sizeof(v), 1, f);
    };
    nano_vllm::ModelConfig mc{.vocab_size = std::size_t(vocab), .hidden_dim = std::size_t(hidden),
                              .num_layers = std::size_t(layers), .num_heads = std::size_t(heads),
                              .head_dim = std::size_t(head_dim), .ffn_dim = std::size_t(ffn)};
    nano_vllm::TransformerModel model(mc);
    nano_vllm::ThreadPool pool(num_threads > 0 ? std::size_t(num_threads)
                                               : std::thread::hardware_concurrency());
    nano_vllm::PagedKVCache cache(nano_vllm::KVCacheConfig{
        .num_blocks = std::size_t(num_blocks), .block_size = std::size_t(block_size),
        .num_layers = std::size_t(layers), .num_heads = std::size_t(heads),
        .head_dim = std::size_t(head_dim)});
    nano_vllm::ContinuousScheduler sched(nano_vllm::SchedulerConfig{
        .max_batch_size = std::size_t(max_batch),
        .max_tokens_per_step = std::size_t(max_tokens_per_step),
        .watermark_blocks = std::size_t(watermark), .eos_token_id = std::nullopt});
    int64_t off = 0;
    for (int64_t i = 0; i < num_requests; ++i) {
        std::vector<std::size_t> prompt;
        for (int64_t j = 0; j < prompt_lens[i]; ++j) prompt.push_back(std::size_t(prompt_tokens[off + j]));
        off += prompt_lens[i];
        sched.add_request(nano_vllm::SequenceState(nano_vllm::SeqId(i + 1), std::move(prompt),
                                                   std::size_t(max_new_tokens[i]), nullptr));
    }
    int64_t step = 0;
    g_plan.active = false;
    const auto t_loop = std::chrono::steady_clock::now();
    while (sched.has_pending_work() && (max_steps <= 0 || step < max_steps)) {
        (void)sched.schedule_step(cache);
        const auto running = sched.running();
        put(-1);
        put(step);
        put(int64_t(running.size()));
        for (const auto& seq : running) {
            put(int64_t(seq.seq_id));
            put(int64_t(seq.num_computed_tokens));
            put(int64_t(seq.tokens.size()));
            put(seq.tokens.empty() ? 0 : int64_t(seq.tokens.back()));
            put(int64_t(seq.block_table.size()));
            for (const BlockId b : seq.block_table) put(int64_t(b));
            const auto unc = seq.uncomputed_tokens();
            put(int64_t(unc.size()));
            for (const std::size_t t : unc) put(int64_t(t));
        }
        g_lm = LogitsCapture{.active = tracing, .call = 0, .target = std::size_t(6 * layers),
                             .logits = {}};
        const auto sampled = model.forward_batch(running, cache, pool);
        g_lm.active = false;
        put(-2);
        for (const std::size_t t : sampled) put(int64_t(t));
        auto bits = [](float x) { uint32_t u; std::memcpy(&u, &x, 4); return int64_t(u); };
        for (std::size_t i = 0; tracing && i < running.size(); ++i) {
            const float* row = g_lm.logits.data() + i * std::size_t(vocab);
            const std::size_t prev = running[i].tokens.empty() ? 0 : running[i].tokens.back();
            float b1 = -INFINITY, b2 = -INFINITY;
            for (int64_t t = 0; t < vocab; ++t) {
                const float adj = std::size_t(t) == prev ? row[t] - 1.5f : row[t];
                if (adj > b1) { b2 = b1; b1 = adj; } else if (adj > b2) { b2 = adj; }
            }
            put(bits(b1 - b2));
            std::vector<int64_t> idx(static_cast<std::size_t>(vocab));
            for (int64_t t = 0; t < vocab; ++t) idx[std::size_t(t)] = t;
            std::partial_sort(idx.begin(), idx.begin() + 8, idx.end(),
                              [row](int64_t x, int64_t y) { return row[x] > row[y] || (row[x] == row[y] && x < y); });
            for (int j = 0; j < 8; ++j) {
                put(idx[std::size_t(j)]);
                put(bits(row[idx[std::size_t(j)]]));
            }
        }
        (void)sched.process_step_outputs(sampled, cache, model.vocab());
        ++step;
    }
    if (loop_seconds != nullptr) {
        *loop_seconds =
            std::chrono::duration<double>(std::chrono::steady_clock::now() - t_loop).count();
    }
    if (f != nullptr) std::fclose(f);
    return step;
}

// 1.0f / std::sqrt(x) as the reference computes its weight and softmax scales
// (src/model.cpp:81-82, :205), compiled with the reference's flags: under
// -ffast-math GCC lowers it to rsqrtss plus one Newton step, which can differ
// from the correctly rounded value in the last place.
float ref_inv_sqrt(float x) { return 1.0f / std::sqrt(x); }

// Builds the reference TransformerModel for the given configuration and runs one
// forward_batch over a single one-token sequence (token id `token`, one block of
// a fresh cache), capturing the A and W operands of every matmul_batched call
// (per layer Q, K, V, W_o, up, down; then the LM head). Returns the number of
// calls captured; ref_operand_dims / ref_operand_copy read them back.
int64_t ref_model_operands(int64_t vocab, int64_t hidden, int64_t layers, int64_t heads,
                           int64_t head_dim, int64_t ffn, int64_t token) {
    if (hidden != heads * head_dim || token < 0) return -1;
    nano_vllm::ModelConfig mc{.vocab_size = std::size_t(vocab), .hidden_dim = std::size_t(hidden),
                              .num_layers = std::size_t(layers), .num_heads = std::size_t(heads),
                              .head_dim = std::size_t(head_dim), .ffn_dim = std::size_t(ffn)};
    nano_vllm::TransformerModel model(mc);
    nano_vllm::ThreadPool pool(1);
    nano_vllm::PagedKVCache cache(nano_vllm::KVCacheConfig{
        .num_blocks = 1, .block_size = 1, .num_layers = std::size_t(layers),
        .num_heads = std::size_t(heads), .head_dim = std::size_t(head_dim)});
    std::vector<nano_vllm::SequenceState> seqs;
    seqs.emplace_back(nano_vllm::SeqId(1), std::vector<std::size_t>{std::size_t(token)}, 1);
    seqs.back().block_table.push_back(BlockId(0));
    g_plan.active = false;
    g_ops = OperandCapture{};
    g_ops.active = true;
    (void)model.forward_batch(seqs, cache, pool);
    g_ops.active = false;
    return int64_t(g_ops.dims.size());
}

int ref_operand_dims(int64_t i, int64_t* batch, int64_t* k, int64_t* n) {
    if (i < 0 || std::size_t(i) >= g_ops.dims.size()) return -1;
    *batch = int64_t(g_ops.dims[std::size_t(i)][0]);
    *k = int64_t(g_ops.dims[std::size_t(i)][1]);
    *n = int64_t(g_ops.dims[std::size_t(i)][2]);
    return 0;
}

int ref_operand_copy(int64_t i, float* a, float* w) {
    if (i < 0 || std::size_t(i) >= g_ops.dims.size()) return -1;
    std::copy(g_ops.a[std::size_t(i)].begin(), g_ops.a[std::size_t(i)].end(), a);
    std::copy(g_ops.w[std::size_t(i)].begin(), g_ops.w[std::size_t(i)].end(), w);
    return 0;
}

}  // extern "C"
