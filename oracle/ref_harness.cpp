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
// reference's own loop computes for the given Q/K/V and KV history.

#include "nano_vllm/kv_cache.hpp"
#include "nano_vllm/model.hpp"
#include "nano_vllm/scheduler.hpp"
#include "nano_vllm/thread_pool.hpp"

#include <algorithm>
#include <cstdint>
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
    std::span<const float> /*w*/,
    std::span<float> c,
    std::size_t batch_size,
    std::size_t /*k_dim*/,
    std::size_t n_dim,
    ThreadPool& /*pool*/) {
    const std::size_t count = batch_size * n_dim;
    if (!g_plan.active) {
        std::fill_n(c.data(), count, 0.0f);
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

}  // extern "C"
