// extern "C" wrappers of the host library (declared in include/nvllm_host.h).
#include <algorithm>
#include <cstring>
#include <memory>
#include <new>
#include <vector>

#include "../../include/nvllm_host.h"
#include "block_allocator.hpp"
#include "engine.hpp"
#include "metadata.hpp"
#include "generator.hpp"
#include "model.hpp"
#include "router.hpp"
#include "scheduler.hpp"
#include "server.hpp"

struct nvllm_block_allocator {
    nvllm::BlockAllocator impl;
    explicit nvllm_block_allocator(std::size_t n) : impl(n) {}
};

struct nvllm_engine {
    std::unique_ptr<nvllm::AttentionEngine> impl;
};

struct nvllm_model {
    std::unique_ptr<nvllm::DeviceModel> impl;
};

struct nvllm_scheduler {
    nvllm::Scheduler impl;
};

struct nvllm_generator {
    std::unique_ptr<nvllm::Generator> impl;
};

struct nvllm_router {
    std::unique_ptr<nvllm::Router> impl;
};

struct nvllm_server {
    std::unique_ptr<nvllm::HttpServer> impl;
};

namespace {

int kv_status(nvllm::KVError e) {
    return e == nvllm::KVError::OutOfPhysicalBlocks ? NVLLM_HOST_OUT_OF_BLOCKS
                                                    : NVLLM_HOST_INVALID_BLOCK;
}

int engine_status(const nvllm::EngineError& e) {
    switch (e.kind) {
        case nvllm::EngineError::Kind::Cuda: return NVLLM_ERR_CUDA;
        case nvllm::EngineError::Kind::Blas: return NVLLM_ERR_CUDA;
        case nvllm::EngineError::Kind::Unsupported: return NVLLM_ERR_UNSUPPORTED;
        case nvllm::EngineError::Kind::Pack: return NVLLM_HOST_PACK_ERROR;
        case nvllm::EngineError::Kind::Kernel: return e.code;
        default: return NVLLM_ERR_INVALID;
    }
}

int allocate(nvllm::BlockAllocator& a, int64_t count, int64_t* out) {
    if (count < 0 || (count > 0 && out == nullptr)) return NVLLM_ERR_INVALID;
    auto r = a.allocate_blocks(static_cast<std::size_t>(count));
    if (!r) return kv_status(r.error());
    for (std::size_t i = 0; i < r->size(); ++i) out[i] = static_cast<int64_t>((*r)[i]);
    return NVLLM_OK;
}

int release(nvllm::BlockAllocator& a, const int64_t* ids, int64_t n) {
    if (n < 0 || (n > 0 && ids == nullptr)) return NVLLM_ERR_INVALID;
    std::vector<nvllm::BlockId> v;
    v.reserve(static_cast<std::size_t>(n));
    for (int64_t i = 0; i < n; ++i) {
        if (ids[i] < 0) return NVLLM_HOST_INVALID_BLOCK;
        v.push_back(static_cast<nvllm::BlockId>(ids[i]));
    }
    auto r = a.free_blocks(v);
    return r ? NVLLM_OK : kv_status(r.error());
}

// Builds the sequence views (tables copied into `storage`).
bool make_views(int32_t num_seqs, const int32_t* num_computed, const int32_t* total_len,
                const int64_t* block_ids, const int32_t* table_lens,
                std::vector<nvllm::BlockId>& storage, std::vector<nvllm::SequenceView>& views) {
    if (num_seqs < 0) return false;
    if (num_seqs == 0) return true;
    if (!num_computed || !total_len || !table_lens) return false;
    std::size_t total = 0;
    for (int32_t s = 0; s < num_seqs; ++s) {
        if (table_lens[s] < 0) return false;
        total += static_cast<std::size_t>(table_lens[s]);
    }
    if (total > 0 && block_ids == nullptr) return false;
    storage.resize(total);
    for (std::size_t i = 0; i < total; ++i) {
        if (block_ids[i] < 0) return false;
        storage[i] = static_cast<nvllm::BlockId>(block_ids[i]);
    }
    views.resize(static_cast<std::size_t>(num_seqs));
    std::size_t off = 0;
    for (int32_t s = 0; s < num_seqs; ++s) {
        const std::size_t len = static_cast<std::size_t>(table_lens[s]);
        views[s] = nvllm::SequenceView{num_computed[s], total_len[s],
                                       std::span<const nvllm::BlockId>(storage.data() + off, len)};
        off += len;
    }
    return true;
}

bool scheduler_config(const nvllm_scheduler_config* c, nvllm::SchedulerConfig& out) {
    if (c == nullptr || c->max_batch_size < 0 || c->max_tokens_per_step < 0 ||
        c->watermark_blocks < 0) {
        return false;
    }
    out.max_batch_size = std::size_t(c->max_batch_size);
    out.max_tokens_per_step = std::size_t(c->max_tokens_per_step);
    out.watermark_blocks = std::size_t(c->watermark_blocks);
    if (c->eos_token_id >= 0) out.eos_token_id = c->eos_token_id;
    return true;
}

void fill_summary(const nvllm::StepSummary& s, nvllm_step_summary* out) {
    if (out == nullptr) return;
    out->admitted = int64_t(s.admitted);
    out->preempted = int64_t(s.preempted);
    out->retired = int64_t(s.retired);
    out->batch_size = int64_t(s.batch_size);
    out->scheduled_tokens = int64_t(s.scheduled_tokens);
}

bool make_prompt(const int64_t* prompt, int64_t len, std::vector<int64_t>& out) {
    if (len < 0 || (len > 0 && prompt == nullptr)) return false;
    out.assign(prompt, prompt + len);
    for (const int64_t t : out) {
        if (t < 0) return false;
    }
    return true;
}

void fill_offsets(const nvllm::MetadataLayout& m, nvllm_metadata_offsets* out) {
    out->cu_seqlens_q = int64_t(m.cu_off);
    out->context_lens = int64_t(m.ctx_off);
    out->last_token_idx = int64_t(m.last_off);
    out->slot_mapping = int64_t(m.slot_off);
    out->block_tables = int64_t(m.table_off);
    out->bytes = int64_t(m.bytes);
    out->num_seqs = m.num_seqs;
    out->num_tokens = m.num_tokens;
    out->max_blocks = m.max_blocks;
    out->max_query_len = m.max_query_len;
    out->max_context_len = m.max_context_len;
}

}  // namespace

extern "C" {

nvllm_block_allocator* nvllm_block_allocator_create(int64_t num_blocks) {
    if (num_blocks < 0) return nullptr;
    return new (std::nothrow) nvllm_block_allocator(static_cast<std::size_t>(num_blocks));
}

void nvllm_block_allocator_destroy(nvllm_block_allocator* a) { delete a; }

int nvllm_block_allocator_allocate_block(nvllm_block_allocator* a, int64_t* out_id) {
    if (a == nullptr || out_id == nullptr) return NVLLM_ERR_INVALID;
    auto r = a->impl.allocate_block();
    if (!r) return kv_status(r.error());
    *out_id = static_cast<int64_t>(*r);
    return NVLLM_OK;
}

int nvllm_block_allocator_allocate_blocks(nvllm_block_allocator* a, int64_t count,
                                          int64_t* out_ids) {
    return a ? allocate(a->impl, count, out_ids) : NVLLM_ERR_INVALID;
}

int nvllm_block_allocator_free_blocks(nvllm_block_allocator* a, const int64_t* ids, int64_t n) {
    return a ? release(a->impl, ids, n) : NVLLM_ERR_INVALID;
}

int64_t nvllm_block_allocator_num_free(const nvllm_block_allocator* a) {
    return a ? static_cast<int64_t>(a->impl.num_free_blocks()) : -1;
}

size_t nvllm_metadata_bytes(int32_t num_seqs, int32_t num_tokens, int32_t max_blocks) {
    if (num_seqs < 0 || num_tokens < 0 || max_blocks < 0) return 0;
    return nvllm::metadata_layout(num_seqs, num_tokens, max_blocks).bytes;
}

int nvllm_pack_metadata(int32_t num_seqs, const int32_t* num_computed, const int32_t* total_len,
                        const int64_t* block_ids, const int32_t* table_lens, int32_t block_size,
                        int32_t max_blocks, void* buf, size_t buf_bytes,
                        nvllm_metadata_offsets* out) {
    std::vector<nvllm::BlockId> storage;
    std::vector<nvllm::SequenceView> views;
    if (!make_views(num_seqs, num_computed, total_len, block_ids, table_lens, storage, views) ||
        buf == nullptr || out == nullptr) {
        return NVLLM_ERR_INVALID;
    }
    auto r = nvllm::pack_metadata(
        views, block_size, max_blocks,
        std::span<std::byte>(static_cast<std::byte*>(buf), buf_bytes));
    if (!r) return NVLLM_HOST_PACK_ERROR;
    fill_offsets(*r, out);
    return NVLLM_OK;
}

int nvllm_pack_metadata_padded(int32_t num_seqs, const int32_t* num_computed,
                               const int32_t* total_len, const int64_t* block_ids,
                               const int32_t* table_lens, int32_t block_size, int32_t max_blocks,
                               int32_t pad_seqs, int32_t pad_tokens, void* buf,
                               size_t buf_bytes, nvllm_metadata_offsets* out) {
    std::vector<nvllm::BlockId> storage;
    std::vector<nvllm::SequenceView> views;
    if (!make_views(num_seqs, num_computed, total_len, block_ids, table_lens, storage, views) ||
        buf == nullptr || out == nullptr || pad_seqs < 1 || pad_tokens < 1) {
        return NVLLM_ERR_INVALID;
    }
    auto r = nvllm::pack_metadata(views, block_size, max_blocks,
                                  std::span<std::byte>(static_cast<std::byte*>(buf), buf_bytes),
                                  pad_seqs, pad_tokens);
    if (!r) return NVLLM_HOST_PACK_ERROR;
    fill_offsets(*r, out);
    return NVLLM_OK;
}

int nvllm_engine_create(const nvllm_engine_config* cfg, nvllm_engine** out) {
    if (cfg == nullptr || out == nullptr) return NVLLM_ERR_INVALID;
    *out = nullptr;
    nvllm::EngineConfig c;
    c.layout = cfg->layout;
    c.max_seqs = cfg->max_seqs;
    c.max_tokens = cfg->max_tokens;
    c.max_blocks_per_seq = cfg->max_blocks_per_seq;
    c.device = cfg->device;
    auto r = nvllm::AttentionEngine::create(c);
    if (!r) return engine_status(r.error());
    *out = new (std::nothrow) nvllm_engine{std::move(*r)};
    return *out ? NVLLM_OK : NVLLM_ERR_INVALID;
}

void nvllm_engine_destroy(nvllm_engine* e) { delete e; }

int nvllm_engine_allocate_blocks(nvllm_engine* e, int64_t count, int64_t* out_ids) {
    return e ? allocate(e->impl->allocator(), count, out_ids) : NVLLM_ERR_INVALID;
}

int nvllm_engine_free_blocks(nvllm_engine* e, const int64_t* ids, int64_t n) {
    return e ? release(e->impl->allocator(), ids, n) : NVLLM_ERR_INVALID;
}

int64_t nvllm_engine_num_free_blocks(const nvllm_engine* e) {
    return e ? static_cast<int64_t>(e->impl->allocator().num_free_blocks()) : -1;
}

int nvllm_engine_begin_step(nvllm_engine* e, int32_t num_seqs, const int32_t* num_computed,
                            const int32_t* total_len, const int64_t* block_ids,
                            const int32_t* table_lens) {
    if (e == nullptr) return NVLLM_ERR_INVALID;
    std::vector<nvllm::BlockId> storage;
    std::vector<nvllm::SequenceView> views;
    if (!make_views(num_seqs, num_computed, total_len, block_ids, table_lens, storage, views)) {
        return NVLLM_ERR_INVALID;
    }
    auto r = e->impl->begin_step(views);
    return r ? NVLLM_OK : engine_status(r.error());
}

int nvllm_engine_begin_step_padded(nvllm_engine* e, int32_t num_seqs, const int32_t* num_computed,
                                   const int32_t* total_len, const int64_t* block_ids,
                                   const int32_t* table_lens, int32_t pad_seqs,
                                   int32_t pad_tokens) {
    if (e == nullptr || pad_seqs < 1 || pad_tokens < 1) return NVLLM_ERR_INVALID;
    std::vector<nvllm::BlockId> storage;
    std::vector<nvllm::SequenceView> views;
    if (!make_views(num_seqs, num_computed, total_len, block_ids, table_lens, storage, views)) {
        return NVLLM_ERR_INVALID;
    }
    auto r = e->impl->begin_step(views, pad_seqs, pad_tokens);
    return r ? NVLLM_OK : engine_status(r.error());
}

int nvllm_engine_attention(nvllm_engine* e, int32_t layer, const float* q, const float* k,
                           const float* v, float* out, int32_t precision) {
    if (e == nullptr) return NVLLM_ERR_INVALID;
    if (e->impl->step().num_tokens > 0 && (!q || !k || !v || !out)) return NVLLM_ERR_INVALID;
    auto r = e->impl->attention(layer, q, k, v, out, precision);
    return r ? NVLLM_OK : engine_status(r.error());
}

int nvllm_engine_host_buffers(nvllm_engine* e, float** q, float** k, float** v, float** out) {
    if (e == nullptr) return NVLLM_ERR_INVALID;
    if (q) *q = e->impl->host_query();
    if (k) *k = e->impl->host_key();
    if (v) *v = e->impl->host_value();
    if (out) *out = e->impl->host_output();
    return NVLLM_OK;
}

int nvllm_engine_slot_buffers(nvllm_engine* e, int32_t slot, float** q, float** k, float** v,
                              float** out) {
    if (e == nullptr) return NVLLM_ERR_INVALID;
    auto r = e->impl->slot_buffers(slot, q, k, v, out);
    return r ? NVLLM_OK : engine_status(r.error());
}

int nvllm_engine_attention_submit(nvllm_engine* e, int32_t layer, int32_t slot,
                                  int32_t precision) {
    if (e == nullptr) return NVLLM_ERR_INVALID;
    auto r = e->impl->submit(layer, slot, precision);
    return r ? NVLLM_OK : engine_status(r.error());
}

int nvllm_engine_attention_collect(nvllm_engine* e, int32_t slot) {
    if (e == nullptr) return NVLLM_ERR_INVALID;
    auto r = e->impl->collect(slot);
    return r ? NVLLM_OK : engine_status(r.error());
}

int nvllm_engine_arenas(nvllm_engine* e, float** k_arena, float** v_arena) {
    if (e == nullptr) return NVLLM_ERR_INVALID;
    if (k_arena) *k_arena = e->impl->k_arena();
    if (v_arena) *v_arena = e->impl->v_arena();
    return NVLLM_OK;
}

void* nvllm_engine_stream(nvllm_engine* e) { return e ? e->impl->stream() : nullptr; }

int32_t nvllm_engine_step_tokens(const nvllm_engine* e) {
    return e ? e->impl->step().num_tokens : -1;
}

int nvllm_model_create(const nvllm_model_config* cfg, nvllm_engine* engine, nvllm_model** out) {
    if (cfg == nullptr || engine == nullptr || out == nullptr) return NVLLM_ERR_INVALID;
    nvllm::ModelConfig mc{.vocab = cfg->vocab, .hidden = cfg->hidden, .layers = cfg->layers,
                          .heads = cfg->heads, .head_dim = cfg->head_dim, .ffn = cfg->ffn,
                          .emb_scale = cfg->emb_scale, .ffn_scale = cfg->ffn_scale,
                          .gemm_math = cfg->gemm_math,
                          .graph_max_tokens = cfg->graph_max_tokens,
                          .head_ranks = cfg->head_ranks > 0 ? cfg->head_ranks : 1};
    auto r = nvllm::DeviceModel::create(mc, *engine->impl);
    if (!r) return engine_status(r.error());
    auto* m = new (std::nothrow) nvllm_model{std::move(*r)};
    if (m == nullptr) return NVLLM_ERR_INVALID;
    *out = m;
    return NVLLM_OK;
}

void nvllm_model_destroy(nvllm_model* m) { delete m; }

int nvllm_model_set_head_group(nvllm_model* m, const nvllm_model_head_group* g) {
    if (m == nullptr || g == nullptr || g->world < 1 || g->world > NVLLM_MAX_RANKS) {
        return NVLLM_ERR_INVALID;
    }
    nvllm::HeadGroup hg;
    hg.rank = g->rank;
    hg.world = g->world;
    for (int r = 0; r < g->world; ++r) {
        hg.outs[0][r] = g->outs[0][r];
        hg.outs[1][r] = g->outs[1][r];
        hg.flags[r] = g->flags[r];
    }
    const auto r = m->impl->set_head_group(hg);
    return r ? NVLLM_OK : engine_status(r.error());
}

int nvllm_model_forward(nvllm_model* m, const int64_t* token_ids, int64_t num_tokens,
                        const int64_t* prev_tokens, int64_t num_seqs, int64_t* sampled,
                        int32_t precision, float* margins, int32_t* top_idx, float* top_val,
                        int32_t top_k) {
    if (m == nullptr || num_tokens < 0 || num_seqs < 0 ||
        (num_tokens > 0 && token_ids == nullptr) ||
        (num_seqs > 0 && (prev_tokens == nullptr || sampled == nullptr))) {
        return NVLLM_ERR_INVALID;
    }
    auto r = m->impl->forward(
        std::span<const int64_t>(token_ids, std::size_t(num_tokens)),
        std::span<const int64_t>(prev_tokens, std::size_t(num_seqs)), sampled, precision, margins,
        top_idx, top_val, top_k);
    return r ? NVLLM_OK : engine_status(r.error());
}

int nvllm_model_weights(const nvllm_model* m, const float** weights, int64_t* count) {
    if (m == nullptr || weights == nullptr || count == nullptr) return NVLLM_ERR_INVALID;
    *weights = m->impl->weights();
    *count = int64_t(m->impl->weight_floats());
    return NVLLM_OK;
}

nvllm_scheduler* nvllm_scheduler_create(const nvllm_scheduler_config* cfg, int32_t block_size) {
    nvllm::SchedulerConfig sc;
    if (!scheduler_config(cfg, sc) || block_size <= 0) return nullptr;
    return new (std::nothrow) nvllm_scheduler{nvllm::Scheduler(sc, std::size_t(block_size))};
}

void nvllm_scheduler_destroy(nvllm_scheduler* s) { delete s; }

int nvllm_scheduler_add_request(nvllm_scheduler* s, uint64_t seq_id, const int64_t* prompt,
                                int64_t prompt_len, int64_t max_new_tokens) {
    std::vector<int64_t> p;
    if (s == nullptr || !make_prompt(prompt, prompt_len, p)) return NVLLM_ERR_INVALID;
    s->impl.add_request(
        nvllm::Sequence(seq_id, std::move(p), std::size_t(std::max<int64_t>(max_new_tokens, 1))));
    return NVLLM_OK;
}

int nvllm_scheduler_schedule_step(nvllm_scheduler* s, nvllm_block_allocator* blocks,
                                  nvllm_step_summary* out) {
    if (s == nullptr || blocks == nullptr) return NVLLM_ERR_INVALID;
    fill_summary(s->impl.schedule_step(blocks->impl), out);
    return NVLLM_OK;
}

int64_t nvllm_scheduler_batch_record(const nvllm_scheduler* s, int64_t step, int64_t* out,
                                     int64_t cap) {
    if (s == nullptr) return -1;
    std::vector<int64_t> rec;
    nvllm::append_batch_record(s->impl, step, rec);
    if (out != nullptr && int64_t(rec.size()) <= cap) std::memcpy(out, rec.data(), rec.size() * 8);
    return int64_t(rec.size());
}

int nvllm_scheduler_process_outputs(nvllm_scheduler* s, nvllm_block_allocator* blocks,
                                    const int64_t* sampled, int64_t n, int64_t* retired) {
    if (s == nullptr || blocks == nullptr || n < 0 || (n > 0 && sampled == nullptr) ||
        std::size_t(n) != s->impl.running().size()) {
        return NVLLM_ERR_INVALID;
    }
    const std::size_t r = s->impl.process_step_outputs(
        std::span<const int64_t>(sampled, std::size_t(n)), blocks->impl);
    if (retired != nullptr) *retired = int64_t(r);
    return NVLLM_OK;
}

int nvllm_scheduler_counts(const nvllm_scheduler* s, int64_t* running, int64_t* waiting,
                           int64_t* preemptions, int64_t* completed) {
    if (s == nullptr) return NVLLM_ERR_INVALID;
    if (running) *running = int64_t(s->impl.running().size());
    if (waiting) *waiting = int64_t(s->impl.waiting().size());
    if (preemptions) *preemptions = int64_t(s->impl.total_preemptions());
    if (completed) *completed = int64_t(s->impl.total_completed());
    return NVLLM_OK;
}

int nvllm_generator_create(nvllm_engine* engine, nvllm_model* model,
                           const nvllm_scheduler_config* cfg, int32_t precision,
                           nvllm_generator** out) {
    nvllm::SchedulerConfig sc;
    if (engine == nullptr || model == nullptr || out == nullptr || !scheduler_config(cfg, sc)) {
        return NVLLM_ERR_INVALID;
    }
    auto g = std::make_unique<nvllm::Generator>(*engine->impl, *model->impl, sc, precision);
    auto* h = new (std::nothrow) nvllm_generator{std::move(g)};
    if (h == nullptr) return NVLLM_ERR_INVALID;
    *out = h;
    return NVLLM_OK;
}

void nvllm_generator_destroy(nvllm_generator* g) { delete g; }

int nvllm_generator_add_request(nvllm_generator* g, uint64_t seq_id, const int64_t* prompt,
                                int64_t prompt_len, int64_t max_new_tokens) {
    std::vector<int64_t> p;
    if (g == nullptr || !make_prompt(prompt, prompt_len, p)) return NVLLM_ERR_INVALID;
    g->impl->add_request(seq_id, std::move(p),
                         std::size_t(std::max<int64_t>(max_new_tokens, 1)));
    return NVLLM_OK;
}

int nvllm_generator_step(nvllm_generator* g, nvllm_step_summary* out) {
    if (g == nullptr) return NVLLM_ERR_INVALID;
    auto r = g->impl->step();
    if (!r) return engine_status(r.error());
    fill_summary(*r, out);
    return NVLLM_OK;
}

int nvllm_generator_run(nvllm_generator* g, int64_t max_steps, int64_t* steps_done) {
    if (g == nullptr) return NVLLM_ERR_INVALID;
    auto r = g->impl->run(max_steps);
    if (!r) return engine_status(r.error());
    if (steps_done != nullptr) *steps_done = *r;
    return NVLLM_OK;
}

int nvllm_generator_has_pending_work(const nvllm_generator* g) {
    return g != nullptr && g->impl->has_pending_work() ? 1 : 0;
}

int64_t nvllm_generator_output(const nvllm_generator* g, uint64_t seq_id, int64_t* tokens,
                               int64_t cap) {
    if (g == nullptr) return -1;
    const auto* t = g->impl->output(seq_id);
    if (t == nullptr) return -1;
    if (tokens != nullptr && int64_t(t->size()) <= cap) {
        std::memcpy(tokens, t->data(), t->size() * sizeof(int64_t));
    }
    return int64_t(t->size());
}

int nvllm_generator_trace(nvllm_generator* g, const char* path) {
    if (g == nullptr) return NVLLM_ERR_INVALID;
    return g->impl->set_trace(path ? std::string(path) : std::string()) ? NVLLM_OK
                                                                         : NVLLM_ERR_INVALID;
}

namespace {
nvllm_metrics c_metrics(const nvllm::Metrics& m) {
    return nvllm_metrics{m.uptime_secs, m.total_requests_received, m.total_requests_completed,
                         m.total_tokens_generated, m.throughput_tokens_per_sec,
                         m.active_batch_size, m.waiting_queue_depth, m.kv_cache_used_blocks,
                         m.kv_cache_total_blocks, m.kv_cache_utilization_pct, m.avg_ttft_ms,
                         m.avg_iteration_latency_ms, m.total_preemptions, m.total_iterations,
                         m.total_tokens_computed, m.h2d_bytes, m.d2h_bytes, m.kernel_launches};
}
}  // namespace

int nvllm_generator_metrics(const nvllm_generator* g, nvllm_metrics* out) {
    if (g == nullptr || out == nullptr) return NVLLM_ERR_INVALID;
    *out = c_metrics(g->impl->metrics());
    return NVLLM_OK;
}

int nvllm_router_create(nvllm_generator* const* gens, int32_t n, nvllm_router** out) {
    if (gens == nullptr || n <= 0 || out == nullptr) return NVLLM_ERR_INVALID;
    std::vector<nvllm::Generator*> g;
    for (int32_t i = 0; i < n; ++i) {
        if (gens[i] == nullptr) return NVLLM_ERR_INVALID;
        for (nvllm::Generator* other : g) {
            if (other == gens[i]->impl.get()) return NVLLM_ERR_INVALID;  // one lane each
        }
        g.push_back(gens[i]->impl.get());
    }
    auto* h = new (std::nothrow) nvllm_router{std::make_unique<nvllm::Router>(g)};
    if (h == nullptr) return NVLLM_ERR_INVALID;
    *out = h;
    return NVLLM_OK;
}

void nvllm_router_destroy(nvllm_router* r) { delete r; }

int nvllm_router_add_request(nvllm_router* r, uint64_t seq_id, const int64_t* prompt,
                             int64_t prompt_len, int64_t max_new_tokens, int32_t* gpu) {
    std::vector<int64_t> p;
    if (r == nullptr || !make_prompt(prompt, prompt_len, p)) return NVLLM_ERR_INVALID;
    auto res = r->impl->add_request(seq_id, std::move(p),
                                    std::size_t(std::max<int64_t>(max_new_tokens, 1)));
    if (!res) return engine_status(res.error());
    if (gpu != nullptr) *gpu = *res;
    return NVLLM_OK;
}

int nvllm_router_add_requests(nvllm_router* r, int64_t n, const uint64_t* seq_ids,
                              const int64_t* tokens, const int64_t* offsets,
                              const int64_t* max_new_tokens, int32_t* gpus) {
    if (r == nullptr || n < 0 || (n > 0 && (seq_ids == nullptr || tokens == nullptr ||
                                            offsets == nullptr || max_new_tokens == nullptr))) {
        return NVLLM_ERR_INVALID;
    }
    if (n == 0) return NVLLM_OK;
    std::vector<nvllm::SeqId> ids(seq_ids, seq_ids + n);
    std::vector<std::vector<int64_t>> prompts(static_cast<std::size_t>(n));
    std::vector<std::size_t> mx(static_cast<std::size_t>(n));
    for (int64_t k = 0; k < n; ++k) {
        if (offsets[k] < 0 || offsets[k + 1] < offsets[k]) return NVLLM_ERR_INVALID;
        if (!make_prompt(tokens + offsets[k], offsets[k + 1] - offsets[k], prompts[k])) {
            return NVLLM_ERR_INVALID;
        }
        mx[k] = std::size_t(std::max<int64_t>(max_new_tokens[k], 1));
    }
    auto res = r->impl->add_requests(ids, prompts, mx,
                                     gpus ? std::span<int32_t>(gpus, std::size_t(n))
                                          : std::span<int32_t>());
    return res ? NVLLM_OK : engine_status(res.error());
}

int nvllm_router_wait_idle(nvllm_router* r) {
    if (r == nullptr) return NVLLM_ERR_INVALID;
    auto res = r->impl->wait_idle();
    return res ? NVLLM_OK : engine_status(res.error());
}

int64_t nvllm_router_output(nvllm_router* r, uint64_t seq_id, int64_t* tokens, int64_t cap) {
    if (r == nullptr) return -1;
    const auto t = r->impl->output(seq_id);
    if (!t) return -1;
    if (tokens != nullptr && int64_t(t->size()) <= cap) {
        std::memcpy(tokens, t->data(), t->size() * sizeof(int64_t));
    }
    return int64_t(t->size());
}

int nvllm_router_metrics(nvllm_router* r, int32_t gpu, nvllm_metrics* out) {
    if (r == nullptr || out == nullptr || gpu < 0 || gpu >= r->impl->num_gpus()) {
        return NVLLM_ERR_INVALID;
    }
    *out = c_metrics(r->impl->metrics(gpu));
    return NVLLM_OK;
}

int64_t nvllm_router_placed(const nvllm_router* r, int32_t gpu) {
    if (r == nullptr || gpu < 0 || gpu >= r->impl->num_gpus()) return -1;
    return int64_t(r->impl->placed(gpu));
}

int64_t nvllm_metrics_to_json(const nvllm_metrics* m, char* buf, int64_t cap) {
    if (m == nullptr) return -1;
    nvllm::Metrics x;
    x.uptime_secs = m->uptime_secs;
    x.total_requests_received = m->total_requests_received;
    x.total_requests_completed = m->total_requests_completed;
    x.total_tokens_generated = m->total_tokens_generated;
    x.throughput_tokens_per_sec = m->throughput_tokens_per_sec;
    x.active_batch_size = m->active_batch_size;
    x.waiting_queue_depth = m->waiting_queue_depth;
    x.kv_cache_used_blocks = m->kv_cache_used_blocks;
    x.kv_cache_total_blocks = m->kv_cache_total_blocks;
    x.kv_cache_utilization_pct = m->kv_cache_utilization_pct;
    x.avg_ttft_ms = m->avg_ttft_ms;
    x.avg_iteration_latency_ms = m->avg_iteration_latency_ms;
    x.total_preemptions = m->total_preemptions;
    const std::string js = x.to_json();
    if (buf != nullptr && int64_t(js.size()) < cap) std::memcpy(buf, js.c_str(), js.size() + 1);
    return int64_t(js.size());
}

int nvllm_ipc_alloc(size_t bytes, void** dev_ptr, void* handle) {
    if (dev_ptr == nullptr || handle == nullptr || bytes == 0) return NVLLM_ERR_INVALID;
    static_assert(sizeof(cudaIpcMemHandle_t) == NVLLM_IPC_HANDLE_BYTES, "IPC handle size");
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return NVLLM_ERR_CUDA;
    if (cudaMemset(p, 0, bytes) != cudaSuccess ||
        cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p) != cudaSuccess) {
        cudaFree(p);
        return NVLLM_ERR_CUDA;
    }
    *dev_ptr = p;
    return NVLLM_OK;
}

int nvllm_ipc_open(const void* handle, void** dev_ptr) {
    if (dev_ptr == nullptr || handle == nullptr) return NVLLM_ERR_INVALID;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    return cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
               ? NVLLM_OK
               : NVLLM_ERR_CUDA;
}

int nvllm_ipc_close(void* dev_ptr) {
    return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? NVLLM_OK : NVLLM_ERR_CUDA;
}

int nvllm_ipc_free(void* dev_ptr) {
    return cudaFree(dev_ptr) == cudaSuccess ? NVLLM_OK : NVLLM_ERR_CUDA;
}

}  // extern "C"

int nvllm_server_start(nvllm_router* r, int64_t vocab_size, const char* bind_address,
                       int32_t port, nvllm_server** out) {
    if (r == nullptr || out == nullptr || vocab_size < 2 || port < 0 || port > 65535) {
        return NVLLM_ERR_INVALID;
    }
    nvllm::ServerConfig cfg;
    if (bind_address != nullptr && bind_address[0] != '\0') cfg.bind_address = bind_address;
    cfg.port = uint16_t(port);
    cfg.vocab_size = std::size_t(vocab_size);
    auto s = nvllm::HttpServer::start(*r->impl, cfg);
    if (!s) return NVLLM_ERR_INVALID;
    auto* h = new (std::nothrow) nvllm_server{std::move(*s)};
    if (h == nullptr) return NVLLM_ERR_INVALID;
    *out = h;
    return NVLLM_OK;
}

int32_t nvllm_server_port(const nvllm_server* s) { return s ? int32_t(s->impl->port()) : -1; }

void nvllm_server_stop(nvllm_server* s) { delete s; }

int64_t nvllm_tokenize_prompt(const char* text, int64_t vocab_size, int64_t* out, int64_t cap) {
    if (text == nullptr || vocab_size < 2) return -1;
    const auto t = nvllm::tokenize_prompt(text, std::size_t(vocab_size));
    if (out != nullptr && int64_t(t.size()) <= cap) {
        std::memcpy(out, t.data(), t.size() * sizeof(int64_t));
    }
    return int64_t(t.size());
}
