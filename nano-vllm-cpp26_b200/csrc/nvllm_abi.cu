// The extern "C" boundary of libnvllm.so (declared in include/nvllm.h):
// argument validation, workspace carve-up and kernel dispatch.
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/nvllm.h"
#include "common.cuh"
#include "kernels.cuh"

namespace nvllm {

namespace {

constexpr size_t kAlign = 256;
// SMs for a prefill beside the decode by default (0: one after the other)
constexpr int kDefaultPrefillSms = 0;

size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

bool head_dim_supported(int32_t hd) { return hd == 32 || hd == 64 || hd == 128 || hd == 256; }

int validate_layout(const nvllm_kv_layout* lay) {
    if (lay == nullptr) return NVLLM_ERR_INVALID;
    if (lay->num_blocks <= 0 || lay->num_layers <= 0 || lay->block_size <= 0 ||
        lay->num_heads <= 0 || lay->head_dim <= 0) {
        return NVLLM_ERR_INVALID;
    }
    if (!head_dim_supported(lay->head_dim)) return NVLLM_ERR_UNSUPPORTED;
    // slot ids are int32: num_blocks * block_size must fit
    if (lay->num_blocks > INT32_MAX / lay->block_size) return NVLLM_ERR_INVALID;
    return NVLLM_OK;
}

ArenaGeom make_geom(const nvllm_kv_layout* lay) {
    ArenaGeom g{};
    g.num_blocks = lay->num_blocks;
    g.row = int64_t(lay->num_heads) * lay->head_dim;
    g.layer_stride = int64_t(lay->block_size) * g.row;
    g.block_stride = int64_t(lay->num_layers) * g.layer_stride;
    g.num_layers = lay->num_layers;
    g.block_size = lay->block_size;
    g.num_heads = lay->num_heads;
    g.head_dim = lay->head_dim;
    return g;
}

}  // namespace

WorkspaceLayout workspace_layout(int32_t num_seqs, int32_t max_query_len, int32_t max_context_len,
                                 int32_t num_heads, int32_t head_dim) {
    WorkspaceLayout w{};
    w.split_tokens = decode_split_tokens(head_dim);
    w.prefill_tile = prefill_tile_rows(head_dim);
    w.max_splits = (max_context_len + w.split_tokens - 1) / w.split_tokens;
    if (w.max_splits < 1) w.max_splits = 1;
    const int64_t tiles = (int64_t(max_query_len) + w.prefill_tile - 1) / w.prefill_tile;
    const size_t S = size_t(num_seqs);
    size_t off = 0;
    w.counters_off = off;
    off = align_up(off + sizeof(PlanCounters));
    w.decode_items_off = off;
    off = align_up(off + S * w.max_splits * sizeof(WorkItem));
    w.prefill_items_off = off;
    off = align_up(off + S * size_t(tiles > 0 ? tiles : 1) * sizeof(WorkItem));
    w.part_acc_off = off;
    off = align_up(off + S * num_heads * w.max_splits * size_t(head_dim) * sizeof(float));
    w.part_ml_off = off;
    off = align_up(off + S * num_heads * w.max_splits * sizeof(float2));
    w.total = off;
    return w;
}

}  // namespace nvllm

using namespace nvllm;

extern "C" {

int nvllm_reshape_and_cache(const float* key, const float* value, float* k_arena,
                            float* v_arena, const int32_t* slot_mapping, int64_t num_tokens,
                            int32_t layer, const nvllm_kv_layout* layout, void* stream) {
    const int lv = validate_layout(layout);
    if (lv != NVLLM_OK) return lv;
    if (num_tokens < 0 || layer < 0 || layer >= layout->num_layers) return NVLLM_ERR_INVALID;
    if (num_tokens == 0) return NVLLM_OK;
    if (num_tokens > INT32_MAX) return NVLLM_ERR_INVALID;
    if (!key || !value || !k_arena || !v_arena || !slot_mapping) return NVLLM_ERR_INVALID;
    const bool vec4 = aligned16(key) && aligned16(value) && aligned16(k_arena) && aligned16(v_arena);
    const ArenaGeom g = make_geom(layout);
    const cudaError_t e = launch_reshape_and_cache(key, value, k_arena, v_arena, slot_mapping,
                                                   num_tokens, layer, g, vec4,
                                                   static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? NVLLM_OK : NVLLM_ERR_CUDA;
}

size_t nvllm_paged_attention_workspace_size(int32_t num_seqs, int32_t max_query_len,
                                            int32_t max_context_len,
                                            const nvllm_kv_layout* layout) {
    if (validate_layout(layout) != NVLLM_OK || num_seqs < 0 || max_query_len < 0 ||
        max_context_len < 0) {
        return 0;
    }
    return workspace_layout(num_seqs, max_query_len, max_context_len, layout->num_heads,
                            layout->head_dim)
        .total;
}

}  // extern "C"

namespace {

// Validates the arguments shared by the attention entry points and fills p
// (everything except the output routing).
int prepare_attention(AttnParams& p, const float* query, const float* k_arena,
                      const float* v_arena, const int32_t* block_tables,
                      int32_t max_blocks_per_seq, const int32_t* cu_seqlens_q,
                      const int32_t* context_lens, int32_t num_seqs, int32_t max_query_len,
                      int32_t max_context_len, int32_t layer, float scale, int32_t precision,
                      void* workspace, size_t workspace_bytes, const nvllm_kv_layout* layout) {
    if (precision != NVLLM_PRECISION_FP32 && precision != NVLLM_PRECISION_TF32) {
        return NVLLM_ERR_INVALID;
    }
    if (max_query_len < 1 || max_context_len < 1 || max_query_len > max_context_len ||
        max_blocks_per_seq < 1 ||
        int64_t(max_context_len) > int64_t(max_blocks_per_seq) * layout->block_size) {
        return NVLLM_ERR_INVALID;
    }
    if (!query || !k_arena || !v_arena || !block_tables || !cu_seqlens_q || !context_lens) {
        return NVLLM_ERR_INVALID;
    }
    if (!aligned16(query) || !aligned16(k_arena) || !aligned16(v_arena)) return NVLLM_ERR_INVALID;
    if (!(scale > 0.0f) || scale != scale) return NVLLM_ERR_INVALID;

    const WorkspaceLayout w = workspace_layout(num_seqs, max_query_len, max_context_len,
                                               layout->num_heads, layout->head_dim);
    if (workspace == nullptr || workspace_bytes < w.total ||
        (reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) != 0) {
        return NVLLM_ERR_WORKSPACE;
    }
    auto* ws = static_cast<unsigned char*>(workspace);
    p = AttnParams{};
    p.q = query;
    p.k_arena = k_arena;
    p.v_arena = v_arena;
    p.block_tables = block_tables;
    p.cu_seqlens_q = cu_seqlens_q;
    p.context_lens = context_lens;
    p.max_blocks = max_blocks_per_seq;
    p.num_seqs = num_seqs;
    p.max_query_len = max_query_len;
    p.max_context_len = max_context_len;
    p.layer = layer;
    p.qk_scale_log2 = scale * kLog2e;
    p.g = make_geom(layout);
    p.counters = reinterpret_cast<PlanCounters*>(ws + w.counters_off);
    p.decode_items = reinterpret_cast<WorkItem*>(ws + w.decode_items_off);
    p.prefill_items = reinterpret_cast<WorkItem*>(ws + w.prefill_items_off);
    p.part_acc = reinterpret_cast<float*>(ws + w.part_acc_off);
    p.part_ml = reinterpret_cast<float2*>(ws + w.part_ml_off);
    p.max_splits = w.max_splits;
    p.split_tokens = w.split_tokens;
    p.prefill_tile = w.prefill_tile;
    return NVLLM_OK;
}

// SMs given to the prefill when the decode runs beside it (NVLLM_PREFILL_SMS:
// a count of SMs; 0 = the prefill first on the whole GPU, then the decode).
int prefill_beside_sms() {
    static const int v = [] {
        const char* s = std::getenv("NVLLM_PREFILL_SMS");
        return s != nullptr ? std::max(0, std::atoi(s)) : kDefaultPrefillSms;
    }();
    return v;
}

// plan -> prefill (if any multi-row sequence) and decode + merge. With a
// prefill share configured, the prefill's persistent grid is bounded to that
// many SMs and the decode is launched as its programmatic dependent: the
// decode's CTAs start on the other SMs as soon as every prefill CTA is
// resident, and take the prefill's SMs as they retire, so that the HBM-bound
// decode and the tensor-bound prefill overlap. The merge and everything after
// the call are ordinary stream successors and wait for both.
cudaError_t launch_attention(AttnParams& p, int32_t precision, cudaStream_t st) {
    // TF32 prefill runs on the tensor cores where the kernel's geometry allows
    // (hd 128, block size 16); elsewhere the fp32 FFMA kernel serves it, whose
    // error is far inside the TF32 tolerance.
    const bool tc_prefill =
        precision == NVLLM_PRECISION_TF32 && p.max_query_len > 1 && prefill_tc_supported(p.g);
    if (tc_prefill) p.prefill_tile = prefill_tc_tile_rows();
    cudaError_t e = launch_plan(p, st);
    if (e != cudaSuccess) return e;
    const int beside = p.max_query_len > 1 ? prefill_beside_sms() : 0;
    if (p.max_query_len > 1) {
        e = tc_prefill ? launch_prefill_tc(p, st, beside) : launch_prefill_fp32(p, st, beside);
        if (e != cudaSuccess) return e;
    }
    return launch_decode(p, st, /*overlap_previous=*/beside > 0);
}

}  // namespace

extern "C" {

int nvllm_paged_attention(float* out, const float* query, const float* k_arena,
                          const float* v_arena, const int32_t* block_tables,
                          int32_t max_blocks_per_seq, const int32_t* cu_seqlens_q,
                          const int32_t* context_lens, int32_t num_seqs, int32_t max_query_len,
                          int32_t max_context_len, int32_t layer, float scale, int32_t precision,
                          void* workspace, size_t workspace_bytes, const nvllm_kv_layout* layout,
                          void* stream) {
    const int lv = validate_layout(layout);
    if (lv != NVLLM_OK) return lv;
    if (num_seqs < 0 || layer < 0 || layer >= layout->num_layers) return NVLLM_ERR_INVALID;
    if (num_seqs == 0) return NVLLM_OK;
    if (!out || !aligned16(out)) return NVLLM_ERR_INVALID;
    AttnParams p;
    const int rc = prepare_attention(p, query, k_arena, v_arena, block_tables, max_blocks_per_seq,
                                     cu_seqlens_q, context_lens, num_seqs, max_query_len,
                                     max_context_len, layer, scale, precision, workspace,
                                     workspace_bytes, layout);
    if (rc != NVLLM_OK) return rc;
    p.out = out;
    const cudaError_t e = launch_attention(p, precision, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? NVLLM_OK : NVLLM_ERR_CUDA;
}

int nvllm_paged_attention_head_split(const nvllm_head_split* hs, const float* query,
                                     const float* k_arena, const float* v_arena,
                                     const int32_t* block_tables, int32_t max_blocks_per_seq,
                                     const int32_t* cu_seqlens_q, const int32_t* context_lens,
                                     int32_t num_seqs, int32_t max_context_len, int32_t layer,
                                     float scale, void* workspace, size_t workspace_bytes,
                                     const nvllm_kv_layout* layout, void* stream) {
    const int lv = validate_layout(layout);
    if (lv != NVLLM_OK) return lv;
    if (hs == nullptr || hs->world < 1 || hs->world > NVLLM_MAX_RANKS || hs->rank < 0 ||
        hs->rank >= hs->world || hs->epoch == 0) {
        return NVLLM_ERR_INVALID;
    }
    for (int r = 0; r < hs->world; ++r) {
        if (!hs->outs[r] || !aligned16(hs->outs[r]) || !hs->flags[r] ||
            (reinterpret_cast<uintptr_t>(hs->flags[r]) & 3u) != 0) {
            return NVLLM_ERR_INVALID;
        }
    }
    if (num_seqs < 0 || layer < 0 || layer >= layout->num_layers) return NVLLM_ERR_INVALID;
    AttnParams p;
    if (num_seqs > 0) {
        const int rc = prepare_attention(p, query, k_arena, v_arena, block_tables,
                                         max_blocks_per_seq, cu_seqlens_q, context_lens, num_seqs,
                                         1, max_context_len, layer, scale, NVLLM_PRECISION_FP32,
                                         workspace, workspace_bytes, layout);
        if (rc != NVLLM_OK) return rc;
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t local_cols = int64_t(layout->num_heads) * layout->head_dim;
    p.num_outs = hs->world;
    for (int r = 0; r < hs->world; ++r) {
        p.outs[r] = hs->outs[r];
        p.flags[r] = hs->flags[r];
    }
    p.out_stride = local_cols * hs->world;
    p.out_col = local_cols * hs->rank;
    cudaError_t e = cudaSuccess;
    if (num_seqs > 0) {
        e = launch_attention(p, NVLLM_PRECISION_FP32, st);
    } else {
        // nothing to store, but the peers still count on this rank's signal
        e = launch_signal(p.flags, hs->world, st);
    }
    if (e == cudaSuccess) {
        e = launch_flag_wait(hs->flags[hs->rank], hs->epoch * uint32_t(hs->world), st);
    }
    return e == cudaSuccess ? NVLLM_OK : NVLLM_ERR_CUDA;
}

namespace {
std::atomic<uint32_t> g_last_status{0};  // the last nonzero word nvllm_get_last_error cleared
uint32_t g_last_timeout[4] = {0, 0, 0, 0};  // and the timeout record cleared with it
std::mutex g_last_timeout_mu;
}  // namespace

int nvllm_get_last_error(void* stream) {
    if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) {
        return NVLLM_ERR_CUDA;
    }
    uint32_t v = 0;
    if (cudaMemcpyFromSymbol(&v, g_status, sizeof(v)) != cudaSuccess) return NVLLM_ERR_CUDA;
    if (v == 0) return NVLLM_OK;
    g_last_status.store(v);
    if (v & kStatusTimeout) {
        uint32_t info[4] = {0, 0, 0, 0};
        const uint32_t zeros[4] = {0, 0, 0, 0};
        if (cudaMemcpyFromSymbol(info, g_timeout_info, sizeof(info)) != cudaSuccess ||
            cudaMemcpyToSymbol(g_timeout_info, zeros, sizeof(zeros)) != cudaSuccess) {
            return NVLLM_ERR_CUDA;
        }
        std::lock_guard<std::mutex> lk(g_last_timeout_mu);
        std::memcpy(g_last_timeout, info, sizeof(info));
    }
    const uint32_t zero = 0;
    if (cudaMemcpyToSymbol(g_status, &zero, sizeof(zero)) != cudaSuccess) return NVLLM_ERR_CUDA;
    if (v & kStatusTimeout) return NVLLM_ERR_TIMEOUT;
    if (v & kStatusBounds) return NVLLM_ERR_BOUNDS;
    return NVLLM_ERR_INVALID;
}

uint32_t nvllm_last_status_word(void) { return g_last_status.load(); }

int nvllm_last_timeout_info(uint32_t* info) {
    if (info == nullptr) return NVLLM_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_last_timeout_mu);
    std::memcpy(info, g_last_timeout, sizeof(g_last_timeout));
    return NVLLM_OK;
}

int nvllm_device_status_word(const uint32_t** word) {
    if (word == nullptr) return NVLLM_ERR_INVALID;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) return NVLLM_ERR_CUDA;
    *word = static_cast<const uint32_t*>(p);
    return NVLLM_OK;
}

const char* nvllm_status_string(int status) {
    switch (status) {
        case NVLLM_OK: return "ok";
        case NVLLM_ERR_INVALID: return "invalid argument or metadata";
        case NVLLM_ERR_CUDA: return "CUDA runtime error";
        case NVLLM_ERR_TIMEOUT: return "bounded device wait timed out";
        case NVLLM_ERR_BOUNDS: return "block id or slot outside the arena";
        case NVLLM_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
        case NVLLM_ERR_UNSUPPORTED: return "head_dim or precision not supported";
        default: return "unknown status";
    }
}

}  // extern "C"
