// Launch interfaces shared between the kernels and the C ABI (nvllm_abi.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "common.cuh"

namespace nvllm {

// Work items produced by the plan kernel.
//   decode item  (seq, split):  positions [split*P, min((split+1)*P, ctx))
//   prefill item (seq, tile):   query rows [tile*QT, min((tile+1)*QT, q_len))
struct WorkItem {
    int32_t seq;
    int32_t part;
};

// Counters at the head of the workspace.
struct PlanCounters {
    int32_t decode_next;    // dynamic fetch cursor (decode)
    int32_t decode_items;   // number of decode items
    int32_t prefill_next;   // dynamic fetch cursor (prefill)
    int32_t prefill_items;  // number of prefill items
    int32_t decode_seqs;    // sequences with one query row
    int32_t rows_done;      // head split: (sequence, head) rows stored so far
};

// Head split: ranks that share one batch, each owning a slice of the heads.
constexpr int kMaxRanks = 8;

struct AttnParams {
    float* out;
    const float* q;
    const float* k_arena;
    const float* v_arena;
    const int32_t* block_tables;
    const int32_t* cu_seqlens_q;
    const int32_t* context_lens;
    int32_t max_blocks;
    int32_t num_seqs;
    int32_t max_query_len;
    int32_t max_context_len;
    int32_t layer;
    float qk_scale_log2;  // softmax scale * log2(e): scores live in the log2 domain
    ArenaGeom g;
    // workspace views
    PlanCounters* counters;
    WorkItem* decode_items;
    WorkItem* prefill_items;
    float* part_acc;     // [num_seqs, H, max_splits, hd] un-normalised partial outputs
    float2* part_ml;     // [num_seqs, H, max_splits] (running max (log2), running sum)
    int32_t max_splits;
    int32_t split_tokens;     // P: positions per decode item
    int32_t prefill_tile;     // QT: query rows per prefill item
    int32_t beside_prefill;   // decode launched beside a prefill (no wait for it)
    // Head split (num_outs > 0): every decode row leaves through the merge
    // kernel, which stores it at column out_col of row token in each of the
    // num_outs output buffers (this rank's and its peers', row stride
    // out_stride floats), then signals each rank's arrival counter once all
    // of this rank's rows are out.
    int32_t num_outs;
    float* outs[kMaxRanks];
    uint32_t* flags[kMaxRanks];
    int64_t out_stride;
    int64_t out_col;
};

// Workspace carve-up shared by the size query and the launcher.
struct WorkspaceLayout {
    size_t counters_off, decode_items_off, prefill_items_off, part_acc_off, part_ml_off, total;
    int32_t max_splits, split_tokens, prefill_tile;
};

WorkspaceLayout workspace_layout(int32_t num_seqs, int32_t max_query_len, int32_t max_context_len,
                                 int32_t num_heads, int32_t head_dim);

cudaError_t launch_reshape_and_cache(const float* key, const float* value, float* k_arena,
                                     float* v_arena, const int32_t* slot_mapping,
                                     int64_t num_tokens, int32_t layer, const ArenaGeom& g,
                                     bool vec4, cudaStream_t stream);

cudaError_t launch_plan(const AttnParams& p, cudaStream_t stream);
// Head split: increments every rank's arrival counter (one thread).
cudaError_t launch_signal(uint32_t* const* flags, int n, cudaStream_t stream);
// Waits (bounded) until *flag >= target; one thread.
cudaError_t launch_flag_wait(const uint32_t* flag, uint32_t target, cudaStream_t stream);
// overlap_previous: launch the decode kernel as a programmatic dependent of the
// kernel before it in the stream (a prefill kernel, which releases it at its
// start), so that it runs beside that kernel on the SMs it leaves free.
cudaError_t launch_decode(const AttnParams& p, cudaStream_t stream, bool overlap_previous = false);
// max_sms > 0 bounds the persistent grid to that many SMs' worth of CTAs (the
// rest of the GPU is left to a decode kernel running beside it); 0 = all SMs.
cudaError_t launch_prefill_fp32(const AttnParams& p, cudaStream_t stream, int max_sms = 0);
cudaError_t launch_prefill_tc(const AttnParams& p, cudaStream_t stream, int max_sms = 0);
bool prefill_tc_supported(const ArenaGeom& g);
int32_t prefill_tc_tile_rows();

// Positions per decode work item: 16 chunks of 2048/hd positions (256 KiB of
// K+V at any head_dim).
int32_t decode_split_tokens(int32_t head_dim);
int32_t prefill_tile_rows(int32_t head_dim);

}  // namespace nvllm
