/*
 * nvllm host library (libnvllm_host.so): the engine-side half of the boundary,
 * C ABI over the C++23 classes in nano-vllm-cpp26_b200/host/.
 *
 * - Block allocator: the reference BlockManager's semantics
 *   (PagedKVCache::allocate_block / allocate_blocks / free_blocks,
 *   src/kv_cache.cpp:23-55): FIFO free list, all-or-nothing allocation.
 *   Host only, no GPU needed.
 * - Metadata packer: selective token flattening (src/model.cpp:138-159) and
 *   the slot mapping (src/model.cpp:192-194) packed into one int32 buffer.
 *   Host only.
 * - Engine: per-device K/V arenas in HBM with their allocator, one pinned
 *   metadata upload per iteration, and a per-layer attention step with host
 *   rows; the replacement of steps 3c/3d of forward_batch
 *   (src/model.cpp:188-260) on the engine thread (src/engine.cpp:212-213).
 *
 * Block ids are int64 (the reference's BlockId is size_t). Status codes:
 * NVLLM_OK, NVLLM_HOST_OUT_OF_BLOCKS, NVLLM_HOST_INVALID_BLOCK, or the
 * nvllm_status values of nvllm.h.
 */
#ifndef NVLLM_HOST_H
#define NVLLM_HOST_H

#include <stddef.h>
#include <stdint.h>

#include "nvllm.h"

#ifdef __cplusplus
extern "C" {
#endif

enum nvllm_host_status {
    NVLLM_HOST_OUT_OF_BLOCKS = 100, /* KVError::OutOfPhysicalBlocks */
    NVLLM_HOST_INVALID_BLOCK = 101, /* free of an unallocated or out-of-range id */
    NVLLM_HOST_PACK_ERROR = 102     /* tables too short / too wide, bad lengths */
};

/* ---- block allocator (kv_cache.hpp:48-55) -------------------------------- */
typedef struct nvllm_block_allocator nvllm_block_allocator;
nvllm_block_allocator* nvllm_block_allocator_create(int64_t num_blocks);
void nvllm_block_allocator_destroy(nvllm_block_allocator* a);
int nvllm_block_allocator_allocate_block(nvllm_block_allocator* a, int64_t* out_id);
int nvllm_block_allocator_allocate_blocks(nvllm_block_allocator* a, int64_t count,
                                          int64_t* out_ids);
int nvllm_block_allocator_free_blocks(nvllm_block_allocator* a, const int64_t* ids, int64_t n);
int64_t nvllm_block_allocator_num_free(const nvllm_block_allocator* a);

/* ---- metadata packer (model.cpp:138-159, :192-194) ------------------------ */
typedef struct nvllm_metadata_offsets {
    int64_t cu_seqlens_q, context_lens, last_token_idx, slot_mapping, block_tables, bytes;
    int32_t num_seqs, num_tokens, max_blocks, max_query_len, max_context_len;
} nvllm_metadata_offsets;

/* Sequence s: num_computed[s] cached tokens, total_len[s] tokens after the
 * step, table_lens[s] block ids taken in order from block_ids. */
size_t nvllm_metadata_bytes(int32_t num_seqs, int32_t num_tokens, int32_t max_blocks);
int nvllm_pack_metadata(int32_t num_seqs, const int32_t* num_computed, const int32_t* total_len,
                        const int64_t* block_ids, const int32_t* table_lens, int32_t block_size,
                        int32_t max_blocks, void* buf, size_t buf_bytes,
                        nvllm_metadata_offsets* out);
/* The same batch laid out as pad_seqs sequences and pad_tokens token rows
 * (at least the batch's own): extra sequences empty (cu_seqlens repeats the
 * token count, context 0, last_token_idx 0, zero table row), extra token rows
 * with slot -1; sizes from nvllm_metadata_bytes(pad_seqs, pad_tokens, ...). */
int nvllm_pack_metadata_padded(int32_t num_seqs, const int32_t* num_computed,
                               const int32_t* total_len, const int64_t* block_ids,
                               const int32_t* table_lens, int32_t block_size, int32_t max_blocks,
                               int32_t pad_seqs, int32_t pad_tokens, void* buf,
                               size_t buf_bytes, nvllm_metadata_offsets* out);

/* ---- engine --------------------------------------------------------------- */
typedef struct nvllm_engine nvllm_engine;
typedef struct nvllm_engine_config {
    nvllm_kv_layout layout;
    int32_t max_seqs;
    int32_t max_tokens;
    int32_t max_blocks_per_seq;
    int32_t device;
} nvllm_engine_config;

int nvllm_engine_create(const nvllm_engine_config* cfg, nvllm_engine** out);
void nvllm_engine_destroy(nvllm_engine* e);
int nvllm_engine_allocate_blocks(nvllm_engine* e, int64_t count, int64_t* out_ids);
int nvllm_engine_free_blocks(nvllm_engine* e, const int64_t* ids, int64_t n);
int64_t nvllm_engine_num_free_blocks(const nvllm_engine* e);
/* Flattens the batch and uploads its metadata (one cudaMemcpyAsync). */
int nvllm_engine_begin_step(nvllm_engine* e, int32_t num_seqs, const int32_t* num_computed,
                            const int32_t* total_len, const int64_t* block_ids,
                            const int32_t* table_lens);
/* begin_step laid out as pad_seqs sequences and pad_tokens token rows (at
 * least the batch's own; at most max_seqs / max_tokens): the extra sequences
 * are empty and the extra rows have slot -1, and the step's attention bounds
 * become those of the bucket, so that every batch of a bucket issues the same
 * launches. */
int nvllm_engine_begin_step_padded(nvllm_engine* e, int32_t num_seqs, const int32_t* num_computed,
                                   const int32_t* total_len, const int64_t* block_ids,
                                   const int32_t* table_lens, int32_t pad_seqs,
                                   int32_t pad_tokens);
/* One layer, host rows [num_tokens, H*hd]; returns when out holds the result. */
int nvllm_engine_attention(nvllm_engine* e, int32_t layer, const float* q, const float* k,
                           const float* v, float* out, int32_t precision);
/* The engine's pinned row buffers (pass them to nvllm_engine_attention to skip
 * the staging copy), its device arenas and its CUDA stream. */
int nvllm_engine_host_buffers(nvllm_engine* e, float** q, float** k, float** v, float** out);
/* Pipelined host-row attention over two slots (no counterpart in the
 * reference, whose attention is a synchronous CPU loop): fill a slot's pinned
 * rows (nvllm_engine_slot_buffers, slot 0 or 1; slot 0's are those of
 * nvllm_engine_host_buffers), then nvllm_engine_attention_submit queues, for
 * the step begun last, their H2D on the engine's copy stream, the KV write +
 * attention on its compute stream once they have landed, and the D2H of the
 * output into the slot's pinned output buffer once the kernels are done, and
 * returns without waiting; nvllm_engine_attention_collect waits for that
 * output. Alternating slots lets one step's copies overlap the other step's
 * kernels. A slot must be collected before its rows are refilled or it is
 * submitted again; nvllm_engine_attention refuses while a slot is in flight. */
int nvllm_engine_slot_buffers(nvllm_engine* e, int32_t slot, float** q, float** k, float** v,
                              float** out);
int nvllm_engine_attention_submit(nvllm_engine* e, int32_t layer, int32_t slot,
                                  int32_t precision);
int nvllm_engine_attention_collect(nvllm_engine* e, int32_t slot);
int nvllm_engine_arenas(nvllm_engine* e, float** k_arena, float** v_arena);
void* nvllm_engine_stream(nvllm_engine* e);
int32_t nvllm_engine_step_tokens(const nvllm_engine* e);

/* ---- device model (TransformerModel, src/model.cpp:64-312) ----------------
 * The reference's LCG-weighted transformer on the engine's GPU: weights
 * generated on the device in the constructor's draw order, forward_batch as
 * device kernels (embedding gather, RMSNorm, fp32 projections, paged KV write
 * and attention through the engine, SiLU, residual adds, last-token gather,
 * LM head, repetition-penalised greedy sampling). The engine's layout must
 * match (layers, heads, head_dim); destroy the model before its engine. */
typedef struct nvllm_model nvllm_model;
/* Arithmetic of the projections (fp32 in, fp32 out either way). */
enum nvllm_gemm_math {
    NVLLM_GEMM_FP32 = 0,  /* fp32 FFMA (CUDA cores) */
    NVLLM_GEMM_BF16X9 = 1, /* fp32 emulated on the tensor cores: each operand split into three
                              bf16 terms, products accumulated in fp32 (cuBLAS's bf16x9 mode;
                              NVLLM_ERR_UNSUPPORTED when the cuBLAS in the process lacks it) */
    NVLLM_GEMM_TF32X3 = 2  /* this library's kernels, fp32 quality: nvllm_gemm_tf32x3
                              (tcgen05, 3xTF32) for every projection of more than 32 rows,
                              nvllm_gemm_decode_tc (tcgen05, 3xTF32) for 17-32 rows and
                              nvllm_gemm_skinny (FFMA) for at most 16, the LM head included,
                              each with the residual add, SiLU and Q/K/V split in its epilogue.
                              hidden, ffn and vocab must be multiples of 128. */
};
typedef struct nvllm_model_config {
    int64_t vocab, hidden, layers, heads, head_dim, ffn;
    float emb_scale, ffn_scale; /* weight scales; 0 = 1/sqrt(hidden), 1/sqrt(ffn) */
    int32_t gemm_math;          /* nvllm_gemm_math */
    /* Steps begun padded (nvllm_engine_begin_step_padded; the generator pads
     * every step of at most this many new tokens to power-of-two buckets) run
     * as one CUDA graph per bucket, captured on first use. 0: always eager. */
    int32_t graph_max_tokens;
    /* Head parallelism over this many GPUs, one process each (<= 8; 0 or 1:
     * single GPU): the engine holds heads / head_ranks heads (layout num_heads),
     * QKV runs for this rank's heads only, nvllm_head_gather collects every
     * rank's attention rows before W_o, and W_o, the FFN and the LM head run
     * replicated, so that every rank samples the same tokens. Needs
     * nvllm_model_set_head_group before the first forward and graph_max_tokens
     * 0; with gemm_math 2, hidden / head_ranks a multiple of 128. No
     * counterpart in the reference (one CPU process). */
    int32_t head_ranks;
} nvllm_model_config;

int nvllm_model_create(const nvllm_model_config* cfg, nvllm_engine* engine, nvllm_model** out);
void nvllm_model_destroy(nvllm_model* m);

/* The peers of a head-parallel model (head_ranks = world): this rank, the gather
 * buffers of every rank by epoch parity (outs[p][r]: [engine max_tokens, hidden]
 * fp32 on rank r, e.g. nvllm_ipc_alloc'd and opened in every process) and every
 * rank's flag word (uint32, starting at 0). Every rank must run the same steps
 * (the same requests and scheduler settings). */
typedef struct nvllm_model_head_group {
    int32_t rank, world;
    float* outs[2][NVLLM_MAX_RANKS];
    uint32_t* flags[NVLLM_MAX_RANKS];
} nvllm_model_head_group;
int nvllm_model_set_head_group(nvllm_model* m, const nvllm_model_head_group* g);
/* forward_batch over the step begun with nvllm_engine_begin_step: token_ids =
 * the uncomputed tokens of every sequence in batch order (num_tokens of them,
 * taken modulo the vocabulary), prev_tokens[s] = sequence s's last token.
 * Writes sampled[num_seqs]. With top_k in 1..32 also writes margins[s] (top-1
 * minus top-2 of the penalised logits) and the top_k largest raw logits of
 * each row (top_idx / top_val, [num_seqs, top_k]). Returns once the results
 * are on the host. */
int nvllm_model_forward(nvllm_model* m, const int64_t* token_ids, int64_t num_tokens,
                        const int64_t* prev_tokens, int64_t num_seqs, int64_t* sampled,
                        int32_t precision, float* margins, int32_t* top_idx, float* top_val,
                        int32_t top_k);
/* The device weight buffer (read-only; count floats in draw order). */
int nvllm_model_weights(const nvllm_model* m, const float** weights, int64_t* count);

/* ---- continuous-batching scheduler (src/scheduler.cpp) ---------------------
 * The reference ContinuousScheduler's policy: recompute preemption of the
 * youngest running sequences when the arena is full, admission in queue order
 * under a batch-size, token-budget and free-block watermark limit, retirement
 * by swap with the last running sequence. Host logic only; it draws blocks from
 * the allocator passed to each call. */
typedef struct nvllm_scheduler_config {
    int64_t max_batch_size, max_tokens_per_step, watermark_blocks;
    int64_t eos_token_id; /* < 0: none */
} nvllm_scheduler_config;
typedef struct nvllm_step_summary {
    int64_t admitted, preempted, retired, batch_size, scheduled_tokens;
} nvllm_step_summary;
typedef struct nvllm_scheduler nvllm_scheduler;

nvllm_scheduler* nvllm_scheduler_create(const nvllm_scheduler_config* cfg, int32_t block_size);
void nvllm_scheduler_destroy(nvllm_scheduler* s);
/* An empty prompt becomes {1}; max_new_tokens below 1 becomes 1. */
int nvllm_scheduler_add_request(nvllm_scheduler* s, uint64_t seq_id, const int64_t* prompt,
                                int64_t prompt_len, int64_t max_new_tokens);
int nvllm_scheduler_schedule_step(nvllm_scheduler* s, nvllm_block_allocator* blocks,
                                  nvllm_step_summary* out);
/* The running batch as one trace record (int64): -1, step, n, then per
 * sequence seq_id, num_computed, total_len, last token, table_len, table...,
 * n_uncomputed, uncomputed.... Returns the record's length; writes it only when
 * it fits in cap. */
int64_t nvllm_scheduler_batch_record(const nvllm_scheduler* s, int64_t step, int64_t* out,
                                     int64_t cap);
/* One sampled token per running sequence, in batch order. */
int nvllm_scheduler_process_outputs(nvllm_scheduler* s, nvllm_block_allocator* blocks,
                                    const int64_t* sampled, int64_t n, int64_t* retired);
int nvllm_scheduler_counts(const nvllm_scheduler* s, int64_t* running, int64_t* waiting,
                           int64_t* preemptions, int64_t* completed);

/* ---- generator: the engine loop on one GPU (src/engine.cpp:163-246) -------
 * schedule_step -> device forward_batch -> process_step_outputs, on the
 * engine's arena and allocator and the model's forward. Destroy before the
 * model and the engine. */
typedef struct nvllm_generator nvllm_generator;
/* The reference's MetricsSnapshot (include/nano_vllm/engine.hpp:43-60). */
typedef struct nvllm_metrics {
    double uptime_secs;
    uint64_t total_requests_received, total_requests_completed, total_tokens_generated;
    double throughput_tokens_per_sec;
    uint64_t active_batch_size, waiting_queue_depth, kv_cache_used_blocks, kv_cache_total_blocks;
    double kv_cache_utilization_pct, avg_ttft_ms, avg_iteration_latency_ms;
    uint64_t total_preemptions, total_iterations;
    /* beyond the reference's snapshot: flattened rows computed, bytes copied
     * host->device / device->host, launches of this library's kernels */
    uint64_t total_tokens_computed, h2d_bytes, d2h_bytes, kernel_launches;
} nvllm_metrics;

int nvllm_generator_create(nvllm_engine* engine, nvllm_model* model,
                           const nvllm_scheduler_config* cfg, int32_t precision,
                           nvllm_generator** out);
void nvllm_generator_destroy(nvllm_generator* g);
int nvllm_generator_add_request(nvllm_generator* g, uint64_t seq_id, const int64_t* prompt,
                                int64_t prompt_len, int64_t max_new_tokens);
int nvllm_generator_step(nvllm_generator* g, nvllm_step_summary* out);
/* Steps until no work is pending (max_steps <= 0) or max_steps steps ran;
 * NVLLM_ERR_INVALID when the queue head can never be admitted. */
int nvllm_generator_run(nvllm_generator* g, int64_t max_steps, int64_t* steps_done);
int nvllm_generator_has_pending_work(const nvllm_generator* g);
/* Token list (prompt + generated) of finished sequence seq_id: returns its
 * length (writing it when it fits in cap), or -1 if it has not finished. */
int64_t nvllm_generator_output(const nvllm_generator* g, uint64_t seq_id, int64_t* tokens,
                               int64_t cap);
/* Records every following step to path (trace record + -2, sampled ids, per
 * sequence the top-2 margin and 8 largest logits as float bits); NULL or ""
 * stops recording. */
int nvllm_generator_trace(nvllm_generator* g, const char* path);
int nvllm_generator_metrics(const nvllm_generator* g, nvllm_metrics* out);
/* MetricsSnapshot::to_json layout (src/engine.cpp:8-38); returns the length
 * (without the terminator), writing it when it fits in cap. */
int64_t nvllm_metrics_to_json(const nvllm_metrics* m, char* buf, int64_t cap);

/* ---- router: one request stream over the GPUs of a box -------------------
 * Sequence partitioning: each generator (one per GPU, each with its own
 * engine, arena, allocator, scheduler and model) gets its own engine thread
 * and ingress queue, the counterpart of the reference engine's ingress queue
 * and engine thread (src/engine.cpp:79-104, :163-246), one per device here.
 * nvllm_router_add_request places a request on the GPU with the least
 * outstanding work (rows still to run through the forward pass: uncomputed
 * prompt tokens plus tokens still to generate, of what the GPU holds or has
 * queued) and returns that GPU's index in gens. The generators must outlive the
 * router and must not be used directly while it exists. */
typedef struct nvllm_router nvllm_router;
int nvllm_router_create(nvllm_generator* const* gens, int32_t n, nvllm_router** out);
/* Stops and joins the engine threads (work still pending is dropped). */
void nvllm_router_destroy(nvllm_router* r);
int nvllm_router_add_request(nvllm_router* r, uint64_t seq_id, const int64_t* prompt,
                             int64_t prompt_len, int64_t max_new_tokens, int32_t* gpu);
/* A burst of n requests in one call: request k's prompt is
 * tokens[offsets[k] .. offsets[k + 1]) (offsets has n + 1 entries), its
 * completion max_new_tokens[k]. Placed in one decision pass, each on the GPU
 * that is least loaded counting those placed before it in the burst, then each
 * GPU is woken once, so that its engine thread takes its whole share in its
 * next iteration (placing a burst one call at a time while the engines run
 * spreads it over many small iterations). All or nothing: an id in use or
 * repeated places none (NVLLM_ERR_INVALID). gpus, when not NULL, receives each
 * request's GPU. No counterpart in the reference, whose engine takes one
 * request per submit (src/engine.cpp:89-104); this is a batch form of it. */
int nvllm_router_add_requests(nvllm_router* r, int64_t n, const uint64_t* seq_ids,
                              const int64_t* tokens, const int64_t* offsets,
                              const int64_t* max_new_tokens, int32_t* gpus);
/* Blocks until every GPU is idle with an empty queue; the error of a GPU whose
 * loop failed (its thread stops; the others carry on). */
int nvllm_router_wait_idle(nvllm_router* r);
/* As nvllm_generator_output, for a finished request on whichever GPU served
 * it; -1 while that GPU is busy, or for an unknown or unfinished request. */
int64_t nvllm_router_output(nvllm_router* r, uint64_t seq_id, int64_t* tokens, int64_t cap);
/* A GPU's telemetry as of its engine thread's last idle moment. */
int nvllm_router_metrics(nvllm_router* r, int32_t gpu, nvllm_metrics* out);
/* Requests placed on a GPU so far (-1 for a bad index). */
int64_t nvllm_router_placed(const nvllm_router* r, int32_t gpu);

/* ---- HTTP/SSE front end (the reference's HttpSseServer, src/server.cpp) ----
 * Serves GET /health, GET /v1/metrics (the MetricsSnapshot JSON of
 * src/engine.cpp:8-38 summed over the router's GPUs, plus a "gpus" list with
 * each GPU's arena use, iterations, bytes copied and kernel launches) and
 * POST /v1/generate {"prompt": "...", "max_tokens": n}, answered as a
 * text/event-stream with one frame per generated token in the reference's
 * format: data: {"seq_id":S,"token_id":T,"text":"...","finished":B[,"ttft_us":U]}.
 * Prompts are tokenised and tokens named as the reference does
 * (src/engine.cpp:40-64, src/model.cpp:114-121). nvllm_server_start binds
 * bind_address:port (NULL: 127.0.0.1; port 0: any free port) and accepts on a
 * background thread; stop it before destroying the router. */
typedef struct nvllm_server nvllm_server;
int nvllm_server_start(nvllm_router* r, int64_t vocab_size, const char* bind_address,
                       int32_t port, nvllm_server** out);
/* The port the server listens on. */
int32_t nvllm_server_port(const nvllm_server* s);
/* Stops accepting, ends the open streams and joins the server's threads. */
void nvllm_server_stop(nvllm_server* s);
/* The reference engine's prompt tokenisation; returns the token count,
 * writing the ids when they fit in cap. */
int64_t nvllm_tokenize_prompt(const char* text, int64_t vocab_size, int64_t* out, int64_t cap);

/* ---- cross-process device buffers (head split) ---------------------------
 * nvllm_ipc_alloc: cudaMalloc of `bytes` on the current device, zero-filled,
 * and its 64-byte CUDA IPC handle. nvllm_ipc_open maps a peer process's buffer
 * into this process (peer access over NVLink enabled lazily); nvllm_ipc_close
 * unmaps it; nvllm_ipc_free releases an nvllm_ipc_alloc buffer. */
#define NVLLM_IPC_HANDLE_BYTES 64
int nvllm_ipc_alloc(size_t bytes, void** dev_ptr, void* handle);
int nvllm_ipc_open(const void* handle, void** dev_ptr);
int nvllm_ipc_close(void* dev_ptr);
int nvllm_ipc_free(void* dev_ptr);

#ifdef __cplusplus
}
#endif
#endif /* NVLLM_HOST_H */
