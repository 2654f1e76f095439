/*
 * nvllm — B200 (sm_100a) paged-KV write + paged attention for nano-vllm-cpp26.
 *
 * C ABI of libnvllm.so. All tensors are fp32 device pointers owned by the
 * caller; every call is asynchronous on the caller's CUDA stream (passed as
 * void*, i.e. a cudaStream_t; NULL = legacy default stream) and allocates
 * nothing. Return value: NVLLM_OK or one of the NVLLM_ERR_* codes below.
 *
 * Geometry follows the reference's PagedKVCache: one K and one V arena of
 * [num_blocks, num_layers, block_size, num_heads * head_dim] floats
 * (include/nano_vllm/kv_cache.hpp:30-33), i.e. row (block, layer, slot) holds
 * all heads of one token, head h at columns [h * head_dim, (h + 1) * head_dim).
 *
 * Flattened batch: the query/key/value rows of one step are the uncomputed
 * tokens of every scheduled sequence, sequence-major (src/model.cpp:138-159).
 * Sequence s owns rows [cu_seqlens_q[s], cu_seqlens_q[s+1]) and, after this
 * step's cache write, context_lens[s] cached positions; its query row i is at
 * position context_lens[s] - q_len + i and attends causally to positions
 * 0..pos through row s of block_tables ([num_seqs, max_blocks_per_seq] int32
 * physical block ids, the reference's SequenceState::block_table).
 */
#ifndef NVLLM_H
#define NVLLM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum nvllm_status {
    NVLLM_OK = 0,
    NVLLM_ERR_INVALID = 1,     /* bad argument, geometry or metadata */
    NVLLM_ERR_CUDA = 2,        /* a CUDA runtime call or launch failed */
    NVLLM_ERR_TIMEOUT = 3,     /* a bounded device wait gave up */
    NVLLM_ERR_BOUNDS = 4,      /* a block id / slot outside the arena was skipped */
    NVLLM_ERR_WORKSPACE = 5,   /* workspace missing or smaller than required */
    NVLLM_ERR_UNSUPPORTED = 6  /* head_dim or precision not built */
};

enum nvllm_precision {
    NVLLM_PRECISION_FP32 = 0,  /* fp32 FFMA everywhere (max-abs 2e-5 vs the reference) */
    NVLLM_PRECISION_TF32 = 1   /* prefill QK^T / PV tiles on the tcgen05 tensor cores (1e-3):
                                  each fp32 operand split into two bf16 terms, three bf16
                                  products per product, fp32 accumulation; when head_dim is
                                  128 and block_size 16 (other geometries keep the fp32
                                  prefill) */
};

typedef struct nvllm_kv_layout {
    int64_t num_blocks;
    int32_t num_layers;
    int32_t block_size;
    int32_t num_heads;
    int32_t head_dim;  /* 32, 64, 128 or 256 */
} nvllm_kv_layout;

/*
 * KV write of one layer for a batch. Replaces the per-token loop of
 * PagedKVCache::write_kv calls at src/model.cpp:188-202 (write_kv itself:
 * src/kv_cache.cpp:57-68). Row t of key/value ([num_tokens, H*hd]) is copied
 * bit-exactly to arena row (slot_mapping[t] / B, layer, slot_mapping[t] % B);
 * slot_mapping[t] = block_table[pos / B] * B + pos % B (src/model.cpp:192-194).
 * A negative slot skips the token. A slot beyond the arena is skipped and
 * raises NVLLM_ERR_BOUNDS in nvllm_get_last_error().
 */
int nvllm_reshape_and_cache(const float* key, const float* value, float* k_arena,
                            float* v_arena, const int32_t* slot_mapping,
                            int64_t num_tokens, int32_t layer,
                            const nvllm_kv_layout* layout, void* stream);

/* Bytes of device workspace nvllm_paged_attention needs for a batch of at
 * most num_seqs sequences, max_query_len query rows and max_context_len
 * cached positions per sequence. */
size_t nvllm_paged_attention_workspace_size(int32_t num_seqs, int32_t max_query_len,
                                            int32_t max_context_len,
                                            const nvllm_kv_layout* layout);

/*
 * Causal paged attention with online softmax over one layer of the arena.
 * Replaces step 3d of TransformerModel::forward_batch (src/model.cpp:204-260),
 * including read_head_kv (src/kv_cache.cpp:70-81). query/out are
 * [cu_seqlens_q[num_seqs], H*hd]. Sequences with one query row go to the
 * split-K decode kernel, longer ones to the causal prefill kernel; both run
 * in fp32 (precision selects the prefill tile arithmetic). max_query_len and
 * max_context_len bound the per-sequence values (the kernels check them).
 * scale is the softmax scale (the reference uses 1/sqrt(head_dim),
 * src/model.cpp:205).
 */
int nvllm_paged_attention(float* out, const float* query, const float* k_arena,
                          const float* v_arena, const int32_t* block_tables,
                          int32_t max_blocks_per_seq, const int32_t* cu_seqlens_q,
                          const int32_t* context_lens, int32_t num_seqs,
                          int32_t max_query_len, int32_t max_context_len, int32_t layer,
                          float scale, int32_t precision, void* workspace,
                          size_t workspace_bytes, const nvllm_kv_layout* layout,
                          void* stream);

/*
 * nvllm_paged_attention without a caller workspace, for callers that cannot
 * allocate device memory: a host that reaches the GPU only through this C ABI
 * and has no device allocator, or a serving loop whose memory pool forbids
 * extra cudaMalloc / cudaFree (both synchronize the device mid-step). This
 * entry point has no counterpart in the reference (whose attention runs on the
 * CPU and needs no device memory at all).
 *
 * The workspace is owned by the library: a 64 MiB device array of which every
 * GPU that loads libnvllm.so holds one copy until the process exits. A batch
 * whose nvllm_paged_attention_workspace_size() exceeds 64 MiB is refused with
 * NVLLM_ERR_WORKSPACE. The entry point itself allocates nothing. Every call
 * looks up the array's device address (cudaGetSymbolAddress, with the
 * caller's device current); the first one on a device may load the library's
 * module there, so make that first call before any stream capture. Do not use
 * a device across a reset with calls in flight.
 * All calls share the one array, so calls that overlap on the GPU (different
 * streams, or host threads, without ordering between them) race and corrupt
 * each other's results: order them on one stream. Arguments and results are
 * otherwise those of nvllm_paged_attention.
 */
int nvllm_paged_attention_static(float* out, const float* query, const float* k_arena,
                                 const float* v_arena, const int32_t* block_tables,
                                 int32_t max_blocks_per_seq, const int32_t* cu_seqlens_q,
                                 const int32_t* context_lens, int32_t num_seqs,
                                 int32_t max_query_len, int32_t max_context_len,
                                 int32_t layer, float scale, int32_t precision,
                                 const nvllm_kv_layout* layout, void* stream);

/*
 * Head split of one decode batch over `world` GPUs (one process each): rank r
 * holds heads [r*Hl, (r+1)*Hl) of every sequence in its own arena (layout
 * num_heads = Hl) and computes their attention; the merge epilogue stores each
 * finished row straight into every rank's full-width output buffer
 * outs[0..world) ([n_tokens, world*Hl*head_dim], head-major like the
 * single-GPU output), peer memory reached over NVLink, so that on completion
 * (in stream order) every rank's outs[rank] holds all heads. The writer of a
 * rank's last row adds 1 to each rank's flags[r] (a uint32 in that rank's
 * memory); the call returns its stream to the caller after
 * flags[rank] >= epoch * world, waiting at most 2 s (then NVLLM_ERR_TIMEOUT in
 * nvllm_get_last_error). epoch counts the calls on this group from 1; flags
 * start at 0. Output buffers may be alternated by epoch parity: a rank cannot
 * write epoch e + 2 before every rank finished epoch e + 1. Decode batches only
 * (one query row per sequence). The reference has no multi-GPU code; this is
 * the head-split scheme for one long-context sequence batch.
 */
#define NVLLM_MAX_RANKS 8
typedef struct nvllm_head_split {
    int32_t rank;
    int32_t world;
    uint32_t epoch;
    float* outs[NVLLM_MAX_RANKS];      /* device pointers valid in this process */
    uint32_t* flags[NVLLM_MAX_RANKS];  /* device pointers valid in this process */
} nvllm_head_split;

int nvllm_paged_attention_head_split(const nvllm_head_split* hs, const float* query,
                                     const float* k_arena, const float* v_arena,
                                     const int32_t* block_tables, int32_t max_blocks_per_seq,
                                     const int32_t* cu_seqlens_q, const int32_t* context_lens,
                                     int32_t num_seqs, int32_t max_context_len, int32_t layer,
                                     float scale, void* workspace, size_t workspace_bytes,
                                     const nvllm_kv_layout* layout, void* stream);

/* Synchronizes the stream, then returns (and clears) the device status word
 * of the current device that the kernels set on skipped out-of-range accesses,
 * inconsistent metadata or bounded waits that gave up. The reference has
 * assert()s for these (src/kv_cache.cpp:50-51, :63-64). */
int nvllm_get_last_error(void* stream);

/* Device address of that status word on the current device (nonzero = some
 * kernel raised a status since it was last cleared), so that a caller can read
 * it with an asynchronous copy in the same stream as its results instead of
 * the synchronous read of nvllm_get_last_error; call nvllm_get_last_error to
 * decode and clear a nonzero word. */
int nvllm_device_status_word(const uint32_t** word);

/* The raw status word that the last nvllm_get_last_error call (in this process)
 * found nonzero and cleared: bit 1 NVLLM_ERR_TIMEOUT, bit 0 NVLLM_ERR_BOUNDS, bit
 * 2 inconsistent metadata; with a timeout, bits 8-15 name the kernel whose
 * bounded wait gave up (8 decode attention, 9 tensor-core prefill, 10
 * nvllm_gemm_tf32x3, 11 nvllm_gemm_skinny, 12 nvllm_gemm_decode_tc, 13 fp32
 * prefill, 14 nvllm_head_gather's wait for every rank's rows, 15
 * nvllm_paged_attention_head_split's). 0 if none was seen. */
uint32_t nvllm_last_status_word(void);

/* With that word, where the first bounded wait that gave up was: info[0] its
 * kernel bits (as above, | 1), info[1] a kernel-specific code (the role,
 * barrier and pipeline stage of the wait), info[2] the CTA, info[3] the low
 * word of the mbarrier at the time. For the two cross-GPU flag waits (bits 14
 * and 15) info[1] is the flag value awaited and info[3] the value last read.
 * All 0 when no wait gave up. */
int nvllm_last_timeout_info(uint32_t* info);

/* Static string for a status code. */
const char* nvllm_status_string(int status);

#ifdef __cplusplus
}
#endif
#endif /* NVLLM_H */
