/* CPU oracle for the paged-KV write + paged attention path (test
 * infrastructure only: tests, the smoke check and the benchmark's CPU-baseline
 * leg load it as the checker; the product never does).
 *
 * A plain-C restatement of the reference's algorithm. Each function names the
 * reference lines it follows; index arithmetic is bit-exact with the reference,
 * and the float attention keeps the reference's per-position accumulation
 * order (src/model.cpp:225-258).
 */
#ifndef NVLLM_ORACLE_H
#define NVLLM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Arena geometry: [num_blocks, num_layers, block_size, num_heads * head_dim]
 * floats per K and per V (include/nano_vllm/kv_cache.hpp:30-33). */
typedef struct oracle_kv_layout {
    int64_t num_blocks;
    int32_t num_layers;
    int32_t block_size;
    int32_t num_heads;
    int32_t head_dim;
} oracle_kv_layout;

/* Selective token flattening (src/model.cpp:138-159). Sequence s has
 * total_len[s] tokens, the first num_computed[s] already in the cache. Emits
 * cu_seqlens_q[num_seqs + 1], context_lens[num_seqs] (= total_len, the KV
 * extent after this step), and per flattened token its position and sequence
 * index; last_token_idx[s] is the flat index of sequence s's last token
 * (model.cpp:156). Returns the number of flattened tokens. */
int64_t oracle_flatten(int32_t num_seqs, const int32_t* num_computed,
                       const int32_t* total_len, int32_t* cu_seqlens_q,
                       int32_t* context_lens, int32_t* positions,
                       int32_t* seq_of_token, int32_t* last_token_idx);

/* Slot of each flattened token: block_table[pos / B] * B + pos % B
 * (src/model.cpp:192-194). block_tables is [num_seqs, max_blocks] int32. */
void oracle_slot_mapping(int32_t num_seqs, const int32_t* cu_seqlens_q,
                         const int32_t* context_lens, const int32_t* block_tables,
                         int32_t max_blocks, int32_t block_size,
                         int32_t* slot_mapping);

/* PagedKVCache::write_kv for a batch (src/kv_cache.cpp:57-68 with offset() at
 * include/nano_vllm/kv_cache.hpp:73-78): row t of k/v ([n_tokens, D]) goes to
 * (slot / B, layer, slot % B). Tokens with a negative slot are skipped. */
void oracle_reshape_and_cache(const float* k, const float* v, float* k_arena,
                              float* v_arena, const int32_t* slot_mapping,
                              int64_t n_tokens, int32_t layer,
                              const oracle_kv_layout* lay);

/* Causal paged attention with online softmax (src/model.cpp:204-260). Query
 * token i of sequence s sits at position context_lens[s] - q_len + i and
 * attends to positions 0..pos through the block table. q/out are
 * [n_tokens, D]. use_f64 = 0 follows the reference's float arithmetic and
 * order; 1 accumulates in double (a tighter yardstick for error reports).
 * seq_select (may be NULL) restricts the work to flagged sequences; other rows
 * of out are left untouched. num_threads <= 0 uses one thread. */
void oracle_paged_attention(float* out, const float* q, const float* k_arena,
                            const float* v_arena, const int32_t* block_tables,
                            int32_t max_blocks, const int32_t* cu_seqlens_q,
                            const int32_t* context_lens, int32_t num_seqs,
                            int32_t layer, float scale, const oracle_kv_layout* lay,
                            int32_t use_f64, const uint8_t* seq_select,
                            int32_t num_threads);

#ifdef __cplusplus
}
#endif
#endif
