/* CPU oracle for the paged-KV write + paged attention path. Test
 * infrastructure: only tests, the smoke check and the benchmark's CPU-baseline
 * leg call it, as the checker. See nvllm_oracle.h for the contract. */
#include "nvllm_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

int64_t oracle_flatten(int32_t num_seqs, const int32_t* num_computed,
                       const int32_t* total_len, int32_t* cu_seqlens_q,
                       int32_t* context_lens, int32_t* positions,
                       int32_t* seq_of_token, int32_t* last_token_idx) {
    /* src/model.cpp:144-157: one record per uncomputed token, sequence-major. */
    int64_t n = 0;
    cu_seqlens_q[0] = 0;
    for (int32_t s = 0; s < num_seqs; ++s) {
        const int32_t start = num_computed[s];
        for (int32_t off = 0; start + off < total_len[s]; ++off) {
            if (positions) positions[n] = start + off;
            if (seq_of_token) seq_of_token[n] = s;
            ++n;
        }
        cu_seqlens_q[s + 1] = (int32_t)n;
        context_lens[s] = total_len[s];
        if (last_token_idx) last_token_idx[s] = (int32_t)(n - 1);
    }
    return n;
}

void oracle_slot_mapping(int32_t num_seqs, const int32_t* cu_seqlens_q,
                         const int32_t* context_lens, const int32_t* block_tables,
                         int32_t max_blocks, int32_t block_size,
                         int32_t* slot_mapping) {
    for (int32_t s = 0; s < num_seqs; ++s) {
        const int32_t q_len = cu_seqlens_q[s + 1] - cu_seqlens_q[s];
        const int32_t first_pos = context_lens[s] - q_len;
        for (int32_t i = 0; i < q_len; ++i) {
            const int32_t pos = first_pos + i;
            const int32_t logical_block = pos / block_size;  /* model.cpp:192 */
            const int32_t slot_in_block = pos % block_size;  /* model.cpp:193 */
            const int32_t phys = block_tables[(int64_t)s * max_blocks + logical_block];
            slot_mapping[cu_seqlens_q[s] + i] = phys * block_size + slot_in_block;
        }
    }
}

static inline int64_t arena_offset(const oracle_kv_layout* lay, int64_t block,
                                   int64_t layer, int64_t slot) {
    /* include/nano_vllm/kv_cache.hpp:73-78 with the intended strides
     * stride_slot = H*hd, stride_layer = B*stride_slot,
     * stride_block = L*stride_layer (src/kv_cache.cpp:10-12). */
    const int64_t d = (int64_t)lay->num_heads * lay->head_dim;
    const int64_t stride_layer = (int64_t)lay->block_size * d;
    const int64_t stride_block = (int64_t)lay->num_layers * stride_layer;
    return block * stride_block + layer * stride_layer + slot * d;
}

void oracle_reshape_and_cache(const float* k, const float* v, float* k_arena,
                              float* v_arena, const int32_t* slot_mapping,
                              int64_t n_tokens, int32_t layer,
                              const oracle_kv_layout* lay) {
    const int64_t d = (int64_t)lay->num_heads * lay->head_dim;
    for (int64_t t = 0; t < n_tokens; ++t) {
        const int32_t slot = slot_mapping[t];
        if (slot < 0) continue;
        const int64_t base =
            arena_offset(lay, slot / lay->block_size, layer, slot % lay->block_size);
        memcpy(k_arena + base, k + t * d, (size_t)d * sizeof(float));
        memcpy(v_arena + base, v + t * d, (size_t)d * sizeof(float));
    }
}

typedef struct attn_job {
    float* out;
    const float* q;
    const float* k_arena;
    const float* v_arena;
    const int32_t* block_tables;
    int32_t max_blocks;
    const int32_t* cu_seqlens_q;
    const int32_t* context_lens;
    int32_t num_seqs;
    int32_t layer;
    float scale;
    const oracle_kv_layout* lay;
    int32_t use_f64;
    const uint8_t* seq_select;
    const int32_t* token_seq; /* flattened token -> sequence */
    int64_t n_tokens;
    atomic_llong next;
} attn_job;

/* One flattened token, all heads: src/model.cpp:207-259. */
static void attend_token(const attn_job* j, int64_t t) {
    const int32_t s = j->token_seq[t];
    const int64_t d = (int64_t)j->lay->num_heads * j->lay->head_dim;
    const int32_t hd = j->lay->head_dim;
    const int32_t bs = j->lay->block_size;
    const int32_t q_len = j->cu_seqlens_q[s + 1] - j->cu_seqlens_q[s];
    const int64_t pos = (int64_t)j->context_lens[s] - q_len + (t - j->cu_seqlens_q[s]);
    const int64_t num_active = pos + 1;                                 /* :212 */
    const int64_t num_logical_blocks = (num_active + bs - 1) / bs;      /* :213-214 */
    const float* q_token = j->q + t * d;
    float* out_token = j->out + t * d;
    const int32_t* table = j->block_tables + (int64_t)s * j->max_blocks;

    double* acc64 = NULL;
    if (j->use_f64) acc64 = (double*)malloc(sizeof(double) * (size_t)hd);

    for (int32_t h = 0; h < j->lay->num_heads; ++h) {               /* :216 */
        const float* q_head = q_token + (int64_t)h * hd;
        float* out_head = out_token + (int64_t)h * hd;
        if (!j->use_f64) {
            for (int32_t i = 0; i < hd; ++i) out_head[i] = 0.0f;          /* :219 */
            float running_max = -INFINITY;                                /* :221 */
            float running_sum = 0.0f;                                     /* :222 */
            for (int64_t lb = 0; lb < num_logical_blocks; ++lb) {         /* :225 */
                const int64_t phys = table[lb];
                const int64_t slots = (lb + 1 == num_logical_blocks)
                                          ? (num_active - lb * bs) : bs;  /* :227-230 */
                for (int64_t slot = 0; slot < slots; ++slot) {           /* :232 */
                    const int64_t base = arena_offset(j->lay, phys, j->layer, slot) +
                                         (int64_t)h * hd;                 /* read_head_kv */
                    const float* k_head = j->k_arena + base;
                    const float* v_head = j->v_arena + base;
                    float dot = 0.0f;
                    for (int32_t i = 0; i < hd; ++i) dot += q_head[i] * k_head[i];
                    const float score = dot * j->scale;                   /* :240 */
                    const float new_max = running_max > score ? running_max : score;
                    const float exp_prev = expf(running_max - new_max);   /* :244 */
                    const float exp_curr = expf(score - new_max);         /* :245 */
                    running_sum = running_sum * exp_prev + exp_curr;      /* :247 */
                    for (int32_t i = 0; i < hd; ++i)
                        out_head[i] = out_head[i] * exp_prev + exp_curr * v_head[i];
                    running_max = new_max;
                }
            }
            const float inv_sum = 1.0f / (running_sum > 1e-12f ? running_sum : 1e-12f);
            for (int32_t i = 0; i < hd; ++i) out_head[i] *= inv_sum;      /* :255-258 */
        } else {
            for (int32_t i = 0; i < hd; ++i) acc64[i] = 0.0;
            double running_max = -INFINITY;
            double running_sum = 0.0;
            for (int64_t lb = 0; lb < num_logical_blocks; ++lb) {
                const int64_t phys = table[lb];
                const int64_t slots = (lb + 1 == num_logical_blocks) ? (num_active - lb * bs) : bs;
                for (int64_t slot = 0; slot < slots; ++slot) {
                    const int64_t base = arena_offset(j->lay, phys, j->layer, slot) +
                                         (int64_t)h * hd;
                    const float* k_head = j->k_arena + base;
                    const float* v_head = j->v_arena + base;
                    double dot = 0.0;
                    for (int32_t i = 0; i < hd; ++i) dot += (double)q_head[i] * (double)k_head[i];
                    const double score = dot * (double)j->scale;
                    const double new_max = running_max > score ? running_max : score;
                    const double exp_prev = exp(running_max - new_max);
                    const double exp_curr = exp(score - new_max);
                    running_sum = running_sum * exp_prev + exp_curr;
                    for (int32_t i = 0; i < hd; ++i)
                        acc64[i] = acc64[i] * exp_prev + exp_curr * (double)v_head[i];
                    running_max = new_max;
                }
            }
            const double inv_sum = 1.0 / (running_sum > 1e-12 ? running_sum : 1e-12);
            for (int32_t i = 0; i < hd; ++i) out_head[i] = (float)(acc64[i] * inv_sum);
        }
    }
    free(acc64);
}

static void* attn_worker(void* arg) {
    attn_job* j = (attn_job*)arg;
    for (;;) {
        const long long t = atomic_fetch_add(&j->next, 1);
        if (t >= j->n_tokens) break;
        if (j->seq_select && !j->seq_select[j->token_seq[t]]) continue;
        attend_token(j, (int64_t)t);
    }
    return NULL;
}

void oracle_paged_attention(float* out, const float* q, const float* k_arena,
                            const float* v_arena, const int32_t* block_tables,
                            int32_t max_blocks, const int32_t* cu_seqlens_q,
                            const int32_t* context_lens, int32_t num_seqs,
                            int32_t layer, float scale, const oracle_kv_layout* lay,
                            int32_t use_f64, const uint8_t* seq_select,
                            int32_t num_threads) {
    if (num_seqs <= 0) return;
    const int64_t n_tokens = cu_seqlens_q[num_seqs];
    if (n_tokens <= 0) return;
    int32_t* token_seq = (int32_t*)malloc(sizeof(int32_t) * (size_t)n_tokens);
    for (int32_t s = 0; s < num_seqs; ++s)
        for (int32_t t = cu_seqlens_q[s]; t < cu_seqlens_q[s + 1]; ++t) token_seq[t] = s;

    attn_job job = {out, q, k_arena, v_arena, block_tables, max_blocks, cu_seqlens_q,
                    context_lens, num_seqs, layer, scale, lay, use_f64, seq_select,
                    token_seq, n_tokens, 0};
    atomic_init(&job.next, 0);
    if (num_threads <= 1) {
        attn_worker(&job);
    } else {
        pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)num_threads);
        int32_t started = 0;
        for (int32_t i = 0; i < num_threads; ++i) {
            if (pthread_create(&th[i], NULL, attn_worker, &job) == 0) ++started;
            else break;
        }
        if (started == 0) attn_worker(&job);
        for (int32_t i = 0; i < started; ++i) pthread_join(th[i], NULL);
        free(th);
    }
    free(token_seq);
}
