/*
 * nvllm device ops (libnvllm.so): the rest of TransformerModel::forward_batch
 * around the paged-attention path (src/model.cpp:64-122, :161-187, :262-311),
 * for running the whole forward on the GPU. fp32 device pointers, asynchronous
 * on `stream` (a cudaStream_t), NVLLM_OK or an nvllm_status code.
 */
#ifndef NVLLM_OPS_H
#define NVLLM_OPS_H

#include <stddef.h>
#include <stdint.h>

#include "nvllm.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Weight initialisation of TransformerModel (src/model.cpp:71-112):
 * out[r * ld + c] (r < rows, c < cols) is draw number
 * stream_offset + r * cols + c of the model's 64-bit LCG (seed 0x5DEECE66D,
 * multiplier 6364136223846793005, increment 1), each draw
 * (float(state >> 33) / 2^32 - 0.5) * scale. Every lane jumps ahead in the
 * LCG, so the fill is parallel and bit-identical to the sequential loop. */
int nvllm_lcg_fill(float* out, int64_t rows, int64_t cols, int64_t ld, uint64_t stream_offset,
                   float scale, void* stream);

/* out[c * rows + r] = in[r * cols + c]: out = in^T for a rows x cols row-major
 * matrix (out of place). */
int nvllm_transpose(const float* in, int64_t rows, int64_t cols, float* out, void* stream);

/* out[t] = table[token_ids[t] % vocab] (src/model.cpp:161-166). */
int nvllm_embedding_gather(float* out, const float* table, const int32_t* token_ids, int64_t n,
                           int64_t vocab, int64_t dim, void* stream);

/* RMSNorm per row: out = x / sqrt(mean(x^2) + eps) * weight (weight NULL = 1),
 * src/model.cpp:20-38. out may alias in. */
int nvllm_rms_norm(float* out, const float* in, const float* weight, int64_t rows, int64_t dim,
                   float eps, void* stream);

/* x = x / (1 + exp(-x)) in place (src/model.cpp:271-273). */
int nvllm_silu(float* x, int64_t count, void* stream);

/* x += y (residual adds, src/model.cpp:264-266, :275-277). */
int nvllm_add(float* x, const float* y, int64_t count, void* stream);

/* out[i] = in[rows[i]] for i < count, in holding num_in_rows rows (last-token
 * gather, src/model.cpp:280-286); rows outside in raise NVLLM_ERR_BOUNDS. */
int nvllm_gather_rows(float* out, const float* in, const int32_t* rows, int64_t count,
                      int64_t num_in_rows, int64_t dim, void* stream);

/* Greedy sampling with the reference's repetition penalty
 * (src/model.cpp:293-309): sampled[r] = argmax_t (logits[r][t] - penalty if
 * t == prev_tokens[r]), lowest index on ties. Optional outputs (NULL to skip):
 * margin[r] = top-1 minus top-2 of those penalised values; top_idx / top_val
 * [rows, top_k] = the top_k largest raw logits, descending (top_k <= 32). */
int nvllm_penalized_argmax(const float* logits, const int64_t* prev_tokens, int64_t rows,
                           int64_t vocab, float penalty, int32_t* sampled, float* margin,
                           int32_t* top_idx, float* top_val, int32_t top_k, void* stream);

/* Dense fp32 GEMM on the tcgen05 tensor cores (3xTF32: W_hi X_hi + W_lo X_hi +
 * W_hi X_lo, fp32 quality) for the projections of src/model.cpp:42-62:
 *   C[t, c] = epi(sum_k x[t * lda + k] * wt[c * k + k'])   t < m, c < n
 * i.e. x [m, k] row-major (row stride lda) times W = wt^T, with the weights
 * stored transposed (wt [n, k] row-major). Column c of the product goes to
 * outs[c / out_block][t * ldc + c % out_block] (n_outs = n / out_block <= 3:
 * one output, or the Q/K/V split). n and out_block multiples of 128, k of 32,
 * lda of 4; x and wt 16-byte aligned. When fewer output tiles than SMs exist
 * (small m) K is split over CTAs and the partials, kept in `workspace`
 * (nvllm_gemm_workspace_size bytes), are summed in a fixed order. The products
 * accumulate on the tensor core in chunks of 128 of K, which are summed in fp32
 * registers with round-to-nearest adds. */
enum nvllm_gemm_epilogue {
    NVLLM_GEMM_STORE = 0,      /* C = product */
    NVLLM_GEMM_ACCUMULATE = 1, /* C += product (the residual adds) */
    NVLLM_GEMM_SILU = 2        /* C = silu(product) (the FFN up projection) */
};
size_t nvllm_gemm_workspace_size(int64_t m, int64_t n, int64_t k);
/* wt_lo NULL: wt holds W^T and every tile is split on chip; else wt = W_hi^T and
 * wt_lo = W_lo^T as written by nvllm_tf32_split (static weights split once). */
int nvllm_gemm_tf32x3(const float* x, int64_t lda, int64_t m, int64_t k, const float* wt,
                      const float* wt_lo, int64_t n, float* const* outs, int32_t n_outs,
                      int64_t out_block, int64_t ldc, int32_t epilogue, void* workspace,
                      size_t workspace_bytes, void* stream);
/* hi[i] = in[i] rounded to tf32 (nearest, in an fp32 container), lo[i] = in[i] - hi[i]
 * (exact): the operand parts of nvllm_gemm_tf32x3. */
int nvllm_tf32_split(const float* in, float* hi, float* lo, int64_t count, void* stream);

/* Dense fp32 GEMM (FFMA) for projections of few rows, the decode steps of
 * src/model.cpp:42-62, with the weights in the reference's row-major layout:
 *   outs[b][t * ldc + c] = epi(sum_k x[t * lda + k] * w[b * w_batch_stride + k * ldw + c])
 * for t < m <= 256, c < n, b < batch <= 3 (Q, K and V from one launch). lda and
 * ldw multiples of 4, x and w 16-byte aligned; w_batch_stride >= k * ldw when
 * batch > 1. K is split over CTAs when the columns alone do not fill the GPU;
 * the partials, kept in `workspace` (nvllm_gemm_skinny_workspace_size bytes,
 * 16-byte aligned), are summed in a fixed order, so results are reproducible
 * run to run. */
size_t nvllm_gemm_skinny_workspace_size(int64_t m, int64_t n, int64_t k, int32_t batch);
int nvllm_gemm_skinny(const float* x, int64_t lda, int64_t m, int64_t k, const float* w,
                      int64_t ldw, int64_t n, int32_t batch, int64_t w_batch_stride,
                      float* const* outs, int64_t ldc, int32_t epilogue, void* workspace,
                      size_t workspace_bytes, void* stream);

/* The same product, arguments and rules as nvllm_gemm_skinny for m <= 32, on the
 * tcgen05 tensor cores in 3xTF32 (fp32 quality): W streamed from HBM once and
 * split into tf32 hi / lo parts on chip, accumulated in chunks of 128 of K that
 * are summed in fp32 registers. K is dealt to persistent CTAs in equal ranges
 * (stream-K); the pieces of output tiles that CTAs share, kept in `workspace`
 * (nvllm_gemm_decode_tc_workspace_size bytes), are summed in a fixed order. */
size_t nvllm_gemm_decode_tc_workspace_size(int64_t m, int64_t n, int64_t k, int32_t batch);
int nvllm_gemm_decode_tc(const float* x, int64_t lda, int64_t m, int64_t k, const float* w,
                         int64_t ldw, int64_t n, int32_t batch, int64_t w_batch_stride,
                         float* const* outs, int64_t ldc, int32_t epilogue, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Head-parallel layers: rank hs->rank's attention rows local [rows, local_cols]
 * (its heads, head-major) stored into every rank's full-width buffer
 * hs->outs[q] ([rows, world * local_cols], columns rank * local_cols + c) over
 * NVLink, then one increment of every rank's flag; the call returns its stream
 * once this rank's flag reached epoch * world (every rank's rows landed here;
 * bounded wait, 2 s, then NVLLM_ERR_TIMEOUT in nvllm_get_last_error). epoch
 * counts this group's calls from 1, flags start at 0; alternate two sets of
 * output buffers by epoch parity so that a rank never overwrites rows a slower
 * rank still reads. No counterpart in the reference (one CPU process). */
int nvllm_head_gather(const float* local, int64_t rows, int64_t local_cols,
                      const nvllm_head_split* hs, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* NVLLM_OPS_H */
