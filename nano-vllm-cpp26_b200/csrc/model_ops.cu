// Device ops for the rest of TransformerModel::forward_batch around the paged
// attention path (src/model.cpp:64-122, :161-187, :262-311): the model's LCG
// weight fill, embedding / row gathers, RMSNorm, SiLU, residual add and the
// repetition-penalised greedy sampler. The projections themselves are fp32
// GEMMs issued by the host model (host/model.cpp).
//
// All of these are HBM-bound elementwise or row passes: 128-bit accesses where
// the row length allows, one CTA per row for the row-wise ops, grid-stride
// loops sized to the SM count for the elementwise ones.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "nvllm.h"
#include "nvllm_ops.h"
#include "common.cuh"

namespace nvllm {
namespace {

constexpr int kRowThreads = 256;

int launch_status() {
    return cudaGetLastError() == cudaSuccess ? NVLLM_OK : NVLLM_ERR_CUDA;
}

// 128-bit accesses only where every row start is 16-byte aligned.
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int grid_for(int64_t work_items, int threads) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    const int64_t need = (work_items + threads - 1) / threads;
    const int64_t cap = int64_t(sms) * 8;
    return int(need < 1 ? 1 : (need < cap ? need : cap));
}

// ---- LCG weight fill (src/model.cpp:71-79) ----------------------------------
// The model draws from state' = state * kMul + 1 (mod 2^64), seed kSeed, and
// uses state' >> 33 of each draw. Applying the affine map n times is again an
// affine map (A_n, C_n); composing maps by squaring lets every lane jump to its
// own draw index in 64 steps and then advance by the warp's 32-draw map.
constexpr uint64_t kSeed = 0x5DEECE66Dull;
constexpr uint64_t kMul = 6364136223846793005ull;

struct Affine {
    uint64_t a, c;  // x -> a * x + c
};

__device__ __forceinline__ Affine compose(Affine first, Affine then) {
    // then(first(x)) = then.a * (first.a * x + first.c) + then.c
    return Affine{then.a * first.a, then.a * first.c + then.c};
}

__device__ Affine affine_pow(uint64_t n) {
    Affine result{1ull, 0ull};
    Affine base{kMul, 1ull};
    while (n != 0) {
        if (n & 1ull) result = compose(result, base);
        base = compose(base, base);
        n >>= 1;
    }
    return result;
}

__device__ __forceinline__ float lcg_value(uint64_t state, float scale) {
    // (float(state >> 33) / float(0xFFFFFFFF) - 0.5f) * scale, where
    // float(0xFFFFFFFF) rounds to 2^32 (src/model.cpp:74-77)
    const float unit = (static_cast<float>(state >> 33) / 4294967296.0f) - 0.5f;
    return unit * scale;
}

// out[r * ld + c] = draw number (offset + r * cols + c), for r < rows, c < cols.
// Each warp owns runs of 32 consecutive draws per step of its loop.
__global__ void lcg_fill_kernel(float* __restrict__ out, int64_t rows, int64_t cols, int64_t ld,
                                uint64_t offset, float scale) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    const int64_t count = rows * cols;
    // each warp handles a contiguous span of whole 32-draw groups
    const int64_t groups = (count + 31) / 32;
    const int64_t per_warp = (groups + nwarps - 1) / nwarps;
    const int64_t g0 = warp * per_warp;
    const int64_t g1 = g0 + per_warp < groups ? g0 + per_warp : groups;
    if (g0 >= g1) return;
    int64_t i = g0 * 32 + lane;
    // state after draw (offset + i): the map applied (offset + i + 1) times
    const Affine jump = affine_pow(offset + uint64_t(i) + 1ull);
    uint64_t state = jump.a * kSeed + jump.c;
    const Affine step32 = affine_pow(32);
    int64_t r = i / cols, c = i - r * cols;
    for (int64_t g = g0; g < g1; ++g) {
        if (i < count) out[r * ld + c] = lcg_value(state, scale);
        state = step32.a * state + step32.c;
        i += 32;
        c += 32;
        while (c >= cols) {
            c -= cols;
            ++r;
        }
    }
}

// ---- row gathers (src/model.cpp:161-166, :280-286) ---------------------------
__global__ void gather_rows_kernel(float* __restrict__ out, const float* __restrict__ in,
                                   const int32_t* __restrict__ idx, int64_t dim, int64_t modulo,
                                   int64_t num_in_rows, bool vec) {
    const int64_t t = blockIdx.x;
    int64_t src = idx[t];
    if (modulo > 0) src = ((src % modulo) + modulo) % modulo;
    if (src < 0 || src >= num_in_rows) {
        raise_status(kStatusBounds);
        return;
    }
    const float* s = in + src * dim;
    float* d = out + t * dim;
    if (vec) {
        const float4* s4 = reinterpret_cast<const float4*>(s);
        float4* d4 = reinterpret_cast<float4*>(d);
        for (int64_t i = threadIdx.x; i < dim / 4; i += blockDim.x) d4[i] = s4[i];
    } else {
        for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) d[i] = s[i];
    }
}

// ---- RMSNorm (src/model.cpp:20-38) -------------------------------------------
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum_xor(v, 32);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    v = lane < nw ? red[lane] : 0.0f;
    v = warp_sum_xor(v, 32);
    __syncthreads();
    return v;
}

__global__ void rms_norm_kernel(float* out, const float* in, const float* __restrict__ weight,
                                int64_t dim, float eps, bool vec) {
    __shared__ float red[32];
    const float* x = in + int64_t(blockIdx.x) * dim;
    float* y = out + int64_t(blockIdx.x) * dim;
    float ss = 0.0f;
    if (vec) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
        for (int64_t i = threadIdx.x; i < dim / 4; i += blockDim.x) {
            const float4 v = x4[i];
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    } else {
        for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) ss += x[i] * x[i];
    }
    ss = block_sum(ss, red);
    const float inv_rms = 1.0f / sqrtf(ss / static_cast<float>(dim) + eps);
    if (vec) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
        float4* y4 = reinterpret_cast<float4*>(y);
        for (int64_t i = threadIdx.x; i < dim / 4; i += blockDim.x) {
            float4 v = x4[i];
            float4 w = weight ? reinterpret_cast<const float4*>(weight)[i]
                              : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
            v.x = v.x * inv_rms * w.x;
            v.y = v.y * inv_rms * w.y;
            v.z = v.z * inv_rms * w.z;
            v.w = v.w * inv_rms * w.w;
            y4[i] = v;
        }
    } else {
        for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
            y[i] = x[i] * inv_rms * (weight ? weight[i] : 1.0f);
        }
    }
}

// ---- SiLU and residual add (src/model.cpp:264-277) ---------------------------
__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

__global__ void silu_kernel(float* x, int64_t count, bool vec) {
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    const int64_t n4 = vec ? count / 4 : 0;
    float4* x4 = reinterpret_cast<float4*>(x);
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 v = x4[i];
        v.x = silu(v.x);
        v.y = silu(v.y);
        v.z = silu(v.z);
        v.w = silu(v.w);
        x4[i] = v;
    }
    for (int64_t i = n4 * 4 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
        x[i] = silu(x[i]);
    }
}

__global__ void add_kernel(float* x, const float* y, int64_t count, bool vec) {
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    const int64_t n4 = vec ? count / 4 : 0;
    float4* x4 = reinterpret_cast<float4*>(x);
    const float4* y4 = reinterpret_cast<const float4*>(y);
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 a = x4[i];
        const float4 b = y4[i];
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
        x4[i] = a;
    }
    for (int64_t i = n4 * 4 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
        x[i] += y[i];
    }
}

// ---- penalised greedy sampling (src/model.cpp:293-309) -----------------------
// (value, index) with the reference's preference: larger value, then lower
// index (its scan keeps the first strict maximum).
struct Best {
    float v;
    int32_t i;
};

__device__ __forceinline__ bool better(Best a, Best b) {
    return a.v > b.v || (a.v == b.v && a.i < b.i);
}

__device__ __forceinline__ Best warp_best(Best b) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Best other{__shfl_xor_sync(0xffffffffu, b.v, o), __shfl_xor_sync(0xffffffffu, b.i, o)};
        if (better(other, b)) b = other;
    }
    return b;
}

__device__ Best block_best(Best b, Best* red) {
    b = warp_best(b);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = b;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    b = lane < nw ? red[lane] : Best{-INFINITY, INT32_MAX};
    b = warp_best(b);
    __syncthreads();
    return b;
}

// One CTA per row. Pass 1: best and second-best penalised value (sampled id,
// margin). Passes 2..: the top_k raw logits by repeated exclusion of the ones
// already taken (only when asked for; a verification aid).
__global__ void penalized_argmax_kernel(const float* __restrict__ logits,
                                        const int64_t* __restrict__ prev, int64_t vocab,
                                        float penalty, int32_t* sampled, float* margin,
                                        int32_t* top_idx, float* top_val, int32_t top_k) {
    __shared__ Best red[32];
    __shared__ int32_t taken[32];
    __shared__ float taken_v[32];
    const int64_t row = blockIdx.x;
    const float* x = logits + row * vocab;
    const int64_t p = prev[row];
    Best b1{-INFINITY, INT32_MAX};
    float second = -INFINITY;
    for (int64_t t = threadIdx.x; t < vocab; t += blockDim.x) {
        const float v = t == p ? x[t] - penalty : x[t];
        const Best c{v, int32_t(t)};
        if (better(c, b1)) {
            second = fmaxf(second, b1.v);
            b1 = c;
        } else {
            second = fmaxf(second, v);
        }
    }
    const Best top = block_best(b1, red);
    // second-best penalised value: the largest value left once the winning
    // element (and only it) is removed
    const float cand = (b1.i == top.i) ? second : b1.v;
    const float sec = block_best(Best{cand, 0}, red).v;
    if (threadIdx.x == 0) {
        sampled[row] = top.i;
        if (margin) margin[row] = top.v - sec;
    }
    if (top_idx == nullptr || top_k <= 0) return;
    for (int k = 0; k < top_k; ++k) {
        Best m{-INFINITY, INT32_MAX};
        for (int64_t t = threadIdx.x; t < vocab; t += blockDim.x) {
            bool skip = false;
            for (int j = 0; j < k; ++j) skip |= taken[j] == int32_t(t);
            if (skip) continue;
            const Best c{x[t], int32_t(t)};
            if (better(c, m)) m = c;
        }
        m = block_best(m, red);
        if (threadIdx.x == 0) {
            taken[k] = m.i;
            taken_v[k] = m.v;
        }
        __syncthreads();
    }
    if (threadIdx.x < top_k) {
        top_idx[row * top_k + threadIdx.x] = taken[threadIdx.x];
        top_val[row * top_k + threadIdx.x] = taken_v[threadIdx.x];
    }
}

// out[c * rows + r] = in[r * cols + c]: 32 x 32 tiles through shared memory
// (padded rows: no bank conflicts), coalesced on both sides.
__global__ void transpose_kernel(const float* __restrict__ in, float* __restrict__ out,
                                 int64_t rows, int64_t cols) {
    __shared__ float tile[32][33];
    const int64_t r0 = int64_t(blockIdx.y) * 32, c0 = int64_t(blockIdx.x) * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[i][threadIdx.x] = in[r * cols + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) out[c * rows + r] = tile[threadIdx.x][i];
    }
}

}  // namespace
}  // namespace nvllm

using namespace nvllm;

extern "C" {

int nvllm_lcg_fill(float* out, int64_t rows, int64_t cols, int64_t ld, uint64_t stream_offset,
                   float scale, void* stream) {
    if (rows < 0 || cols < 0 || ld < cols || (out == nullptr && rows * cols > 0)) {
        return NVLLM_ERR_INVALID;
    }
    if (rows * cols == 0) return NVLLM_OK;
    const int threads = 256;
    const int64_t groups = (rows * cols + 31) / 32;
    lcg_fill_kernel<<<grid_for(groups * 32, threads), threads, 0,
                      static_cast<cudaStream_t>(stream)>>>(out, rows, cols, ld, stream_offset,
                                                           scale);
    return launch_status();
}

int nvllm_transpose(const float* in, int64_t rows, int64_t cols, float* out, void* stream) {
    if (rows < 0 || cols < 0 || rows > (int64_t(1) << 36) / 32 || cols > (int64_t(1) << 36) / 32) {
        return NVLLM_ERR_INVALID;
    }
    if (rows == 0 || cols == 0) return NVLLM_OK;
    if (!in || !out || in == out) return NVLLM_ERR_INVALID;
    const int64_t gy = (rows + 31) / 32, gx = (cols + 31) / 32;
    if (gy > 65535 || gx > 2147483647) return NVLLM_ERR_INVALID;
    transpose_kernel<<<dim3(unsigned(gx), unsigned(gy)), dim3(32, 8), 0,
                       static_cast<cudaStream_t>(stream)>>>(in, out, rows, cols);
    return launch_status();
}

int nvllm_embedding_gather(float* out, const float* table, const int32_t* token_ids, int64_t n,
                           int64_t vocab, int64_t dim, void* stream) {
    if (n < 0 || vocab <= 0 || dim <= 0) return NVLLM_ERR_INVALID;
    if (n == 0) return NVLLM_OK;
    if (!out || !table || !token_ids) return NVLLM_ERR_INVALID;
    gather_rows_kernel<<<unsigned(n), kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        out, table, token_ids, dim, vocab, vocab,
        (dim & 3) == 0 && aligned16(out) && aligned16(table));
    return launch_status();
}

int nvllm_gather_rows(float* out, const float* in, const int32_t* rows, int64_t count,
                      int64_t num_in_rows, int64_t dim, void* stream) {
    if (count < 0 || dim <= 0 || num_in_rows < 0) return NVLLM_ERR_INVALID;
    if (count == 0) return NVLLM_OK;
    if (!out || !in || !rows) return NVLLM_ERR_INVALID;
    gather_rows_kernel<<<unsigned(count), kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        out, in, rows, dim, 0, num_in_rows, (dim & 3) == 0 && aligned16(out) && aligned16(in));
    return launch_status();
}

int nvllm_rms_norm(float* out, const float* in, const float* weight, int64_t rows, int64_t dim,
                   float eps, void* stream) {
    if (rows < 0 || dim <= 0) return NVLLM_ERR_INVALID;
    if (rows == 0) return NVLLM_OK;
    if (!out || !in) return NVLLM_ERR_INVALID;
    rms_norm_kernel<<<unsigned(rows), kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        out, in, weight, dim, eps,
        (dim & 3) == 0 && aligned16(out) && aligned16(in) && (weight == nullptr || aligned16(weight)));
    return launch_status();
}

int nvllm_silu(float* x, int64_t count, void* stream) {
    if (count < 0) return NVLLM_ERR_INVALID;
    if (count == 0) return NVLLM_OK;
    if (!x) return NVLLM_ERR_INVALID;
    silu_kernel<<<grid_for((count + 3) / 4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, count, aligned16(x));
    return launch_status();
}

int nvllm_add(float* x, const float* y, int64_t count, void* stream) {
    if (count < 0) return NVLLM_ERR_INVALID;
    if (count == 0) return NVLLM_OK;
    if (!x || !y) return NVLLM_ERR_INVALID;
    add_kernel<<<grid_for((count + 3) / 4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, y, count, aligned16(x) && aligned16(y));
    return launch_status();
}

int nvllm_penalized_argmax(const float* logits, const int64_t* prev_tokens, int64_t rows,
                           int64_t vocab, float penalty, int32_t* sampled, float* margin,
                           int32_t* top_idx, float* top_val, int32_t top_k, void* stream) {
    if (rows < 0 || vocab <= 0 || vocab > INT32_MAX || top_k < 0 || top_k > 32) {
        return NVLLM_ERR_INVALID;
    }
    if (rows == 0) return NVLLM_OK;
    if (!logits || !prev_tokens || !sampled || (top_k > 0 && (!top_idx || !top_val))) {
        return NVLLM_ERR_INVALID;
    }
    penalized_argmax_kernel<<<unsigned(rows), kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        logits, prev_tokens, vocab, penalty, sampled, margin, top_idx, top_val, top_k);
    return launch_status();
}

}  // extern "C"
