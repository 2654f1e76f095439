// K1: KV write of one layer for a flattened batch into the paged arenas.
//
// Replaces the loop at src/model.cpp:188-202 that calls PagedKVCache::write_kv
// (src/kv_cache.cpp:57-68) once per token. Each token's K and V rows
// ([H*hd] floats) move bit-exactly to arena row (slot / B, layer, slot % B).
// The copy is HBM-bound: 2 * 4 * H*hd bytes read and written per token.
#include "common.cuh"
#include "kernels.cuh"

namespace nvllm {

namespace {

// One CTA per token; float4 path when rows are 16-byte aligned.
template <bool kVec4>
__global__ void __launch_bounds__(256)
reshape_and_cache_kernel(const float* __restrict__ key, const float* __restrict__ value,
                         float* __restrict__ k_arena, float* __restrict__ v_arena,
                         const int32_t* __restrict__ slot_mapping, int32_t layer,
                         ArenaGeom g) {
    pdl_release();
    pdl_wait();  // the rows and the slot mapping may come from the kernel before
    const int64_t t = blockIdx.x;
    const int32_t slot = slot_mapping[t];
    if (slot < 0) return;
    const int64_t blk = slot / g.block_size;
    if (blk >= g.num_blocks) {
        if (threadIdx.x == 0) raise_status(kStatusBounds);
        return;
    }
    const int64_t base = blk * g.block_stride + layer * g.layer_stride +
                         static_cast<int64_t>(slot % g.block_size) * g.row;
    const float* ks = key + t * g.row;
    const float* vs = value + t * g.row;
    float* kd = k_arena + base;
    float* vd = v_arena + base;
    if constexpr (kVec4) {
        const int64_t n4 = g.row / 4;
        for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) {
            const float4 kv = __ldcs(reinterpret_cast<const float4*>(ks) + i);
            const float4 vv = __ldcs(reinterpret_cast<const float4*>(vs) + i);
            reinterpret_cast<float4*>(kd)[i] = kv;
            reinterpret_cast<float4*>(vd)[i] = vv;
        }
    } else {
        for (int64_t i = threadIdx.x; i < g.row; i += blockDim.x) {
            kd[i] = ks[i];
            vd[i] = vs[i];
        }
    }
}

}  // namespace

cudaError_t launch_reshape_and_cache(const float* key, const float* value, float* k_arena,
                                     float* v_arena, const int32_t* slot_mapping,
                                     int64_t num_tokens, int32_t layer, const ArenaGeom& g,
                                     bool vec4, cudaStream_t stream) {
    if (num_tokens <= 0) return cudaSuccess;
    const dim3 grid(static_cast<unsigned>(num_tokens));
    const int threads = g.row >= 1024 ? 256 : 128;
    return launch_programmatic(vec4 ? reshape_and_cache_kernel<true> : reshape_and_cache_kernel<false>,
                               grid, dim3(threads), 0, stream, key, value, k_arena, v_arena,
                               slot_mapping, layer, g);
}

}  // namespace nvllm
