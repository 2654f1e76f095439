// Shared device helpers for the nvllm kernels (sm_100a).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace nvllm {

// Device status bits, OR-ed into g_status by any kernel; read and cleared by
// nvllm_get_last_error().
enum : uint32_t {
    kStatusBounds = 1u,    // block id / slot outside the arena (access skipped)
    kStatusTimeout = 2u,   // a bounded mbarrier wait gave up
    kStatusMetadata = 4u,  // cu_seqlens / context_lens inconsistent with the bounds
    // which kernel's wait gave up (with kStatusTimeout)
    kStatusInDecode = 1u << 8,
    kStatusInPrefillTc = 1u << 9,
    kStatusInGemmTf32x3 = 1u << 10,
    kStatusInGemmSkinny = 1u << 11,
    kStatusInGemmDecodeTc = 1u << 12,
    kStatusInPrefill = 1u << 13,
    kStatusInHeadGather = 1u << 14,
    kStatusInHeadSplit = 1u << 15,  // the head split's wait for every rank's rows
};

extern __device__ uint32_t g_status;
// Where the first bounded wait that gave up was: {site bits, where code (set by
// the kernel: role, barrier, unit), block index, raw mbarrier word}; word 0 is 0
// until then. Cleared with the status word.
extern __device__ uint32_t g_timeout_info[4];

__device__ __forceinline__ void raise_status(uint32_t bits) { atomicOr(&g_status, bits); }

__device__ __forceinline__ void record_timeout(uint32_t site, uint32_t where, const uint64_t* bar) {
    if (atomicCAS(&g_timeout_info[0], 0u, site | 1u) == 0u) {
        g_timeout_info[1] = where;
        g_timeout_info[2] = blockIdx.x;
        g_timeout_info[3] = static_cast<uint32_t>(*reinterpret_cast<const volatile uint64_t*>(bar));
        __threadfence();
    }
}

// The same record for a cross-GPU flag wait that gave up: the value awaited
// and the value last read instead of the mbarrier fields.
__device__ __forceinline__ void record_flag_timeout(uint32_t site, uint32_t target,
                                                    uint32_t seen) {
    if (atomicCAS(&g_timeout_info[0], 0u, site | 1u) == 0u) {
        g_timeout_info[1] = target;
        g_timeout_info[2] = blockIdx.x;
        g_timeout_info[3] = seen;
        __threadfence();
    }
}

// Geometry of the reference arena [num_blocks, L, B, H*hd] in floats.
struct ArenaGeom {
    int64_t num_blocks;
    int64_t row;          // H*hd   (stride_slot)
    int64_t layer_stride; // B*row  (stride_layer)
    int64_t block_stride; // L*B*row (stride_block)
    int32_t num_layers;
    int32_t block_size;
    int32_t num_heads;
    int32_t head_dim;
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier (CTA scope) -------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Makes mbarrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Longest a thread waits on one mbarrier phase before declaring it stuck:
// far beyond any DRAM / copy-engine latency, short enough that a broken
// launch ends by itself.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Bounded wait: returns false (and raises kStatusTimeout | site) if the phase
// does not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t site = 0) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > kWaitLimitNs) {
            raise_status(kStatusTimeout | site);
            return false;
        }
    }
}

// ---- bulk async copy global -> shared (TMA, no multicast) -----------------
// dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// L2 policy for data read exactly once per call (the KV stream).
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ float4 ld_shared4(const float* p) {
    return *reinterpret_cast<const float4*>(p);
}

__device__ __forceinline__ float warp_max_xor(float v, int lanes) {
    for (int o = 1; o < lanes; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum_xor(float v, int lanes) {
    for (int o = 1; o < lanes; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

constexpr float kLog2e = 1.4426950408889634f;

// Programmatic dependent launch. A kernel launched with
// launch_programmatic() may start while the kernel before it in the stream
// is still running: it calls pdl_wait() before its first access to memory
// that kernel may write (which returns at once when the predecessor was not a
// kernel), and pdl_release() to let its own successor start early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_programmatic(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

}  // namespace nvllm
