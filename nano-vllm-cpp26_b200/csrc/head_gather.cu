// Head-parallel model layers (tensor parallelism over attention heads): after
// rank r has computed its heads' attention rows [rows, local_cols] (heads
// [r*Hl, (r+1)*Hl), head-major), every rank needs all heads for W_o
// (src/model.cpp:262-266 reads the full [T, H*hd] attention output). This is
// the gather, over NVLink by plain peer stores (no multicast):
//   outs[q][t * (world * local_cols) + r * local_cols + c] = local[t * local_cols + c]
// for every rank q, then a system-scope fence and one increment of every rank's
// flag; the call returns its stream after this rank's flag reached
// epoch * world (bounded wait, 2 s, then NVLLM_ERR_TIMEOUT), i.e. after every
// rank's rows have landed here.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "nvllm.h"
#include "nvllm_ops.h"

namespace nvllm {
namespace {

constexpr int kGatherRanks = NVLLM_MAX_RANKS;

struct GatherParams {
    const float* local;
    int64_t rows, local_cols, full_cols, col0;
    float* outs[kGatherRanks];
    int32_t world;
    int32_t vec;  // float4 stores (every row start 16-byte aligned)
};

__global__ void head_gather_kernel(const GatherParams p) {
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    if (p.vec) {
        const int64_t c4 = p.local_cols / 4;
        const int64_t total = p.rows * c4;
        for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
            const int64_t t = i / c4, c = (i - t * c4) * 4;
            const float4 v = *reinterpret_cast<const float4*>(p.local + t * p.local_cols + c);
            const int64_t o = t * p.full_cols + p.col0 + c;
            for (int r = 0; r < p.world; ++r) *reinterpret_cast<float4*>(p.outs[r] + o) = v;
        }
    } else {
        const int64_t total = p.rows * p.local_cols;
        for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
            const int64_t t = i / p.local_cols, c = i - t * p.local_cols;
            const float v = p.local[i];
            const int64_t o = t * p.full_cols + p.col0 + c;
            for (int r = 0; r < p.world; ++r) p.outs[r][o] = v;
        }
    }
    __threadfence_system();  // this thread's peer stores are visible before the signal
}

struct SignalParams {
    uint32_t* flags[kGatherRanks];
    int32_t world;
};

// After the gather kernel (stream order): one increment of every rank's flag.
__global__ void gather_signal_kernel(const SignalParams p) {
    if (threadIdx.x != 0) return;
    __threadfence_system();
    for (int r = 0; r < p.world; ++r) atomicAdd_system(p.flags[r], 1u);
}

__global__ void gather_wait_kernel(const uint32_t* flag, uint32_t target) {
    if (threadIdx.x != 0) return;
    const uint64_t t0 = global_ns();
    for (;;) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (int32_t(v - target) >= 0) return;
        if (global_ns() - t0 > kWaitLimitNs) {
            record_flag_timeout(kStatusInHeadGather, target, v);
            raise_status(kStatusTimeout | kStatusInHeadGather);
            return;
        }
        __nanosleep(200);
    }
}

int sm_count() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    return sms;
}

bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace
}  // namespace nvllm

using namespace nvllm;

extern "C" int nvllm_head_gather(const float* local, int64_t rows, int64_t local_cols,
                                 const nvllm_head_split* hs, void* stream) {
    if (hs == nullptr || hs->world < 1 || hs->world > NVLLM_MAX_RANKS || hs->rank < 0 ||
        hs->rank >= hs->world || hs->epoch == 0 || rows < 0 || local_cols <= 0) {
        return NVLLM_ERR_INVALID;
    }
    GatherParams p{};
    p.local = local;
    p.rows = rows;
    p.local_cols = local_cols;
    p.full_cols = local_cols * hs->world;
    p.col0 = local_cols * hs->rank;
    p.world = hs->world;
    bool vec = local_cols % 4 == 0 && aligned16(local);
    SignalParams sp{};
    sp.world = hs->world;
    for (int r = 0; r < hs->world; ++r) {
        if (hs->outs[r] == nullptr || hs->flags[r] == nullptr) return NVLLM_ERR_INVALID;
        p.outs[r] = hs->outs[r];
        sp.flags[r] = hs->flags[r];
        vec = vec && aligned16(hs->outs[r]);
    }
    if (rows > 0 && local == nullptr) return NVLLM_ERR_INVALID;
    p.vec = vec ? 1 : 0;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (rows > 0) {
        const int64_t work = rows * (vec ? local_cols / 4 : local_cols);
        const int64_t blocks =
            std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, int64_t(sm_count()) * 4));
        head_gather_kernel<<<unsigned(blocks), 256, 0, st>>>(p);
        if (cudaGetLastError() != cudaSuccess) return NVLLM_ERR_CUDA;
    }
    gather_signal_kernel<<<1, 32, 0, st>>>(sp);
    if (cudaGetLastError() != cudaSuccess) return NVLLM_ERR_CUDA;
    gather_wait_kernel<<<1, 32, 0, st>>>(hs->flags[hs->rank], hs->epoch * uint32_t(hs->world));
    return cudaGetLastError() == cudaSuccess ? NVLLM_OK : NVLLM_ERR_CUDA;
}
