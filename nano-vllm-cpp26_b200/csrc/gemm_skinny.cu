// fp32 GEMM for projections of few rows (decode steps: one row per running
// sequence), src/model.cpp:42-62 at small m:
//
//   C_b[t, c] = epi( sum_k X[t, k] * W_b[k, c] )    X [m, k], W_b [k, n] row-major
//
// With m <= 32 a weight element is used at most 32 times, so the product is a
// stream of W from HBM (about 8 FMAs per byte at m = 32, a little above what
// the FP32 pipes do per byte of HBM bandwidth). The kernel therefore keeps
// many weight bytes in flight: one thread moves 32-row x 128-column tiles of W
// and the matching 32-column slice of X into a 4-stage shared-memory ring with
// TMA (cp.async.bulk.tensor, no multicast), and the CTA's four warps take
// 8 of the 32 rows each, every lane 4 adjacent columns for all the CTA's rows
// of X (4 * MP fp32 accumulators; above 16 rows two warps per K slice take
// half of the rows each). The K slices' partial sums meet in shared
// memory in a fixed order; K is split over CTAs when the column blocks alone
// do not fill the GPU, and the splits are summed in a fixed order by a second
// kernel, so the result does not depend on scheduling. m > 32 runs in row
// groups of at most 32 rows, the groups of one column block adjacent in the
// grid so that the W tile they share is read from L2. The epilogue is that of
// the projection (store, residual add, SiLU), and up to three weight matrices
// with their own outputs run in one launch (Q, K, V).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "nvllm.h"
#include "nvllm_ops.h"

namespace nvllm {
namespace {

constexpr int kCols = 128;          // columns of W per CTA (32 lanes x 4)
constexpr int kStageK = 32;         // rows of W per stage
constexpr int kStages = 4;
constexpr int kKWarps = 4;          // warps over K: each takes kStageK / 4 rows of a stage
constexpr int kRowsPerWarp = kStageK / kKWarps;
constexpr int kMaxBatch = 3;
constexpr int kMaxRows = 256;       // 8 row groups of 32
constexpr int kWBytes = kStageK * kCols * 4;  // one W tile: 16 KB

struct SkinnyParams {
    int64_t m, n, k, ldc;
    float* outs[kMaxBatch];
    float* partial;  // [batch, splits, m, n] when splits > 1
    int32_t epilogue, splits, stages_per_split, row_groups, rows_per_group;
};

struct Control {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    int32_t abort;
};

// MP rows of X per CTA; above 16 rows two warps share each K slice, one half of
// the rows each (MR rows: 4 * MR accumulators a thread).
template <int MP>
struct Layout {
    static constexpr int kRowSplit = MP > 16 ? 2 : 1;
    static constexpr int MR = MP / kRowSplit;
    static constexpr int kWarps = kKWarps * kRowSplit;
    static constexpr int kThreads = 32 * kWarps;
    static constexpr int kXBytes = MP * kStageK * 4;  // one X tile: MP rows x 32 columns
    static constexpr int kRing = kStages * (kWBytes + kXBytes);
    static constexpr int kReduce = kKWarps * MP * kCols * 4;
    static constexpr int kData = kRing > kReduce ? kRing : kReduce;
    static constexpr int kSmem = kData + 128 + 128;  // + control block + alignment slack
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, Control* ctl) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*reinterpret_cast<volatile int32_t*>(&ctl->abort)) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            raise_status(kStatusTimeout | kStatusInGemmSkinny);
            atomicExch(&ctl->abort, 1);
            return false;
        }
    }
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

__device__ __forceinline__ void fma4(float4& a, float s, const float4& w) {
    a.x = fmaf(s, w.x, a.x);
    a.y = fmaf(s, w.y, a.y);
    a.z = fmaf(s, w.z, a.z);
    a.w = fmaf(s, w.w, a.w);
}

__device__ __forceinline__ void apply(float* o, float v, int32_t epilogue) {
    if (epilogue == NVLLM_GEMM_STORE) {
        *o = v;
    } else if (epilogue == NVLLM_GEMM_ACCUMULATE) {
        *o += v;
    } else {
        *o = silu(v);
    }
}

__device__ __forceinline__ unsigned char* align128(unsigned char* p) {
    return reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 127) & ~uintptr_t(127));
}

// grid: (column blocks x row groups, splits, batch); MP = rows of a row group.
// Three CTAs share an SM up to 16 rows (the ring's shared memory), two above.
template <int MP>
__global__ void __launch_bounds__(Layout<MP>::kThreads, MP <= 16 ? 3 : 2)
    skinny_kernel(const SkinnyParams p, const __grid_constant__ CUtensorMap wmap,
                  const __grid_constant__ CUtensorMap xmap) {
    using Ly = Layout<MP>;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = align128(smem_raw);
    float* wring = reinterpret_cast<float*>(smem);                      // [stage][32][128]
    float* xring = reinterpret_cast<float*>(smem + kStages * kWBytes);  // [stage][MP][32]
    Control* ctl = reinterpret_cast<Control*>(smem + Ly::kData);
    const int warp = int(threadIdx.x) / 32, lane = int(threadIdx.x) % 32;
    const int kw = warp % kKWarps;           // K slice of a stage
    const int rw = warp / kKWarps;           // row half (rows rw * MR ..)
    constexpr int MR = Ly::MR;
    const int rg = int(blockIdx.x) % p.row_groups;
    const int c0 = (int(blockIdx.x) / p.row_groups) * kCols;
    const int split = int(blockIdx.y), b = int(blockIdx.z);
    const int r0 = rg * MP;
    const int rows = min(MP, int(p.m) - r0);
    const int s0 = split * p.stages_per_split;
    const int nst = min(p.stages_per_split, int((p.k + kStageK - 1) / kStageK) - s0);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&ctl->full[i], 1);
            mbar_init(&ctl->empty[i], Ly::kWarps);
        }
        ctl->abort = 0;
    }
    fence_barrier_init();
    __syncthreads();

    float4 acc[MR];
#pragma unroll
    for (int t = 0; t < MR; ++t) acc[t] = make_float4(0.f, 0.f, 0.f, 0.f);

    // Lane 0 of warp 0 issues the copies: the first kStages stages up front, then
    // the refill of a slot once every warp has released it.
    const bool issuer = threadIdx.x == 0;
    int issued = 0;
    auto issue = [&](int g) {
        const int slot = g % kStages;
        mbar_arrive_expect_tx(&ctl->full[slot], uint32_t(kWBytes + Ly::kXBytes));
        const int kr = (s0 + g) * kStageK;
        tma_load_3d(wring + slot * (kStageK * kCols), &wmap, c0, kr, b, &ctl->full[slot]);
        tma_load_2d(xring + slot * (MP * kStageK), &xmap, kr, r0, &ctl->full[slot]);
        issued = g + 1;
    };
    if (issuer) {
        for (int g = 0; g < min(nst, kStages); ++g) issue(g);
    }
#pragma unroll 1
    for (int g = 0; g < nst; ++g) {
        const int slot = g % kStages;
        if (!wait_or_abort(&ctl->full[slot], uint32_t(g / kStages) & 1u, ctl)) break;
        const float* wt = wring + slot * (kStageK * kCols) + kw * kRowsPerWarp * kCols + lane * 4;
        const float* xt = xring + slot * (MP * kStageK) + rw * MR * kStageK + kw * kRowsPerWarp;
        // two halves of 4 rows: 16 registers of W live next to the 4 * MR sums
#pragma unroll
        for (int h = 0; h < kRowsPerWarp; h += 4) {
            const float4 w0 = ld_shared4(wt + (h + 0) * kCols);
            const float4 w1 = ld_shared4(wt + (h + 1) * kCols);
            const float4 w2 = ld_shared4(wt + (h + 2) * kCols);
            const float4 w3 = ld_shared4(wt + (h + 3) * kCols);
#pragma unroll
            for (int t = 0; t < MR; ++t) {
                const float4 xv = ld_shared4(xt + t * kStageK + h);
                fma4(acc[t], xv.x, w0);
                fma4(acc[t], xv.y, w1);
                fma4(acc[t], xv.z, w2);
                fma4(acc[t], xv.w, w3);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->empty[slot]);
        if (issuer && g + kStages < nst) {
            if (!wait_or_abort(&ctl->empty[slot], uint32_t(g / kStages) & 1u, ctl)) break;
            issue(g + kStages);
        }
    }
    // copies still in flight (only after an abort) land before the CTA ends
    if (issuer) {
        for (int h = max(0, issued - kStages); h < issued; ++h) {
            mbar_wait(&ctl->full[h % kStages], uint32_t(h / kStages) & 1u, kStatusInGemmSkinny);
        }
    }
    __syncthreads();
    if (*reinterpret_cast<volatile int32_t*>(&ctl->abort)) return;

    // the K slices' sums, over the (now idle) ring: red[K slice][row][column]
    float* red = reinterpret_cast<float*>(smem);
    float* const out = b == 0 ? p.outs[0] : (b == 1 ? p.outs[1] : p.outs[2]);
#pragma unroll
    for (int t = 0; t < MR; ++t) {
        *reinterpret_cast<float4*>(red + (kw * MP + rw * MR + t) * kCols + lane * 4) = acc[t];
    }
    __syncthreads();
    for (int e = int(threadIdx.x); e < rows * kCols; e += Ly::kThreads) {
        const int t = e / kCols, c = e - t * kCols;
        const int64_t col = int64_t(c0) + c;
        if (col >= p.n) continue;
        float v = red[t * kCols + c];
#pragma unroll
        for (int w = 1; w < kKWarps; ++w) v += red[(w * MP + t) * kCols + c];
        const int64_t row = int64_t(r0) + t;
        if (p.splits > 1) {
            p.partial[((int64_t(b) * p.splits + split) * p.m + row) * p.n + col] = v;
        } else {
            apply(out + row * p.ldc + col, v, p.epilogue);
        }
    }
}

// out_b = epi(sum of the splits' partials), the splits in a fixed order
__global__ void skinny_reduce_kernel(const SkinnyParams p, int32_t batch) {
    const int64_t per = p.m * p.n;
    const int64_t total = per * batch;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t b = i / per;
        const int64_t r = i - b * per;
        const float* src = p.partial + b * p.splits * per + r;
        float v = src[0];
        for (int s = 1; s < p.splits; ++s) v += src[int64_t(s) * per];
        const int64_t t = r / p.n, c = r - t * p.n;
        float* const out = b == 0 ? p.outs[0] : (b == 1 ? p.outs[1] : p.outs[2]);
        apply(out + t * p.ldc + c, v, p.epilogue);
    }
}

// ------------------------------------------------------------------ host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        }
    });
    return fn;
}

// W_b [k, n] (row stride ldw, matrix stride wbs floats) as {n, k, batch} in
// boxes of 128 columns x 32 rows; X [m, k] (row stride lda) as {k, m} in boxes
// of 32 columns x rows. No swizzle; reads past the ends are zero.
bool make_maps(CUtensorMap* wmap, CUtensorMap* xmap, const float* w, int64_t ldw, int64_t wbs,
               int64_t n, int64_t k, int32_t batch, const float* x, int64_t lda, int64_t m,
               int rows) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t wdims[3] = {cuuint64_t(n), cuuint64_t(k), cuuint64_t(batch)};
    const cuuint64_t wstr[2] = {cuuint64_t(ldw) * 4, cuuint64_t(wbs) * 4};
    const cuuint32_t wbox[3] = {uint32_t(kCols), uint32_t(kStageK), 1};
    const cuuint32_t e3[3] = {1, 1, 1};
    if (fn(wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(w), wdims, wstr, wbox, e3,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        return false;
    }
    const cuuint64_t xdims[2] = {cuuint64_t(k), cuuint64_t(m)};
    const cuuint64_t xstr[1] = {cuuint64_t(lda) * 4};
    const cuuint32_t xbox[2] = {uint32_t(kStageK), uint32_t(rows)};
    return fn(xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), xdims, xstr, xbox,
              e3, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    return sms;
}

template <int MP>
cudaError_t configure() {
    static bool done[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!done[dev]) {
        e = cudaFuncSetAttribute(skinny_kernel<MP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Layout<MP>::kSmem);
        if (e != cudaSuccess) return e;
        done[dev] = true;
    }
    return cudaSuccess;
}

// CTAs of skinny_kernel<MP> resident per SM (2 when the device cannot be asked)
template <int MP>
int resident() {
    int occ = 0;
    if (configure<MP>() != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, skinny_kernel<MP>, Layout<MP>::kThreads,
                                                      Layout<MP>::kSmem) != cudaSuccess ||
        occ < 1) {
        cudaGetLastError();
        return 2;
    }
    return occ;
}

int resident_for(int rows) {
    switch (rows) {
        case 4: return resident<4>();
        case 8: return resident<8>();
        case 12: return resident<12>();
        case 16: return resident<16>();
        case 20: return resident<20>();
        case 24: return resident<24>();
        case 28: return resident<28>();
        default: return resident<32>();
    }
}

struct Plan {
    int32_t row_groups, rows, splits, stages_per_split;
};

// Row groups of at most 32 rows (a multiple of 4), and the K split. A split
// count s costs ceil(CTAs / resident) waves of (stages per split + 2) stage
// times (the 2: pipeline fill and the epilogue), plus the partials' traffic
// (2 s m n floats written and read against k n of W); the cheapest s <= 16
// wins, the smaller one within 3 %.
Plan plan(int64_t m, int64_t n, int64_t k, int32_t batch) {
    Plan pl{};
    pl.row_groups = int32_t((m + 31) / 32);
    pl.rows = int32_t(((m + pl.row_groups - 1) / pl.row_groups + 3) / 4 * 4);
    const int64_t base = ((n + kCols - 1) / kCols) * pl.row_groups * batch;
    const int64_t wave = int64_t(sm_count()) * resident_for(pl.rows);
    const int64_t total = (k + kStageK - 1) / kStageK;
    const int64_t max_s = std::min<int64_t>(16, std::max<int64_t>(1, total / 4));  // >= 4 stages
    double best = 0.0;
    for (int64_t s = 1; s <= max_s; ++s) {
        const int64_t sps = (total + s - 1) / s;
        const int64_t se = (total + sps - 1) / sps;
        const int64_t waves = (base * se + wave - 1) / wave;
        const double traffic = se > 1 ? 1.0 + 2.0 * double(se) * double(m) / double(k) : 1.0;
        const double cost = double(waves) * double(sps + 2) * traffic;
        if (s == 1 || cost < best * 0.97) {
            best = cost;
            pl.stages_per_split = int32_t(sps);
            pl.splits = int32_t(se);
        }
    }
    return pl;
}

bool valid_shape(int64_t m, int64_t n, int64_t k, int32_t batch) {
    return m >= 0 && m <= kMaxRows && n > 0 && k > 0 && n < (int64_t(1) << 31) &&
           k < (int64_t(1) << 31) && batch >= 1 && batch <= kMaxBatch;
}

bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

template <int MP>
cudaError_t launch(const SkinnyParams& p, const CUtensorMap& wmap, const CUtensorMap& xmap,
                   int64_t col_blocks, int32_t batch, cudaStream_t st) {
    cudaError_t e = configure<MP>();
    if (e != cudaSuccess) return e;
    const dim3 grid(unsigned(col_blocks * p.row_groups), unsigned(p.splits), unsigned(batch));
    skinny_kernel<MP><<<grid, Layout<MP>::kThreads, Layout<MP>::kSmem, st>>>(p, wmap, xmap);
    return cudaGetLastError();
}

}  // namespace
}  // namespace nvllm

using namespace nvllm;

extern "C" {

size_t nvllm_gemm_skinny_workspace_size(int64_t m, int64_t n, int64_t k, int32_t batch) {
    if (!valid_shape(m, n, k, batch) || m == 0) return 0;
    const Plan pl = plan(m, n, k, batch);
    if (pl.splits <= 1) return 0;
    return size_t(batch) * size_t(pl.splits) * size_t(m) * size_t(n) * sizeof(float);
}

int nvllm_gemm_skinny(const float* x, int64_t lda, int64_t m, int64_t k, const float* w,
                      int64_t ldw, int64_t n, int32_t batch, int64_t w_batch_stride,
                      float* const* outs, int64_t ldc, int32_t epilogue, void* workspace,
                      size_t workspace_bytes, void* stream) {
    if (!valid_shape(m, n, k, batch) || lda < k || lda % 4 != 0 || ldw < n || ldw % 4 != 0 ||
        ldc < n || outs == nullptr || epilogue < NVLLM_GEMM_STORE || epilogue > NVLLM_GEMM_SILU ||
        (batch > 1 && (w_batch_stride < k * ldw || w_batch_stride % 4 != 0))) {
        return NVLLM_ERR_INVALID;
    }
    if (m == 0) return NVLLM_OK;
    if (x == nullptr || w == nullptr || !aligned16(x) || !aligned16(w)) return NVLLM_ERR_INVALID;
    SkinnyParams p{};
    p.m = m;
    p.n = n;
    p.k = k;
    p.ldc = ldc;
    p.epilogue = epilogue;
    for (int i = 0; i < batch; ++i) {
        if (outs[i] == nullptr) return NVLLM_ERR_INVALID;
        p.outs[i] = outs[i];
    }
    const Plan pl = plan(m, n, k, batch);
    p.row_groups = pl.row_groups;
    p.rows_per_group = pl.rows;
    p.splits = pl.splits;
    p.stages_per_split = pl.stages_per_split;
    if (p.splits > 1) {
        const size_t need = size_t(batch) * size_t(p.splits) * size_t(m) * size_t(n) * sizeof(float);
        if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)) {
            return NVLLM_ERR_WORKSPACE;
        }
        p.partial = static_cast<float*>(workspace);
    }
    CUtensorMap wmap, xmap;
    if (!make_maps(&wmap, &xmap, w, ldw, batch > 1 ? w_batch_stride : k * ldw, n, k, batch, x,
                   lda, m, pl.rows)) {
        return NVLLM_ERR_CUDA;
    }
    const int64_t col_blocks = (n + kCols - 1) / kCols;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    switch (pl.rows) {
        case 4: e = launch<4>(p, wmap, xmap, col_blocks, batch, st); break;
        case 8: e = launch<8>(p, wmap, xmap, col_blocks, batch, st); break;
        case 12: e = launch<12>(p, wmap, xmap, col_blocks, batch, st); break;
        case 16: e = launch<16>(p, wmap, xmap, col_blocks, batch, st); break;
        case 20: e = launch<20>(p, wmap, xmap, col_blocks, batch, st); break;
        case 24: e = launch<24>(p, wmap, xmap, col_blocks, batch, st); break;
        case 28: e = launch<28>(p, wmap, xmap, col_blocks, batch, st); break;
        default: e = launch<32>(p, wmap, xmap, col_blocks, batch, st); break;
    }
    if (e != cudaSuccess) return NVLLM_ERR_CUDA;
    if (p.splits > 1) {
        const int64_t work = m * n * batch;
        const int64_t blocks = std::min<int64_t>((work + 255) / 256, int64_t(sm_count()) * 8);
        skinny_reduce_kernel<<<unsigned(blocks), 256, 0, st>>>(p, batch);
        if (cudaGetLastError() != cudaSuccess) return NVLLM_ERR_CUDA;
    }
    return NVLLM_OK;
}

}  // extern "C"
