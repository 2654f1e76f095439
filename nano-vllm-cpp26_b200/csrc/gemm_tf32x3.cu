// Dense fp32 GEMM on the tcgen05 tensor cores (3xTF32) for the model's
// projections (src/model.cpp:42-62 matmul_batched, called at :184-186, :263,
// :270, :274, :291), with the elementwise work that follows a projection fused
// into its epilogue (residual add, SiLU, the Q/K/V split).
//
//   C[t, c] = epi( sum_k X[t, k] * W[k, c] )     X [m, k] row-major (activations)
//                                                Wt [n, k] row-major (W transposed)
//
// Weights are stored transposed so that both operands are K-major in shared
// memory. One CTA computes a 128 x BT tile: 128 output features (MMA M = TMEM
// lanes) by BT token rows (MMA N), D = Wt_tile . X_tile^T accumulated in TMEM
// in chunks of 128 of K: the tensor core's fp32 accumulation truncates, so a
// long sum in one accumulator drifts (measured: linear in the chunk length);
// the epilogue warps fold every chunk into fp32 registers with round-to-nearest
// adds while the MMAs fill the other of two TMEM accumulators.
// Every product is 3xTF32: hi = x rounded to tf32 (nearest), lo = x - hi, both
// exact in their fp32 containers (the tensor core reads a tf32 operand as the
// top 19 bits); W_hi X_hi + W_lo X_hi + W_hi X_lo then carries each product
// to ~2^-21 relative, the quality of an fp32 GEMM.
//
// 8 warps per CTA (persistent grid, tiles dealt round-robin):
//   warp 0     producer: TMA loads of the W and X tiles (32 columns of K per
//              stage, 128-byte swizzle, no multicast) and every tcgen05.mma;
//   warps 1-7  converters: round each landed tile to its hi part in place and
//              write its lo part (the X tile only when the weights come
//              pre-split as W_hi / W_lo); warps 4-7, one per TMEM lane quarter,
//              also fold each finished accumulation chunk into their fp32
//              registers (tcgen05.ld) and, at the end of a tile, apply the
//              epilogue op and store the output (or split-K partials, summed
//              by a second kernel in a fixed order, so results do not depend
//              on scheduling).
// Every wait is bounded; on a timeout the CTA records NVLLM_ERR_TIMEOUT, lets
// its copies and MMAs finish and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <initializer_list>
#include <mutex>

#include "nvllm.h"
#include "nvllm_ops.h"
#include "common.cuh"
#include "tcgen05.cuh"

namespace nvllm {
namespace {

constexpr int kBN = 128;  // output features per tile (MMA M, TMEM lanes)
constexpr int kBK = 32;   // K columns per stage (one 128-byte swizzle atom)
constexpr int kThreads = 288;      // producer, 7 converter warps, MMA issuer
constexpr int kConvThreads = 224;  // warps 1-7
constexpr int kEpiThreads = 128;   // warps 4-7 (also converters)
constexpr int kEpiWarp0 = 4;
constexpr int kMmaWarp = 8;
constexpr int kMaxSplits = 16;
constexpr int kMaxOuts = 3;
constexpr int kChunkSteps = 4;  // stages (of 32 K) per TMEM accumulation chunk

template <int BT>
struct Cfg {
    static constexpr int kStages = BT <= 32 ? 5 : 3;
    static constexpr uint32_t kABytes = kBN * 128;  // 128 rows x 32 fp32
    static constexpr uint32_t kBBytes = BT * 128;
    static constexpr uint32_t kStageBytes = 2 * kABytes + 2 * kBBytes;  // W, W_lo, X, X_lo
    static constexpr uint32_t kOffBar = kStages * kStageBytes;
    static constexpr uint32_t kSmem = kOffBar + 256 + 1024;
    // two accumulators of BT columns (MMA targets) and the fp32 sum of the tile's
    // folded chunks (BT columns)
    static constexpr uint32_t kColSum = 2 * BT;
    static constexpr uint32_t kTmemCols = BT <= 32 ? 128 : 512;
    static constexpr uint32_t kIdesc = tc::tf32_idesc(kBN, BT, false, false);
    static_assert(kSmem <= 227u * 1024u, "shared memory");
    static_assert(kTmemCols >= 3 * BT && (kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation");
};

struct GemmParams {
    int64_t m, n, k;
    int32_t n_tiles, t_tiles, splits, steps_per_split, total_steps;
    int64_t items;
    float* outs[kMaxOuts];
    int64_t out_block, ldc;
    int32_t epilogue;  // nvllm_gemm_epilogue
    int32_t w_split;   // the weights arrive as W_hi / W_lo (two tensor maps)
    float* partial;    // [splits, m, n] when splits > 1
};

struct Control {
    uint64_t kv_full[8];   // TMA landed (transaction bytes)
    uint64_t cv_full[8];   // lo parts written (kConvThreads arrivals)
    uint64_t st_free[8];   // the stage's MMAs completed
    uint64_t d_full[2];    // accumulator complete
    uint64_t d_free[2];    // accumulator read by the epilogue (kEpiThreads arrivals)
    uint64_t drain;
    uint32_t tmem_base;
    int32_t abort;
};
static_assert(sizeof(Control) <= 256, "control block");

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, Control* ctl) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*reinterpret_cast<volatile int32_t*>(&ctl->abort)) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            raise_status(kStatusTimeout | kStatusInGemmTf32x3);
            atomicExch(&ctl->abort, 1);
            return false;
        }
    }
}

// v -> (hi, lo): hi = v rounded to tf32 (to nearest), lo = v - hi (exact)
__device__ __forceinline__ void tf32_split4(float4 v, float4& hi, float4& lo) {
    hi = make_float4(tc::to_tf32(v.x), tc::to_tf32(v.y), tc::to_tf32(v.z), tc::to_tf32(v.w));
    lo = make_float4(v.x - hi.x, v.y - hi.y, v.z - hi.z, v.w - hi.w);
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// The item (tile, split) this CTA handles j-th, and its K range.
struct Item {
    int64_t n0, t0;
    int32_t split, step0, nsteps;
};

__device__ __forceinline__ Item item_of(const GemmParams& p, int64_t it, int BT) {
    Item r;
    const int64_t tt = it % p.t_tiles;
    const int64_t rest = it / p.t_tiles;
    r.n0 = (rest % p.n_tiles) * kBN;
    r.split = int32_t(rest / p.n_tiles);
    r.t0 = tt * BT;
    r.step0 = r.split * p.steps_per_split;
    r.nsteps = min(p.steps_per_split, p.total_steps - r.step0);
    return r;
}

template <int BT>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const GemmParams p, const __grid_constant__ CUtensorMap wmap,
            const __grid_constant__ CUtensorMap wlomap, const __grid_constant__ CUtensorMap xmap) {
    using C = Cfg<BT>;
    constexpr int S = C::kStages;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Control* ctl = reinterpret_cast<Control*>(base + C::kOffBar);
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    auto stage_ptr = [&](uint32_t g) { return base + (g % S) * C::kStageBytes; };

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&ctl->kv_full[i], 1);
            mbar_init(&ctl->cv_full[i], kConvThreads);
            mbar_init(&ctl->st_free[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&ctl->d_full[i], 1);
            mbar_init(&ctl->d_free[i], kEpiThreads);
        }
        mbar_init(&ctl->drain, 1);
        ctl->abort = 0;
    }
    fence_barrier_init();
    if (warp == 0) {
        tc::tmem_alloc(&ctl->tmem_base, C::kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------- producer (TMA copies)
        if (lane == 0) {
            uint32_t g = 0;  // steps loaded (ring slot g % S)
            bool ok = true;
            for (int64_t it = blockIdx.x; ok && it < p.items; it += gridDim.x) {
                const Item im = item_of(p, it, BT);
                for (int s = 0; s < im.nsteps; ++s, ++g) {
                    // the slot's previous step (g - S) has been read by its MMAs
                    if (g >= uint32_t(S) &&
                        !wait_or_abort(&ctl->st_free[g % S], ((g / S) - 1) & 1u, ctl)) {
                        ok = false;
                        break;
                    }
                    unsigned char* st = stage_ptr(g);
                    mbar_arrive_expect_tx(&ctl->kv_full[g % S],
                                          (p.w_split ? 2 : 1) * C::kABytes + C::kBBytes);
                    const int x = (im.step0 + s) * kBK;
                    tc::tma_load_2d(st, &wmap, x, int(im.n0), &ctl->kv_full[g % S]);
                    if (p.w_split) {
                        tc::tma_load_2d(st + C::kABytes, &wlomap, x, int(im.n0), &ctl->kv_full[g % S]);
                    }
                    tc::tma_load_2d(st + 2 * C::kABytes, &xmap, x, int(im.t0), &ctl->kv_full[g % S]);
                }
            }
            // copies in flight land before the CTA ends (bounded waits)
            for (uint32_t h = g > uint32_t(S) ? g - S : 0; h < g; ++h) {
                mbar_wait(&ctl->kv_full[h % S], (h / S) & 1u, kStatusInGemmTf32x3);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------------ MMAs
        if (lane == 0) {
            uint32_t g = 0, q = 0;  // steps issued, accumulation chunks issued
            bool ok = true, issued_mma = false;
            for (int64_t it = blockIdx.x; ok && it < p.items; it += gridDim.x) {
                const Item im = item_of(p, it, BT);
                for (int s = 0; s < im.nsteps; ++s, ++g) {
                    const uint32_t buf = q & 1u;
                    const bool chunk_first = s % kChunkSteps == 0;
                    const bool chunk_last = s % kChunkSteps == kChunkSteps - 1 || s + 1 == im.nsteps;
                    if (!wait_or_abort(&ctl->cv_full[g % S], (g / S) & 1u, ctl) ||
                        (chunk_first && q >= 2 &&
                         !wait_or_abort(&ctl->d_free[buf], ((q >> 1) - 1) & 1u, ctl))) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t a = smem_addr(stage_ptr(g));
                    const uint32_t alo = a + C::kABytes;
                    const uint32_t b = a + 2 * C::kABytes;
                    const uint32_t blo = b + C::kBBytes;
                    const uint32_t d = tmem + buf * uint32_t(BT);
#pragma unroll
                    for (int kk = 0; kk < kBK / 8; ++kk) {
                        const uint32_t off = uint32_t(kk) * 32u;  // 8 tf32 = 32 bytes
                        const uint64_t da = tc::sw128_desc(a + off, 16, 1024);
                        const uint64_t dalo = tc::sw128_desc(alo + off, 16, 1024);
                        const uint64_t db = tc::sw128_desc(b + off, 16, 1024);
                        const uint64_t dblo = tc::sw128_desc(blo + off, 16, 1024);
                        tc::mma_tf32(d, dalo, db, C::kIdesc, !chunk_first || kk > 0);
                        tc::mma_tf32(d, da, dblo, C::kIdesc, true);
                        tc::mma_tf32(d, da, db, C::kIdesc, true);
                    }
                    tc::commit(&ctl->st_free[g % S]);
                    if (chunk_last) {
                        tc::commit(&ctl->d_full[buf]);
                        ++q;
                    }
                    issued_mma = true;
                }
            }
            // issued MMAs complete before the TMEM is freed (bounded wait)
            if (issued_mma) {
                tc::commit(&ctl->drain);
                mbar_wait(&ctl->drain, 0, kStatusInGemmTf32x3);
            }
        }
    } else {
        // --------------------------------------------------- converters (+ epilogue)
        const int c = tid - 32;
        const bool drains = warp >= kEpiWarp0;
        const int e = tid - kEpiWarp0 * 32;  // TMEM lane = output feature within the tile
        const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
        const uint32_t sum = tmem + C::kColSum + lane_off;
        // Chunks wait to be folded in the order they end: a chunk that ends at step
        // g is folded into the tile's sum (in TMEM) once step g + 2 is converted, so
        // that the wait on the chunk's MMAs never holds up the next conversions. At
        // most two are pending (one chunk ends per step).
        struct Pending {
            int64_t n0, t0;
            uint32_t step;
            int32_t split;
            bool first, last;  // the tile's first / last chunk
        };
        Pending pend[2];
        int n_pend = 0;
        uint32_t qf = 0;  // chunks folded
        auto fold = [&](const Pending& pc) -> bool {
            const uint32_t buf = qf & 1u;
            if (!wait_or_abort(&ctl->d_full[buf], (qf >> 1) & 1u, ctl)) return false;
            tc::fence_after_sync();
            int64_t col = 0, ld = 0;
            float* out = nullptr;
            if (pc.last) {
                col = pc.n0 + e;
                if (p.splits > 1) {
                    out = p.partial + int64_t(pc.split) * p.m * p.n + col;
                    ld = p.n;
                } else {
                    out = p.outs[col / p.out_block] + (col % p.out_block);
                    ld = p.ldc;
                }
            }
#pragma unroll 1
            for (int cc = 0; cc < BT / 32; ++cc) {
                float v[32];
                tc::tmem_ld32(tmem + buf * uint32_t(BT) + uint32_t(cc * 32) + lane_off, v);
                tc::tmem_ld_wait();
                if (!pc.first) {
                    float a[32];
                    tc::tmem_ld32(sum + uint32_t(cc * 32), a);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) v[jj] = a[jj] + v[jj];
                }
                if (!pc.last) {
                    tc::tmem_st32(sum + uint32_t(cc * 32), v);
                    continue;
                }
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    const int64_t t = pc.t0 + cc * 32 + jj;
                    if (t < p.m) {
                        float* o = out + t * ld;
                        if (p.splits > 1 || p.epilogue == NVLLM_GEMM_STORE) {
                            *o = v[jj];
                        } else if (p.epilogue == NVLLM_GEMM_ACCUMULATE) {
                            *o += v[jj];
                        } else {
                            *o = silu(v[jj]);
                        }
                    }
                }
            }
            if (!pc.last) tc::tmem_st_wait();
            tc::fence_before_sync();
            mbar_arrive(&ctl->d_free[buf]);
            ++qf;
            return true;
        };
        auto fold_pending = [&](uint32_t upto) -> bool {
            while (n_pend > 0 && pend[0].step + 2 <= upto) {
                if (!fold(pend[0])) return false;
                pend[0] = pend[1];
                --n_pend;
            }
            return true;
        };
        uint32_t g = 0;  // stages converted
        bool ok = true;
        for (int64_t it = blockIdx.x; ok && it < p.items; it += gridDim.x) {
            const Item im = item_of(p, it, BT);
            for (int s = 0; s < im.nsteps; ++s, ++g) {
                if (!wait_or_abort(&ctl->kv_full[g % S], (g / S) & 1u, ctl)) {
                    ok = false;
                    break;
                }
                unsigned char* st = stage_ptr(g);
                if (!p.w_split) {
                    float4* a = reinterpret_cast<float4*>(st);
                    float4* alo = reinterpret_cast<float4*>(st + C::kABytes);
                    for (int i = c; i < int(C::kABytes / 16); i += kConvThreads) {
                        float4 hi, lo;
                        tf32_split4(a[i], hi, lo);
                        a[i] = hi;
                        alo[i] = lo;
                    }
                }
                float4* b = reinterpret_cast<float4*>(st + 2 * C::kABytes);
                float4* blo = reinterpret_cast<float4*>(st + 2 * C::kABytes + C::kBBytes);
                for (int i = c; i < int(C::kBBytes / 16); i += kConvThreads) {
                    float4 hi, lo;
                    tf32_split4(b[i], hi, lo);
                    b[i] = hi;
                    blo[i] = lo;
                }
                tc::fence_async_smem();
                mbar_arrive(&ctl->cv_full[g % S]);
                if (!drains) continue;
                if (!fold_pending(g)) {
                    ok = false;
                    break;
                }
                const bool chunk_last = s % kChunkSteps == kChunkSteps - 1 || s + 1 == im.nsteps;
                if (chunk_last) {
                    pend[n_pend++] = Pending{im.n0, im.t0, g, im.split, s < kChunkSteps,
                                             s + 1 == im.nsteps};
                }
            }
        }
        if (drains && ok) fold_pending(g + 2);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, C::kTmemCols);
    }
}

// hi = x rounded to tf32 (nearest), lo = x - hi, elementwise
__global__ void tf32_split_kernel(const float* __restrict__ in, float* __restrict__ hi,
                                  float* __restrict__ lo, int64_t count) {
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
        const float x = in[i];
        const float h = tc::to_tf32(x);
        hi[i] = h;
        lo[i] = x - h;
    }
}

// Split-K: out = epi(sum over splits of the partials), splits in a fixed order.
__global__ void splitk_reduce_kernel(const GemmParams p) {
    const int64_t total = p.m * (p.n / 4);
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t t = i / (p.n / 4);
        const int64_t c = (i - t * (p.n / 4)) * 4;
        float4 acc = reinterpret_cast<const float4*>(p.partial + t * p.n + c)[0];
        for (int sp = 1; sp < p.splits; ++sp) {
            const float4 v = reinterpret_cast<const float4*>(p.partial + (int64_t(sp) * p.m + t) * p.n + c)[0];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        float* o = p.outs[c / p.out_block] + t * p.ldc + (c % p.out_block);
        const float r[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (p.epilogue == NVLLM_GEMM_STORE) {
                o[q] = r[q];
            } else if (p.epilogue == NVLLM_GEMM_ACCUMULATE) {
                o[q] += r[q];
            } else {
                o[q] = silu(r[q]);
            }
        }
    }
}

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

// rows x cols fp32 matrix with row stride ld (floats), boxes of 32 columns x box_rows
// rows in the 128-byte swizzle; rows past the end read as zero
bool make_map(CUtensorMap* map, const float* ptr, int64_t rows, int64_t cols, int64_t ld,
              int box_rows) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(ld) * sizeof(float)};
    const cuuint32_t box[2] = {uint32_t(kBK), uint32_t(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides,
              box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    return sms;
}

int token_tile(int64_t m) { return m <= 32 ? 32 : 128; }

// Tiles of the problem, and the K split that gives the grid enough work when
// there are fewer tiles than SMs (decode-size m). Returns the split count.
int32_t plan_splits(int64_t m, int64_t n, int64_t k, int32_t* steps_per_split) {
    const int64_t tiles = (n / kBN) * ((m + token_tile(m) - 1) / token_tile(m));
    const int32_t total = int32_t(k / kBK);
    const int sms = sm_count();
    int32_t splits = 1;
    if (tiles < sms) {
        const int64_t want = (sms + tiles - 1) / tiles;
        splits = int32_t(std::min<int64_t>({want, int64_t(kMaxSplits), int64_t(total / 4)}));
        if (splits < 1) splits = 1;
    }
    const int32_t sps = (total + splits - 1) / splits;
    *steps_per_split = sps;
    return (total + sps - 1) / sps;  // no empty split
}

template <int BT>
cudaError_t launch(const GemmParams& p, const CUtensorMap& wmap, const CUtensorMap& wlomap,
                   const CUtensorMap& xmap, cudaStream_t st) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        e = cudaFuncSetAttribute(gemm_kernel<BT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(Cfg<BT>::kSmem));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const int64_t grid = std::min<int64_t>(p.items, sm_count());
    gemm_kernel<BT><<<unsigned(grid), kThreads, Cfg<BT>::kSmem, st>>>(p, wmap, wlomap, xmap);
    e = cudaGetLastError();
    if (e != cudaSuccess || p.splits <= 1) return e;
    const int64_t work = p.m * (p.n / 4);
    const int64_t blocks = std::min<int64_t>((work + 255) / 256, int64_t(sm_count()) * 8);
    splitk_reduce_kernel<<<unsigned(blocks), 256, 0, st>>>(p);
    return cudaGetLastError();
}

bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace
}  // namespace nvllm

using namespace nvllm;

extern "C" {

int nvllm_tf32_split(const float* in, float* hi, float* lo, int64_t count, void* stream) {
    if (count < 0 || (count > 0 && (in == nullptr || hi == nullptr || lo == nullptr))) {
        return NVLLM_ERR_INVALID;
    }
    if (count == 0) return NVLLM_OK;
    const int64_t blocks = std::min<int64_t>((count + 255) / 256, int64_t(sm_count()) * 8);
    tf32_split_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(in, hi, lo,
                                                                                       count);
    return cudaGetLastError() == cudaSuccess ? NVLLM_OK : NVLLM_ERR_CUDA;
}

size_t nvllm_gemm_workspace_size(int64_t m, int64_t n, int64_t k) {
    if (m <= 0 || n <= 0 || k <= 0 || n % kBN != 0 || k % kBK != 0) return 0;
    int32_t sps = 0;
    const int32_t splits = plan_splits(m, n, k, &sps);
    return splits > 1 ? size_t(splits) * size_t(m) * size_t(n) * sizeof(float) : 0;
}

int nvllm_gemm_tf32x3(const float* x, int64_t lda, int64_t m, int64_t k, const float* wt,
                      const float* wt_lo, int64_t n, float* const* outs, int32_t n_outs,
                      int64_t out_block,
                      int64_t ldc, int32_t epilogue, void* workspace, size_t workspace_bytes,
                      void* stream) {
    if (m < 0 || n <= 0 || k <= 0 || n % kBN != 0 || k % kBK != 0 || lda < k || lda % 4 != 0 ||
        n_outs < 1 || n_outs > kMaxOuts || out_block <= 0 || out_block % kBN != 0 ||
        out_block * n_outs != n || ldc < out_block || epilogue < NVLLM_GEMM_STORE ||
        epilogue > NVLLM_GEMM_SILU || outs == nullptr) {
        return NVLLM_ERR_INVALID;
    }
    if (m == 0) return NVLLM_OK;
    if (x == nullptr || wt == nullptr || !aligned16(x) || !aligned16(wt) ||
        (wt_lo != nullptr && !aligned16(wt_lo))) {
        return NVLLM_ERR_INVALID;
    }
    GemmParams p{};
    for (int i = 0; i < n_outs; ++i) {
        if (outs[i] == nullptr) return NVLLM_ERR_INVALID;
        p.outs[i] = outs[i];
    }
    p.m = m;
    p.n = n;
    p.k = k;
    p.out_block = out_block;
    p.ldc = ldc;
    p.epilogue = epilogue;
    p.w_split = wt_lo != nullptr ? 1 : 0;
    p.n_tiles = int32_t(n / kBN);
    const int BT = token_tile(m);
    p.t_tiles = int32_t((m + BT - 1) / BT);
    p.total_steps = int32_t(k / kBK);
    p.splits = plan_splits(m, n, k, &p.steps_per_split);
    if (p.splits > 1) {
        const size_t need = size_t(p.splits) * size_t(m) * size_t(n) * sizeof(float);
        if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)) {
            return NVLLM_ERR_WORKSPACE;
        }
        p.partial = static_cast<float*>(workspace);
    }
    p.items = int64_t(p.n_tiles) * p.t_tiles * p.splits;
    CUtensorMap wmap, wlomap, xmap;
    if (!make_map(&wmap, wt, n, k, k, kBN) || !make_map(&xmap, x, m, k, lda, BT) ||
        !make_map(&wlomap, wt_lo != nullptr ? wt_lo : wt, n, k, k, kBN)) {
        return NVLLM_ERR_CUDA;
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const cudaError_t e = BT == 32 ? launch<32>(p, wmap, wlomap, xmap, st)
                                   : launch<128>(p, wmap, wlomap, xmap, st);
    return e == cudaSuccess ? NVLLM_OK : NVLLM_ERR_CUDA;
}

}  // extern "C"
