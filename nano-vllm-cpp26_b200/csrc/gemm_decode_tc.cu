// fp32-quality GEMM on the tcgen05 tensor cores for projections of few rows
// (decode steps, src/model.cpp:42-62 at m <= 32), the weights in the
// reference's row-major layout:
//
//   C_b[t, c] = epi( sum_k X[t, k] * W_b[k, c] )    X [m, k], W_b [k, n] row-major
//
// At m <= 32 the product is a stream of W (8 KB of weights per 128 x 32 x 32
// block of MACs), so W crosses HBM once, unsplit, and everything else happens
// on chip. The MMA computes D[128 columns of W, 32 token rows] = W^T_tile .
// X_tile^T (M = 128 output features in TMEM lanes, N = 32 tokens, K = 8 per
// instruction), every product in 3xTF32: hi = x rounded to tf32 (nearest),
// lo = x - hi, and W_hi X_hi + W_lo X_hi + W_hi X_lo (the tensor core reads a
// tf32 operand as the top 19 bits of its fp32 container). X_lo is stored right
// after X_hi, so W_hi [X_hi | X_lo] is a single N = 64 MMA into a 64-column
// accumulator whose halves are added when it is folded.
//
// Per stage (32 rows of K), with 11 warps per CTA (one CTA per SM, all 512
// TMEM columns):
//   warp 8, lane 0: the TMA copies into an 8-stage ring (W tile 32 x 128 fp32,
//     no swizzle; X tile 32 rows x 32 fp32, 128-byte swizzle; no multicast);
//   warps 9-10, lane 0: the 8 MMAs of a stage, alternate stages each into its
//     own accumulators (a single issuing thread leaves the tensor core idle
//     around each of its mbarrier waits and commits), never waiting on an MMA;
//   warps 0-7: converters in two groups of four that take alternate stages.
//     Lane r of warp w owns output feature 32 (w % 4) + r: it reads column r
//     of the W tile (32 conflict-free scalar loads: the transpose happens
//     here), splits it and stores hi and lo into its own TMEM lane
//     (tcgen05.st) in one of four A buffers, so the MMA takes A from TMEM
//     (.ts form); it also splits a share of the X tile in shared memory (hi
//     in place, lo beside). Group 0 also folds every finished accumulation
//     chunk (an issuer's 4 stages = 128 of K: the tensor core's fp32
//     accumulation truncates, so long sums stay in fp32 registers) into
//     registers, two stages behind, and writes the result.
// Work is split stream-K: the (tile, stage) units of all output tiles are
// dealt to the persistent CTAs in equal contiguous ranges; a tile that one CTA
// covers whole is written directly with the epilogue op, the pieces of a
// shared tile go to a workspace and a second kernel sums them in CTA order
// (fixed), so results do not depend on scheduling.
// Every wait is bounded; on a timeout the CTA records NVLLM_ERR_TIMEOUT, lets
// its copies and MMAs finish and frees its TMEM.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "nvllm.h"
#include "nvllm_ops.h"
#include "tcgen05.cuh"

namespace nvllm {
namespace {

constexpr int kTileN = 128;    // output features per tile (MMA M, TMEM lanes)
constexpr int kBT = 32;        // token rows (MMA N)
constexpr int kStageK = 32;    // K rows per stage
constexpr int kStages = 8;
constexpr int kChunk = 4;      // an issuer's stages per TMEM accumulation chunk
constexpr int kABufs = 4;      // A operand buffers in TMEM (units converted ahead)
constexpr int kGroupThreads = 128;  // one converter group: a warp per TMEM lane quarter
constexpr int kProducerWarp = 8;
constexpr int kIssuers = 2;    // MMA-issuing warps: the CTA's unit g to issuer g % 2
constexpr int kMmaWarp0 = 9;   // warps 9-10
constexpr int kThreads = 32 * (kMmaWarp0 + kIssuers);  // converters, producer, issuers
constexpr int kMaxBatch = 3;
constexpr int kMinUnits = 8;   // stages a CTA handles at least
constexpr uint32_t kWBytes = kStageK * kTileN * 4;  // 16 KB
constexpr uint32_t kXBytes = kBT * kStageK * 4;     // 4 KB
constexpr uint32_t kStageBytes = kWBytes + 2 * kXBytes;  // W, X (hi in place), X lo
// TMEM: four A buffers (hi 32 + lo 32 columns each) and two accumulators (64
// columns each: W_hi X_hi + W_lo X_hi in 0-31, W_hi X_lo in 32-63) for each MMA issuer
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColA = 0;
constexpr uint32_t kColD = kABufs * 64;
constexpr uint32_t kDCols = 2 * kBT;
// X lo lies directly after X hi in the stage (same swizzle, 1024-byte row groups),
// so W_hi [X_hi | X_lo] is one N = 64 MMA
constexpr uint32_t kIdescHi = tc::tf32_idesc(kTileN, 2 * kBT, false, false);
constexpr uint32_t kIdescLo = tc::tf32_idesc(kTileN, kBT, false, false);
constexpr uint32_t kSmem = kStages * kStageBytes + 512 + 1024;
static_assert(kSmem <= 227u * 1024u, "shared memory");
// every ring slot (and every A buffer) belongs to one issuer: units g and g + kStages
// (g + kABufs) go to the same issuer
static_assert(kStages % kIssuers == 0 && kABufs % kIssuers == 0, "issuer assignment");
static_assert(kABufs * 64 + kIssuers * 2 * kDCols <= kTmemCols, "TMEM columns");

struct DecodeParams {
    int64_t m, n, k, ldc;
    float* outs[kMaxBatch];
    float* partial;            // [tiles, max_seg, kBT, kTileN]
    int32_t epilogue;
    int32_t n_tiles, tiles;    // column tiles of one matrix; all tiles (x batch)
    int32_t spt;               // stages per tile
    int64_t units;             // tiles * spt
    int32_t ctas, max_seg;
};

struct Control {
    uint64_t full[kStages];    // TMA landed (transaction bytes)
    uint64_t conv[kStages];    // A in TMEM, X split (kGroupThreads arrivals)
    uint64_t empty[kStages];   // the stage's MMAs completed
    uint64_t d_full[kIssuers][2];  // [issuer][buffer] accumulation chunk complete
    uint64_t d_free[kIssuers][2];  // chunk folded into registers (kGroupThreads arrivals)
    uint64_t drain[kIssuers];
    uint32_t tmem_base;
    int32_t abort;
};
static_assert(sizeof(Control) <= 512, "control block");

// The units of CTA c: [first(c), first(c + 1)).
__host__ __device__ __forceinline__ int64_t first_unit(int64_t c, int64_t units, int64_t ctas) {
    return c * units / ctas;
}

// The CTA whose range holds unit u.
__host__ __device__ __forceinline__ int64_t owner(int64_t u, int64_t units, int64_t ctas) {
    int64_t c = u * ctas / units;
    if (c > ctas - 1) c = ctas - 1;
    while (c > 0 && first_unit(c, units, ctas) > u) --c;
    while (c + 1 < ctas && first_unit(c + 1, units, ctas) <= u) ++c;
    return c;
}

// where: role << 24 | barrier << 16 | unit, recorded if this wait gives up first
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, Control* ctl,
                                              uint32_t where = 0) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*reinterpret_cast<volatile int32_t*>(&ctl->abort)) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            raise_status(kStatusTimeout | kStatusInGemmDecodeTc);
            record_timeout(kStatusInGemmDecodeTc, where | (parity << 15), bar);
            atomicExch(&ctl->abort, 1);
            return false;
        }
    }
}
// roles and barriers of the where code
enum : uint32_t { kWhoProducer = 1, kWhoIssuer = 2, kWhoConverter = 4 };
enum : uint32_t { kBarFull = 1, kBarConv = 2, kBarEmpty = 3, kBarDFull = 4, kBarDFree = 5 };
__device__ __forceinline__ uint32_t where_code(uint32_t who, uint32_t bar, uint32_t g) {
    return (who << 24) | (bar << 16) | (g & 0x7fffu);
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

__device__ __forceinline__ void apply(float* o, float v, int32_t epilogue) {
    if (epilogue == NVLLM_GEMM_STORE) {
        *o = v;
    } else if (epilogue == NVLLM_GEMM_ACCUMULATE) {
        *o += v;
    } else {
        *o = silu(v);
    }
}

__device__ __forceinline__ float* out_of(const DecodeParams& p, int b) {
    return b == 0 ? p.outs[0] : (b == 1 ? p.outs[1] : p.outs[2]);
}

__device__ __forceinline__ unsigned char* align1024(unsigned char* p) {
    return reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// hi = x rounded to tf32 (nearest), lo = x - hi (exact), elementwise
__device__ __forceinline__ void split4(float4& v, float4& lo) {
    const float4 hi = make_float4(tc::to_tf32(v.x), tc::to_tf32(v.y), tc::to_tf32(v.z),
                                  tc::to_tf32(v.w));
    lo = make_float4(v.x - hi.x, v.y - hi.y, v.z - hi.z, v.w - hi.w);
    v = hi;
}

// grid: p.ctas persistent CTAs, CTA c owning units [first_unit(c), first_unit(c + 1))
__global__ void __launch_bounds__(kThreads, 1)
    decode_gemm_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap wmap,
                       const __grid_constant__ CUtensorMap xmap) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = align1024(smem_raw);
    Control* ctl = reinterpret_cast<Control*>(smem + kStages * kStageBytes);
    const int tid = int(threadIdx.x), warp = tid / 32, lane = tid % 32;
    const int64_t u0 = first_unit(blockIdx.x, p.units, p.ctas);
    const uint32_t nu = uint32_t(first_unit(int64_t(blockIdx.x) + 1, p.units, p.ctas) - u0);

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&ctl->full[i], 1);
            mbar_init(&ctl->conv[i], kGroupThreads);
            mbar_init(&ctl->empty[i], 1);
        }
        for (int i = 0; i < kIssuers; ++i) {
            for (int b = 0; b < 2; ++b) {
                mbar_init(&ctl->d_full[i][b], 1);
                mbar_init(&ctl->d_free[i][b], kGroupThreads);
            }
            mbar_init(&ctl->drain[i], 1);
        }
        ctl->abort = 0;
    }
    fence_barrier_init();
    if (warp == 0) {
        tc::tmem_alloc(&ctl->tmem_base, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == kProducerWarp) {
        // ------------------------------------------------------------ TMA copies
        if (lane == 0) {
            uint32_t loaded = 0;
            int tile = int(u0 / p.spt), stage = int(u0 % p.spt);
            for (uint32_t g = 0; g < nu; ++g) {
                const uint32_t s = g % kStages;
                if (g >= uint32_t(kStages) &&
                    !wait_or_abort(&ctl->empty[s], ((g / kStages) - 1) & 1u, ctl,
                                   where_code(kWhoProducer, kBarEmpty, g))) {
                    break;
                }
                unsigned char* st = smem + s * kStageBytes;
                mbar_arrive_expect_tx(&ctl->full[s], kWBytes + kXBytes);
                tma_load_3d(st, &wmap, (tile % p.n_tiles) * kTileN, stage * kStageK,
                            tile / p.n_tiles, &ctl->full[s]);
                tc::tma_load_2d(st + kWBytes, &xmap, stage * kStageK, 0, &ctl->full[s]);
                loaded = g + 1;
                if (++stage == p.spt) {
                    stage = 0;
                    ++tile;
                }
            }
            // copies in flight land before the CTA ends (bounded waits)
            for (uint32_t h = loaded > uint32_t(kStages) ? loaded - kStages : 0; h < loaded; ++h) {
                mbar_wait(&ctl->full[h % kStages], (h / kStages) & 1u, kStatusInGemmDecodeTc);
            }
        }
    } else if (warp >= kMmaWarp0 && warp < kMmaWarp0 + kIssuers) {
        // ------------------------------------------------------------------ MMAs
        // issuer i takes the CTA's units g with g % kIssuers == i, into its own
        // accumulators: the threads keep the tensor core busy between the waits
        // and commits that each of them makes. Assigning by g (not by the position
        // within a tile's segment) gives every ring slot one issuer, which waits on
        // that slot's barrier phases in order; an issuer waiting on a slot another
        // issuer still has to consume could see the phase before its own as done.
        const int me = warp - kMmaWarp0;
        if (lane == 0) {
            uint32_t q = 0;  // this issuer's accumulation chunks
            bool issued_mma = false;
            int j = 0, len = 0;  // stage within its segment, segment length
            int stage = int(u0 % p.spt);
            for (uint32_t g = 0; g < nu; ++g, stage = stage + 1 == p.spt ? 0 : stage + 1) {
                if (g == 0 || stage == 0) {
                    j = 0;
                    len = min(p.spt - stage, int(nu - g));
                }
                const int jj = j++;
                if (int(g % kIssuers) != me) continue;
                // chunks: windows of kIssuers * kChunk units of the segment, kChunk
                // of them this issuer's
                const int w = jj % (kIssuers * kChunk);
                const bool chunk_first = w < kIssuers;
                const bool chunk_last = w >= kIssuers * (kChunk - 1) || jj + kIssuers >= len;
                const uint32_t s = g % kStages, ab = g % kABufs, buf = q & 1u;
                if (!wait_or_abort(&ctl->conv[s], (g / kStages) & 1u, ctl,
                                   where_code(kWhoIssuer + uint32_t(me), kBarConv, g))) {
                    break;
                }
                if (chunk_first && q >= 2 &&
                    !wait_or_abort(&ctl->d_free[me][buf], ((q >> 1) - 1) & 1u, ctl,
                                   where_code(kWhoIssuer + uint32_t(me), kBarDFree, g))) {
                    break;
                }
                tc::fence_after_sync();
                const uint32_t xhi = smem_addr(smem + s * kStageBytes + kWBytes);
                const uint32_t a_hi = tmem + kColA + ab * 64u;
                const uint32_t a_lo = a_hi + 32u;
                const uint32_t d = tmem + kColD + uint32_t(me * 2 + int(buf)) * kDCols;
#pragma unroll
                for (int kk = 0; kk < kStageK / 8; ++kk) {
                    // B = rows 0-31 X_hi, rows 32-63 X_lo (N = 64) / X_hi alone (N = 32)
                    const uint64_t dh = tc::sw128_desc(xhi + uint32_t(kk) * 32u, 16, 1024);
                    tc::mma_tf32_ts(d, a_hi + uint32_t(kk) * 8u, dh, kIdescHi,
                                    !chunk_first || kk > 0);
                    tc::mma_tf32_ts(d, a_lo + uint32_t(kk) * 8u, dh, kIdescLo, true);
                }
                tc::commit(&ctl->empty[s]);
                if (chunk_last) {
                    tc::commit(&ctl->d_full[me][buf]);
                    ++q;
                }
                issued_mma = true;
            }
            // issued MMAs complete before the TMEM is freed (bounded wait)
            if (issued_mma) {
                tc::commit(&ctl->drain[me]);
                mbar_wait(&ctl->drain[me], 0, kStatusInGemmDecodeTc);
            }
        }
    } else {
        // -------------------------- converters (two groups), accumulation, epilogue
        const int grp = warp / 4;          // converts the units g with g % 2 == grp
        const int r = tid % kGroupThreads;  // output feature within the tile = TMEM lane
        const uint32_t lane_off = uint32_t((warp % 4) * 32) << 16;
        float acc[kBT];
#pragma unroll
        for (int t = 0; t < kBT; ++t) acc[t] = 0.f;
        uint32_t qf[kIssuers] = {};  // chunks folded, per issuer (group 0)
        // folds issuer i's next chunk into acc (chunks are folded in the order in
        // which they end, a fixed order)
        auto fold = [&](int i) -> bool {
            const uint32_t q = qf[i], buf = q & 1u;
            if (!wait_or_abort(&ctl->d_full[i][buf], (q >> 1) & 1u, ctl,
                               where_code(kWhoConverter, kBarDFull, (uint32_t(i) << 14) | q))) {
                return false;
            }
            tc::fence_after_sync();
            const uint32_t dcol = tmem + kColD + uint32_t(i * 2 + int(buf)) * kDCols + lane_off;
            float v[kBT], w[kBT];
            tc::tmem_ld32(dcol, v);
            tc::tmem_ld32(dcol + uint32_t(kBT), w);
            tc::tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < kBT; ++t) acc[t] += v[t] + w[t];
            tc::fence_before_sync();
            mbar_arrive(&ctl->d_free[i][buf]);
            qf[i] = q + 1;
            return true;
        };
        // the segment of `tile` is complete: the whole tile (epilogue op) or a piece
        auto finish = [&](int64_t tile) {
            const int64_t c_first = owner(tile * p.spt, p.units, p.ctas);
            const int64_t c_last = owner((tile + 1) * p.spt - 1, p.units, p.ctas);
            const int64_t col = (tile % p.n_tiles) * kTileN + r;
            if (c_first == c_last) {
                if (col < p.n) {
                    float* o = out_of(p, int(tile / p.n_tiles)) + col;
                    for (int t = 0; t < kBT; ++t) {
                        if (t < p.m) apply(o + int64_t(t) * p.ldc, acc[t], p.epilogue);
                    }
                }
            } else {
                float* part = p.partial +
                              ((tile * p.max_seg + (int64_t(blockIdx.x) - c_first)) * kBT) * kTileN + r;
#pragma unroll
                for (int t = 0; t < kBT; ++t) part[t * kTileN] = acc[t];
            }
#pragma unroll
            for (int t = 0; t < kBT; ++t) acc[t] = 0.f;
        };
        // Chunks waiting to be folded, in the order they end: a chunk that ends at
        // unit e is folded when unit e + 2 has been converted, so that folding (a
        // wait on the chunk's MMAs) never delays the conversion of the next units.
        // At most two are pending (one chunk ends per unit at most).
        struct Pending {
            int64_t tile;
            uint32_t unit;
            int issuer;
            bool seg_end;
        };
        Pending pend[2];
        int n_pend = 0;
        auto fold_pending = [&](uint32_t upto) -> bool {
            while (n_pend > 0 && pend[0].unit + 2 <= upto) {
                if (!fold(pend[0].issuer)) return false;
                if (pend[0].seg_end) finish(pend[0].tile);
                pend[0] = pend[1];
                --n_pend;
            }
            return true;
        };
        bool ok = true;
        int j = 0, len = 0;
        int64_t tile = u0 / p.spt;
        int stage = int(u0 % p.spt) - 1;
        for (uint32_t g = 0; ok && g < nu; ++g) {
            if (++stage == p.spt) {
                stage = 0;
                ++tile;
            }
            if (g == 0 || stage == 0) {
                j = 0;
                len = min(p.spt - stage, int(nu - g));
            }
            const int jj = j++;
            const bool seg_end = jj + 1 == len;
            // the same chunk rule as the issuers (issuer g % kIssuers)
            const bool chunk_last =
                jj % (kIssuers * kChunk) >= kIssuers * (kChunk - 1) || jj + kIssuers >= len;
            if (int(g % 2) == grp) {
                const uint32_t s = g % kStages, ab = g % kABufs;
                // A buffer ab was last read by the MMAs of unit g - kABufs, whose
                // completion is that of its stage
                const uint32_t h = g - uint32_t(kABufs);
                if (!wait_or_abort(&ctl->full[s], (g / kStages) & 1u, ctl,
                                   where_code(kWhoConverter + uint32_t(grp), kBarFull, g)) ||
                    (g >= uint32_t(kABufs) &&
                     !wait_or_abort(&ctl->empty[h % kStages], (h / kStages) & 1u, ctl,
                                    where_code(kWhoConverter + uint32_t(grp), kBarEmpty, g)))) {
                    ok = false;
                    break;
                }
                unsigned char* st = smem + s * kStageBytes;
                const float* wt = reinterpret_cast<const float*>(st);
                float hi[kStageK], lo[kStageK];
#pragma unroll
                for (int kk = 0; kk < kStageK; ++kk) {
                    const float x = wt[kk * kTileN + r];
                    hi[kk] = tc::to_tf32(x);
                    lo[kk] = x - hi[kk];
                }
                tc::fence_after_sync();
                tc::tmem_st32(tmem + kColA + ab * 64u + lane_off, hi);
                tc::tmem_st32(tmem + kColA + ab * 64u + 32u + lane_off, lo);
                float4* xs = reinterpret_cast<float4*>(st + kWBytes);
                float4* xl = reinterpret_cast<float4*>(st + kWBytes + kXBytes);
#pragma unroll
                for (int i = r; i < int(kXBytes / 16); i += kGroupThreads) split4(xs[i], xl[i]);
                tc::tmem_st_wait();
                tc::fence_async_smem();
                tc::fence_before_sync();
                mbar_arrive(&ctl->conv[s]);
            }
            if (grp != 0) continue;
            if (!fold_pending(g)) {
                ok = false;
                break;
            }
            if (chunk_last) pend[n_pend++] = Pending{tile, g, int(g % kIssuers), seg_end};
        }
        if (grp == 0 && ok) fold_pending(nu + 2);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

// The tiles that several CTAs share: out = epi(sum of the pieces in CTA order).
__global__ void decode_fixup_kernel(const DecodeParams p) {
    const int64_t per_tile = p.m * kTileN;
    const int64_t total = per_tile * p.tiles;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t tile = i / per_tile;
        const int64_t rem = i - tile * per_tile;
        const int64_t t = rem / kTileN, r = rem - t * kTileN;
        const int64_t c_first = owner(tile * p.spt, p.units, p.ctas);
        const int64_t c_last = owner((tile + 1) * p.spt - 1, p.units, p.ctas);
        const int64_t col = (tile % p.n_tiles) * kTileN + r;
        if (c_first == c_last || col >= p.n) continue;
        const float* src = p.partial + (tile * p.max_seg * kBT + t) * kTileN + r;
        float v = src[0];
        for (int64_t jj = 1; jj <= c_last - c_first; ++jj) v += src[jj * kBT * kTileN];
        apply(out_of(p, int(tile / p.n_tiles)) + t * p.ldc + col, v, p.epilogue);
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
// boxes of 128 columns x 32 rows, no swizzle; X [m, k] (row stride lda) as
// {k, m} in boxes of 32 columns x 32 rows, 128-byte swizzle. Reads past the
// ends are zero.
bool make_maps(CUtensorMap* wmap, CUtensorMap* xmap, const float* w, int64_t ldw, int64_t wbs,
               int64_t n, int64_t k, int32_t batch, const float* x, int64_t lda, int64_t m) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t wdims[3] = {cuuint64_t(n), cuuint64_t(k), cuuint64_t(batch)};
    const cuuint64_t wstr[2] = {cuuint64_t(ldw) * 4, cuuint64_t(wbs) * 4};
    const cuuint32_t wbox[3] = {uint32_t(kTileN), uint32_t(kStageK), 1};
    const cuuint32_t e3[3] = {1, 1, 1};
    if (fn(wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(w), wdims, wstr, wbox, e3,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        return false;
    }
    const cuuint64_t xdims[2] = {cuuint64_t(k), cuuint64_t(m)};
    const cuuint64_t xstr[1] = {cuuint64_t(lda) * 4};
    const cuuint32_t xbox[2] = {uint32_t(kStageK), uint32_t(kBT)};
    return fn(xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), xdims, xstr, xbox,
              e3, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
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

cudaError_t configure() {
    static bool done[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!done[dev]) {
        e = cudaFuncSetAttribute(decode_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(kSmem));
        if (e != cudaSuccess) return e;
        done[dev] = true;
    }
    return cudaSuccess;
}


// Tiles, stages, and the persistent grid: one CTA per SM, each with
// at least kMinUnits stages; max_seg = the most CTAs that share one tile.
DecodeParams plan(int64_t m, int64_t n, int64_t k, int32_t batch) {
    DecodeParams p{};
    p.m = m;
    p.n = n;
    p.k = k;
    p.n_tiles = int32_t((n + kTileN - 1) / kTileN);
    p.tiles = p.n_tiles * batch;
    p.spt = int32_t((k + kStageK - 1) / kStageK);
    p.units = int64_t(p.tiles) * p.spt;
    const int64_t wave = sm_count();  // one CTA per SM (all 512 TMEM columns)
    p.ctas = int32_t(std::max<int64_t>(1, std::min<int64_t>(wave, p.units / kMinUnits)));
    p.max_seg = 1;
    for (int64_t t = 0; t < p.tiles; ++t) {
        const int64_t segs = owner((t + 1) * p.spt - 1, p.units, p.ctas) -
                             owner(t * p.spt, p.units, p.ctas) + 1;
        p.max_seg = int32_t(std::max<int64_t>(p.max_seg, segs));
    }
    return p;
}

size_t workspace_bytes(const DecodeParams& p) {
    if (p.max_seg <= 1) return 0;
    return size_t(p.tiles) * size_t(p.max_seg) * kBT * kTileN * sizeof(float);
}

bool valid_shape(int64_t m, int64_t n, int64_t k, int32_t batch) {
    return m >= 0 && m <= kBT && n > 0 && k > 0 && n < (int64_t(1) << 31) &&
           k < (int64_t(1) << 31) && batch >= 1 && batch <= kMaxBatch;
}

bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace
}  // namespace nvllm

using namespace nvllm;

extern "C" {

size_t nvllm_gemm_decode_tc_workspace_size(int64_t m, int64_t n, int64_t k, int32_t batch) {
    if (!valid_shape(m, n, k, batch) || m == 0) return 0;
    return workspace_bytes(plan(m, n, k, batch));
}

int nvllm_gemm_decode_tc(const float* x, int64_t lda, int64_t m, int64_t k, const float* w,
                         int64_t ldw, int64_t n, int32_t batch, int64_t w_batch_stride,
                         float* const* outs, int64_t ldc, int32_t epilogue, void* workspace,
                         size_t workspace_bytes_given, void* stream) {
    if (!valid_shape(m, n, k, batch) || lda < k || lda % 4 != 0 || ldw < n || ldw % 4 != 0 ||
        ldc < n || outs == nullptr || epilogue < NVLLM_GEMM_STORE || epilogue > NVLLM_GEMM_SILU ||
        (batch > 1 && (w_batch_stride < k * ldw || w_batch_stride % 4 != 0))) {
        return NVLLM_ERR_INVALID;
    }
    if (m == 0) return NVLLM_OK;
    if (x == nullptr || w == nullptr || !aligned16(x) || !aligned16(w)) return NVLLM_ERR_INVALID;
    DecodeParams p = plan(m, n, k, batch);
    p.ldc = ldc;
    p.epilogue = epilogue;
    for (int i = 0; i < batch; ++i) {
        if (outs[i] == nullptr) return NVLLM_ERR_INVALID;
        p.outs[i] = outs[i];
    }
    const size_t need = workspace_bytes(p);
    if (need > 0) {
        if (workspace == nullptr || workspace_bytes_given < need || !aligned16(workspace)) {
            return NVLLM_ERR_WORKSPACE;
        }
        p.partial = static_cast<float*>(workspace);
    }
    CUtensorMap wmap, xmap;
    if (!make_maps(&wmap, &xmap, w, ldw, batch > 1 ? w_batch_stride : k * ldw, n, k, batch, x,
                   lda, m)) {
        return NVLLM_ERR_CUDA;
    }
    if (configure() != cudaSuccess) return NVLLM_ERR_CUDA;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    decode_gemm_kernel<<<unsigned(p.ctas), kThreads, kSmem, st>>>(p, wmap, xmap);
    if (cudaGetLastError() != cudaSuccess) return NVLLM_ERR_CUDA;
    if (need > 0) {
        const int64_t work = int64_t(p.tiles) * m * kTileN;
        const int64_t blocks = std::min<int64_t>((work + 255) / 256, int64_t(sm_count()) * 8);
        decode_fixup_kernel<<<unsigned(blocks), 256, 0, st>>>(p);
        if (cudaGetLastError() != cudaSuccess) return NVLLM_ERR_CUDA;
    }
    return NVLLM_OK;
}

}  // extern "C"
