// fp32-quality GEMM on the tcgen05 tensor cores for projections of few rows
// (decode steps, src/model.cpp:42-62 at m <= 32), the weights in the
// reference's row-major layout:
//
//   C_b[t, c] = epi( sum_k X[t, k] * W_b[k, c] )    X [m, k], W_b [k, n] row-major
//
// At m <= 32 the product is a stream of W (8 KB of weights per 128 x 32 x 32
// block of MACs), so W crosses HBM once, unsplit, and everything else happens
// on chip. The MMA computes D[128 output features (TMEM lanes), 64 columns] =
// W_tile^T . [X_hi | X_lo]^T with W read straight from its TMA tile as an
// MN-major A operand (a row of W is 128 contiguous output features: the
// layout it has in memory, so W is never transposed or moved on chip), and
// X's 32 token rows followed by their lo parts as one K-major B operand of 64
// rows. Every product is fp32-quality through tf32 parts: the tensor core
// reads a tf32 operand as the top 19 bits of its fp32 container, so hi = x as
// stored and lo = x - (x with its low 13 bits cleared), exact. Per 8 of K:
// W [X_hi | X_lo] (N = 64) and W_lo X_hi (N = 32, into the first 32 columns),
// where W_lo, written beside W by the converters, is an MN-major A operand in
// the same layout. Column t + 32 (W X_lo) is added to column t at the fold.
//
// Per stage (32 rows of K), with 15 warps per CTA (one CTA per SM):
//   warp 12: the TMA copies into a 5-stage ring, one per lane (W tile 32 x 128 fp32
//     as four 32-column boxes in the 128-byte swizzle with 32-byte granules,
//     the layout of an MN-major tf32 operand; X tile 32 rows x 32 fp32,
//     128-byte swizzle; no multicast);
//   warps 13 and 14, lane 0: the 8 MMAs of a stage and their commits, the
//     two warps taking alternate accumulation chunks (2 stages each) into
//     their own pairs of accumulators: a tcgen05.mma takes about as long to
//     issue as one of these small ones takes to run;
//   warps 0-7: converters in two groups of four that take alternate stages:
//     W_lo beside W and X_lo beside X, elementwise in the landed layouts;
//   warps 8-11: fold each finished accumulation chunk (2 stages = 64 of K:
//     the tensor core's fp32 accumulation truncates, so long sums stay in
//     fp32 registers) into registers, thread = output feature (TMEM lane),
//     32 token sums each, and write the tile's columns at the end of its
//     segment.
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
constexpr int kBT = 32;        // token rows (X_hi: B rows 0-31, X_lo: 32-63)
constexpr int kStageK = 32;    // K rows per stage
constexpr int kStages = 5;
constexpr int kChunk = 2;      // stages per TMEM accumulation chunk
constexpr int kGroupThreads = 128;  // one converter group
constexpr int kFoldWarp0 = 8;
constexpr int kProducerWarp = 12;
constexpr int kIssuerWarp = 13;     // and 14: the two MMA issuers
constexpr int kIssuers = 2;
constexpr int kThreads = 15 * 32;   // converters 0-7, folders 8-11, producer, 2 issuers
constexpr int kFoldThreads = 128;
constexpr int kMaxBatch = 3;
constexpr int kMinUnits = 8;   // stages a CTA handles at least
constexpr uint32_t kWAtom = kStageK * 128;           // 32 K rows x 32 features: 4 KB
constexpr uint32_t kWBytes = 4 * kWAtom;             // 16 KB
constexpr uint32_t kXBytes = kBT * kStageK * 4;      // 4 KB
constexpr uint32_t kStageBytes = 2 * kWBytes + 2 * kXBytes;  // W, W_lo, X, X_lo
constexpr uint32_t kOffCtl = kStages * kStageBytes;
constexpr uint32_t kSmem = kOffCtl + 512 + 1024;
static_assert(kSmem <= 227u * 1024u, "shared memory");
static_assert(kStageBytes % 1024 == 0 && kWBytes % 1024 == 0 && kXBytes % 1024 == 0,
              "swizzle atoms stay aligned");
// TMEM: two accumulators of 64 columns per issuer
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColsD = 2 * kBT;
constexpr uint32_t kIdescBoth = tc::tf32_idesc(kTileN, 2 * kBT, true, false);  // W [X_hi | X_lo]
constexpr uint32_t kIdescHi = tc::tf32_idesc(kTileN, kBT, true, false);        // W_lo X_hi

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
    uint64_t conv[kStages];    // W_lo and X_lo written (kGroupThreads arrivals)
    uint64_t empty[kStages];   // the stage's MMAs completed
    uint64_t d_full[2 * kIssuers];  // [issuer, buffer] accumulation chunk complete
    uint64_t d_free[2 * kIssuers];  // [issuer, buffer] chunk folded (kFoldThreads arrivals)
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
// The same, its outcome the same on every lane of the warp (a warp whose lanes
// left a spin at different iterations must not split around a collective step).
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, Control* ctl,
                                          uint32_t where = 0) {
    return __all_sync(0xffffffffu, wait_or_abort(bar, parity, ctl, where));
}
// roles and barriers of the where code
enum : uint32_t { kWhoProducer = 1, kWhoIssuer = 2, kWhoConverter = 4, kWhoFolder = 6 };
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

// x minus the part of it the tensor core reads as tf32 (its top 19 bits): exact
__device__ __forceinline__ float lo_part(float x) {
    return x - __uint_as_float(__float_as_uint(x) & 0xffffe000u);
}

// Walks a CTA's units in order: the tile and stage of each, its position in
// the tile's segment (the tile's units in this CTA), and the chunk rule shared
// by the issuer and the folders.
struct UnitWalk {
    int64_t tile;
    int stage, j, len;
    __device__ UnitWalk(int64_t u0, int spt) : tile(u0 / spt), stage(int(u0 % spt) - 1), j(0), len(0) {}
    // advances to unit g (called with g = 0, 1, ...); returns its position in the segment
    __device__ int next(uint32_t g, uint32_t nu, int spt) {
        if (++stage == spt) {
            stage = 0;
            ++tile;
        }
        if (g == 0 || stage == 0) {
            j = 0;
            len = min(spt - stage, int(nu - g));
        }
        return j++;
    }
    __device__ bool chunk_first(int jj) const { return jj % kChunk == 0; }
    __device__ bool chunk_last(int jj) const { return jj % kChunk == kChunk - 1 || jj + 1 == len; }
    __device__ bool seg_end(int jj) const { return jj + 1 == len; }
};

// grid: p.ctas persistent CTAs, CTA c owning units [first_unit(c), first_unit(c + 1))
__global__ void __launch_bounds__(kThreads, 1)
    decode_gemm_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap wmap,
                       const __grid_constant__ CUtensorMap xmap) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = align1024(smem_raw);
    Control* ctl = reinterpret_cast<Control*>(smem + kOffCtl);
    const int tid = int(threadIdx.x), warp = tid / 32, lane = tid % 32;
    const int64_t u0 = first_unit(blockIdx.x, p.units, p.ctas);
    const uint32_t nu = uint32_t(first_unit(int64_t(blockIdx.x) + 1, p.units, p.ctas) - u0);

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&ctl->full[i], 1);
            mbar_init(&ctl->conv[i], kGroupThreads);
            mbar_init(&ctl->empty[i], 1);
        }
        for (int b = 0; b < 2 * kIssuers; ++b) {
            mbar_init(&ctl->d_full[b], 1);
            mbar_init(&ctl->d_free[b], kFoldThreads);
        }
        for (int i = 0; i < kIssuers; ++i) mbar_init(&ctl->drain[i], 1);
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
        // a stage's five copies (four W atoms, the X tile) go one to a lane,
        // so that they leave as one warp instruction
        uint32_t loaded = 0;
        int tile = int(u0 / p.spt), stage = int(u0 % p.spt);
        for (uint32_t g = 0; g < nu; ++g) {
            const uint32_t s = g % kStages;
            if (g >= uint32_t(kStages) &&
                !wait_warp(&ctl->empty[s], ((g / kStages) - 1) & 1u, ctl,
                           where_code(kWhoProducer, kBarEmpty, g))) {
                break;
            }
            unsigned char* st = smem + s * kStageBytes;
            if (lane == 0) mbar_arrive_expect_tx(&ctl->full[s], kWBytes + kXBytes);
            __syncwarp();
            const int x0 = (tile % p.n_tiles) * kTileN, y = stage * kStageK;
            if (lane < kTileN / 32) {
                tma_load_3d(st + lane * kWAtom, &wmap, x0 + lane * 32, y, tile / p.n_tiles,
                            &ctl->full[s]);
            } else if (lane == kTileN / 32) {
                tc::tma_load_2d(st + 2 * kWBytes, &xmap, y, 0, &ctl->full[s]);
            }
            __syncwarp();
            loaded = g + 1;
            if (++stage == p.spt) {
                stage = 0;
                ++tile;
            }
        }
        // copies in flight land before the CTA ends (bounded waits)
        if (lane == 0) {
            for (uint32_t h = loaded > uint32_t(kStages) ? loaded - kStages : 0; h < loaded; ++h) {
                mbar_wait(&ctl->full[h % kStages], (h / kStages) & 1u, kStatusInGemmDecodeTc);
            }
        }
    } else if (warp >= kIssuerWarp) {
        // ------------------------------------------------------------------ MMAs
        // The CTA's units fall into accumulation chunks (kChunk stages, or
        // fewer at a tile's end); chunk q is issued by issuer q % 2 into its
        // own pair of accumulators, so that two threads issue: a tcgen05.mma
        // takes about as long to issue as one of these small ones takes to run.
        const uint32_t me = uint32_t(warp - kIssuerWarp);
        if (lane == 0) {
            // The operands' descriptors, built once: a descriptor's start
            // address is its low 14 bits in 16-byte units and shared-memory
            // addresses stay below 2^18, so a slot's or a K step's operand is
            // the base descriptor plus its byte offset / 16 (no carry out of
            // the field). A: 8 rows of K start 1 KB into each 32-feature atom;
            // the atoms of the 128 features are kWAtom apart (leading byte
            // offset), groups of 4 rows 512 bytes (stride byte offset). B: 8 of
            // K are 32 bytes into each 128-byte row, 8-row groups 1 KB apart.
            const uint32_t base = smem_addr(smem);
            const uint64_t a_hi = tc::sw128_32b_desc(base, kWAtom, 512);
            const uint64_t a_lo = tc::sw128_32b_desc(base + kWBytes, kWAtom, 512);
            const uint64_t b_x = tc::sw128_desc(base + 2 * kWBytes, 16, 1024);
            uint32_t q = 0;  // chunks of the CTA started (both issuers)
            uint32_t s = 0, phase = 0;  // ring slot of unit g and its phase
            bool issued_mma = false;
            UnitWalk walk(u0, p.spt);
            for (uint32_t g = 0; g < nu; ++g) {
                const int jj = walk.next(g, nu, p.spt);
                const bool first = walk.chunk_first(jj), last = walk.chunk_last(jj);
                if ((q % kIssuers) == me) {
                    const uint32_t lq = q / kIssuers;  // this issuer's chunk count
                    const uint32_t ib = me * 2u + (lq & 1u);
                    if (!wait_or_abort(&ctl->conv[s], phase, ctl,
                                       where_code(kWhoIssuer, kBarConv, g))) {
                        break;
                    }
                    if (first && lq >= 2 &&
                        !wait_or_abort(&ctl->d_free[ib], ((lq >> 1) - 1) & 1u, ctl,
                                       where_code(kWhoIssuer, kBarDFree, g))) {
                        break;
                    }
                    tc::fence_after_sync();
                    const uint64_t so = uint64_t(s * (kStageBytes >> 4));
                    const uint32_t d = tmem + ib * kColsD;
#pragma unroll
                    for (int kk = 0; kk < kStageK / 8; ++kk) {
                        const uint64_t b = b_x + so + uint64_t(kk * (32 >> 4));
                        const uint64_t ka = so + uint64_t(kk * (1024 >> 4));
                        tc::mma_tf32(d, a_hi + ka, b, kIdescBoth, !first || kk > 0);
                        tc::mma_tf32(d, a_lo + ka, b, kIdescHi, true);
                    }
                    tc::commit(&ctl->empty[s]);
                    if (last) tc::commit(&ctl->d_full[ib]);
                    issued_mma = true;
                }
                if (last) ++q;
                if (++s == uint32_t(kStages)) {
                    s = 0;
                    phase ^= 1u;
                }
            }
            // issued MMAs complete before the TMEM is freed (bounded wait)
            if (issued_mma) {
                tc::commit(&ctl->drain[me]);
                mbar_wait(&ctl->drain[me], 0, kStatusInGemmDecodeTc);
            }
        }
    } else if (warp < kFoldWarp0) {
        // ------------------------------------------------------------ converters
        const int grp = warp / 4;
        const int r = tid % kGroupThreads;
        for (uint32_t g = uint32_t(grp); g < nu; g += 2) {
            const uint32_t s = g % kStages;
            // a slot is reloaded only after the MMAs that read its previous
            // contents completed (the producer waits on `empty`)
            if (!wait_warp(&ctl->full[s], (g / kStages) & 1u, ctl,
                           where_code(kWhoConverter + uint32_t(grp), kBarFull, g))) {
                break;
            }
            unsigned char* st = smem + s * kStageBytes;
            // W then X (4 KB after W_lo) -> their lo parts, all loads first
            const float4* w = reinterpret_cast<const float4*>(st);
            float4* wl = reinterpret_cast<float4*>(st + kWBytes);
            const float4* x = reinterpret_cast<const float4*>(st + 2 * kWBytes);
            float4* xl = reinterpret_cast<float4*>(st + 2 * kWBytes + kXBytes);
            constexpr int kW4 = int(kWBytes / 16) / kGroupThreads;  // float4 of W per thread
            constexpr int kX4 = int(kXBytes / 16) / kGroupThreads;  // and of X
            float4 v[kW4 + kX4];
#pragma unroll
            for (int i = 0; i < kW4; ++i) v[i] = w[r + i * kGroupThreads];
#pragma unroll
            for (int i = 0; i < kX4; ++i) v[kW4 + i] = x[r + i * kGroupThreads];
#pragma unroll
            for (int i = 0; i < kW4 + kX4; ++i) {
                const float4 lo =
                    make_float4(lo_part(v[i].x), lo_part(v[i].y), lo_part(v[i].z), lo_part(v[i].w));
                if (i < kW4) {
                    wl[r + i * kGroupThreads] = lo;
                } else {
                    xl[r + (i - kW4) * kGroupThreads] = lo;
                }
            }
            tc::fence_async_smem();
            mbar_arrive(&ctl->conv[s]);
        }
    } else if (warp < kFoldWarp0 + 4) {
        // ------------------------------------------------- accumulation, epilogue
        // thread = output feature 32 (warp % 4) + lane of the tile (its TMEM lane)
        const int f = (warp % 4) * 32 + lane;
        const uint32_t lane_off = uint32_t((warp % 4) * 32) << 16;
        float acc[kBT];
#pragma unroll
        for (int i = 0; i < kBT; ++i) acc[i] = 0.f;
        uint32_t q = 0;  // chunks folded, in the CTA's order (issuer q % 2)
        UnitWalk walk(u0, p.spt);
        for (uint32_t g = 0; g < nu; ++g) {
            const int jj = walk.next(g, nu, p.spt);
            if (!walk.chunk_last(jj)) continue;
            const uint32_t lq = q / kIssuers;
            const uint32_t ib = (q % kIssuers) * 2u + (lq & 1u);
            if (!wait_warp(&ctl->d_full[ib], (lq >> 1) & 1u, ctl,
                           where_code(kWhoFolder, kBarDFull, q))) {
                break;
            }
            tc::fence_after_sync();
            float hi[kBT], lo[kBT];
            tc::tmem_ld32(tmem + ib * kColsD + lane_off, hi);
            tc::tmem_ld32(tmem + ib * kColsD + kBT + lane_off, lo);
            tc::tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < kBT; ++i) acc[i] += hi[i] + lo[i];
            tc::fence_before_sync();
            mbar_arrive(&ctl->d_free[ib]);
            ++q;
            if (!walk.seg_end(jj)) continue;
            // the tile's segment is complete: write its column f for every row
            const int64_t tile = walk.tile;
            const int64_t c_first = owner(tile * p.spt, p.units, p.ctas);
            const int64_t c_last = owner((tile + 1) * p.spt - 1, p.units, p.ctas);
            const int64_t col = (tile % p.n_tiles) * kTileN + f;
            if (c_first == c_last) {
                if (col < p.n) {
                    float* o = out_of(p, int(tile / p.n_tiles)) + col;
#pragma unroll
                    for (int t = 0; t < kBT; ++t) {
                        if (t < p.m) apply(o + int64_t(t) * p.ldc, acc[t], p.epilogue);
                    }
                }
            } else {
                float* part = p.partial +
                              (tile * p.max_seg + (int64_t(blockIdx.x) - c_first)) * kBT * kTileN + f;
#pragma unroll
                for (int t = 0; t < kBT; ++t) {
                    if (t < p.m) part[int64_t(t) * kTileN] = acc[t];
                }
            }
#pragma unroll
            for (int i = 0; i < kBT; ++i) acc[i] = 0.f;
        }
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
// boxes of 32 columns x 32 rows, 128-byte swizzle with 32-byte granules (the
// shared-memory layout of an MN-major tf32 operand); X [m, k] (row stride
// lda) as {k, m} in boxes of 32 columns x 32 rows, 128-byte swizzle. Reads
// past the ends are zero.
bool make_maps(CUtensorMap* wmap, CUtensorMap* xmap, const float* w, int64_t ldw, int64_t wbs,
               int64_t n, int64_t k, int32_t batch, const float* x, int64_t lda, int64_t m) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t wdims[3] = {cuuint64_t(n), cuuint64_t(k), cuuint64_t(batch)};
    const cuuint64_t wstr[2] = {cuuint64_t(ldw) * 4, cuuint64_t(wbs) * 4};
    const cuuint32_t wbox[3] = {32u, uint32_t(kStageK), 1};
    const cuuint32_t e3[3] = {1, 1, 1};
    if (fn(wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(w), wdims, wstr, wbox, e3,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
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
