// K3 (tensor cores): causal paged prefill attention on tcgen05.
//
// Same mathematics as src/model.cpp:204-260 for sequences with more than one
// query row, with the two dense products QK^T and PV on the 5th-generation
// tensor cores (fp32 accumulation in TMEM) and the softmax in fp32.
// Geometry: head_dim 128, block size 16 (one TMA box = the 16 rows of one
// physical block and 32 columns of one head).
//
// Operand precision: every fp32 operand x is split into two bf16 terms,
// x0 = bf16(x) and x1 = bf16(x - x0) (16 significant bits together, against
// 11 for one tf32 operand), and each product is taken as three bf16 MMAs
// (kind::f16) with fp32 accumulation: A0 B0 + A0 B1 + A1 B0; the dropped A1 B1
// is ~2^-16 of the product. Against tf32 hi / lo parts, bf16 terms take half
// the bytes in TMEM and shared memory and an MMA covers 16 of the reduction
// instead of 8, so the S tile is 64 keys wide: a 64-key tile takes 24 S MMAs
// (N = 64) and 12 O MMAs (N = 128).
//
// One CTA per SM (persistent), 12 warps:
//   warps 0-3  softmax / epilogue: thread t owns query row t of a 128-row tile
//              and TMEM lane t. Per key tile it reads its row of S from TMEM,
//              applies the causal mask, updates the running maximum and sum,
//              rescales its row of O in TMEM when its reference maximum moved
//              (rarely: see kRescaleMargin), and stores P as two bf16 terms into
//              its TMEM lane, in one of two P buffers (the A operand of P.V).
//   warp 4     MMAs: lane 0 issues every tcgen05.mma and commit: S(t+1) = Q K(t+1)^T
//              is queued while the softmax works on S(t); O(t) += P(t) V(t) once
//              P(t) is in TMEM.
//   warp 5     loader: the TMA gathers of the K and V tiles into a 3-stage ring,
//              one 2 KiB box (a block's 16 rows of one 32-dim atom of K or V)
//              per lane, up to three tiles ahead of the MMAs.
//   warps 6-11 converters: turn each landed fp32 K tile, then V tile, in place,
//              into its two bf16 terms, zeroing the V rows of keys past the
//              visible ones; S waits only for K's terms, O for V's.
// Shared memory per stage (64 keys): K as landed, fp32 in four 128-byte
// swizzled atoms of 32 dims, then in the same 32 KiB its terms K0 and K1, each
// two 128-byte swizzled atoms of 64 bf16 dims (the K-major B operand of S); V
// likewise, its terms read MN-major as the B operand of O (a 16-bit MN-major
// operand takes the plain 128-byte swizzle, so V needs no transpose). The fp32
// atoms land in the order 0, 2, 1, 3, so that the two that hold dims 64 p ..
// 64 p + 63 occupy exactly the bytes their terms go to (term 0 atom p, term 1
// atom p): two rows of an atom pair are read and written back by one warp,
// with no wait on any other.
// TMEM (512 columns): S x2 (2 x 64), P x2 (2 buffers x 2 terms x 32 columns of
// bf16 pairs), O (128), Q (2 terms x 64).
// Every wait is bounded; on a timeout the CTA records NVLLM_ERR_TIMEOUT, lets
// its outstanding copies and MMAs finish and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace nvllm {

namespace {

constexpr int kQT = 128;  // query rows per tile (= TMEM lanes)
constexpr int kKT = 64;   // keys per tile
constexpr int kHD = 128;
constexpr int kStages = 3;
constexpr int kSoftmaxThreads = 128;  // warps 0-3
constexpr int kMmaWarp = 4;
constexpr int kLoaderWarp = 5;
constexpr int kConvWarp0 = 6;
constexpr int kConvThreads = 192;     // warps 6-11
constexpr int kThreads = kSoftmaxThreads + 64 + kConvThreads;
constexpr int kItemReaders = kThreads / 32 - 1;  // every warp but the loader

// TMEM columns: S[0] 0..63, S[1] 64..127, P[b] at 128 + 64 b (term 0 then
// term 1, 32 columns each), O 256..383, Q term 0 384..447, term 1 448..511
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColP = 128;
constexpr uint32_t kColO = 256;
constexpr uint32_t kColQ = 384;

// Shared memory: a stage holds the fp32 K tile (4 atoms of 64 keys x 32 dims)
// then the V tile; after conversion each tile's 32 KiB hold its term 0 (2
// atoms of 64 keys x 64 bf16 dims) then its term 1.
constexpr uint32_t kF32Atom = kKT * 128;      // 64 rows x 32 fp32
constexpr uint32_t kB16Atom = kKT * 128;      // 64 rows x 64 bf16
constexpr uint32_t kTileBytes = 4 * kF32Atom; // one fp32 tile, or its two terms
constexpr uint32_t kTermBytes = 2 * kB16Atom; // one bf16 term of a tile
constexpr uint32_t kStageBytes = 2 * kTileBytes;
constexpr uint32_t kOffKV = 0;
constexpr uint32_t kOffBar = kOffKV + kStages * kStageBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + control block + alignment slack
static_assert(kSmemBytes <= 227u * 1024u, "shared memory");
// Byte offset of fp32 atom a (dims 32 a .. 32 a + 31) in a landed tile: atoms
// 2 p and 2 p + 1 at p * 8 KiB and 16 KiB + p * 8 KiB, where term 0 and term 1
// of atom p go.
__host__ __device__ constexpr uint32_t f32_atom_offset(int a) {
    return uint32_t((a & 1) * 2 + (a >> 1)) * kF32Atom;
}
static_assert(kF32Atom == kB16Atom && kTermBytes == 2 * kF32Atom, "atom pairs hold their terms");
constexpr int kConvUnits = (kKT / 2) * (kHD / 64);  // per tensor: row pairs x atom pairs

// Instruction descriptor for kind::f16 with bf16 A and B and fp32
// accumulation; b_mn: B is MN-major (else K-major).
constexpr uint32_t bf16_idesc(int M, int N, bool b_mn) {
    return (1u << 4)                    // D format: f32
           | (1u << 7)                  // A format: bf16
           | (1u << 10)                 // B format: bf16
           | (uint32_t(b_mn) << 16)     // B major
           | (uint32_t(N >> 3) << 17)   // N / 8
           | (uint32_t(M >> 4) << 24);  // M / 16
}
constexpr uint32_t kIdescS = bf16_idesc(kQT, kKT, false);
constexpr uint32_t kIdescO = bf16_idesc(kQT, kHD, true);

struct Control {
    uint64_t kv_full[kStages];  // TMA landed (transaction count)
    uint64_t kc_full[kStages];  // converters wrote K's bf16 terms (one per converter)
    uint64_t vc_full[kStages];  // converters wrote V's bf16 terms (one per converter)
    uint64_t st_free[kStages];  // O of the stage's tile complete: its K and V read
    uint64_t s_full[2];
    // Per P buffer b (the tiles n with n % 2 == b), so that neither side can
    // run two phases ahead of a waiter: p_full[b] P(n) in TMEM and O rescaled
    // when needed (128 arrivals); p_free[b] O(n) complete (P(n) and O(n) read)
    uint64_t p_full[2];
    uint64_t p_free[2];
    uint64_t drain;
    // work items pass through a two-slot queue: item_full[i] the loader wrote
    // items[i]; item_free[i] every other warp read it (kItemReaders arrivals);
    // q_full the query tile of the current item in TMEM (128 arrivals)
    uint64_t item_full[2];
    uint64_t item_free[2];
    uint64_t q_full;
    uint32_t tmem_base;
    int32_t items[2];
    int32_t abort;
};
static_assert(sizeof(Control) <= 256, "control block");

// Bounded wait that also gives up once another role has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, Control* ctl) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*reinterpret_cast<volatile int32_t*>(&ctl->abort)) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            raise_status(kStatusTimeout | kStatusInPrefillTc);
            atomicExch(&ctl->abort, 1);
            return false;
        }
    }
}

// Two-term bf16 split of a and b: x = x0 + x1 + r with x0 = bf16(x),
// x1 = bf16(x - x0), |r| <= 2^-17 |x|. t0 packs a0 (low half) and b0, t1 a1 and b1.
__device__ __forceinline__ void split2(float a, float b, uint32_t& t0, uint32_t& t1) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    t0 = *reinterpret_cast<const uint32_t*>(&h);
    t1 = *reinterpret_cast<const uint32_t*>(&l);
}

// The row's reference maximum moves only when a score exceeds it by more than
// this (log2 units): until then the weights exp2(s - m) stay <= 2^margin, O
// and l keep their scale, and the rescale of O (a TMEM round trip between one
// tile's P.V and the next tile's P) is skipped. The reference cancels in O / l,
// so only rounding differs.
#ifndef NVLLM_RESCALE_MARGIN
#define NVLLM_RESCALE_MARGIN 8.0f
#endif
constexpr float kRescaleMargin = NVLLM_RESCALE_MARGIN;

__device__ __forceinline__ uint32_t stage_of(uint32_t n) { return n % kStages; }
__device__ __forceinline__ uint32_t stage_parity(uint32_t n) { return (n / kStages) & 1u; }

// Stores 32 columns of raw 32-bit words into this warp's TMEM lanes.
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t* v) {
    float f[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
    tc::tmem_st32(taddr, f);
}

// 2^x on the MUFU unit (flush-to-zero: weights below 2^-126 of the row's
// reference maximum become 0, far below the tolerance of this path).
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// In-place conversion of a landed fp32 tile (64 keys x 128 dims) into its two
// bf16 terms. Unit u = (row pair u / 2, atom pair p = u % 2) is the 512 bytes
// that rows 2 (u / 2) and 2 (u / 2) + 1 of fp32 atoms 2 p and 2 p + 1 occupy,
// which are exactly the bytes those rows of term 0 atom p and term 1 atom p
// go to. Converter warp cw takes the units u = cw + 6 i; lane l reads 16
// bytes of atom 2 p + (l / 8) % 2, row 2 (u / 2) + l / 16, swizzle position
// l % 8 (a quarter-warp reads one 128-byte row of one atom), and writes 8
// bytes of each term (a half-warp writes one term row whole: no bank
// conflicts). The offsets depend only on the warp, the lane and i, so they
// are computed once per work item.
constexpr int kConvWarps = kConvThreads / 32;
constexpr int kConvMax = (kConvUnits + kConvWarps - 1) / kConvWarps;  // units per warp, at most
constexpr int kConvBatch = 4;  // units read before the warp writes

struct ConvPlan {
    uint32_t rd[kConvMax];   // read offset in the landed tile
    uint32_t wr[kConvMax];   // term-0 write offset (term 1: + kTermBytes)
    int32_t row[kConvMax];   // key row of the lane's data
    int32_t n;               // units of this warp
};

__device__ __forceinline__ void make_conv_plan(ConvPlan& cp, int cw, int lane) {
    cp.n = (kConvUnits - cw + kConvWarps - 1) / kConvWarps;
#pragma unroll
    for (int i = 0; i < kConvMax; ++i) {
        const int u = cw + kConvWarps * i;
        const int ap = u & 1;
        const int a = 2 * ap + ((lane >> 3) & 1);
        const int row = 2 * (u >> 1) + (lane >> 4);
        const int phys = lane & 7;
        const int dim = 32 * a + ((phys ^ (row & 7)) << 2);  // the first of the lane's 4 dims
        cp.rd[i] = f32_atom_offset(a) + uint32_t(row) * 128u + uint32_t(phys) * 16u;
        // term atom ap, the row, 16-byte chunk (dim % 64) / 8 swizzled by the
        // row, 8 bytes in when dim % 8 == 4
        cp.wr[i] = uint32_t(ap) * kB16Atom + uint32_t(row) * 128u +
                   uint32_t(((dim & 63) >> 3) ^ (row & 7)) * 16u + uint32_t(dim & 4) * 2u;
        cp.row[i] = row;
    }
}

// Converts this warp's units of one tile; rows >= zero_from become 0 (V).
template <bool kZero>
__device__ __forceinline__ void convert_tile(unsigned char* tile, const ConvPlan& cp, int zero_from) {
#pragma unroll
    for (int i0 = 0; i0 < kConvMax; i0 += kConvBatch) {
        float4 x[kConvBatch];
#pragma unroll
        for (int b = 0; b < kConvBatch; ++b) {
            if (i0 + b < kConvMax && i0 + b < cp.n) {
                x[b] = *reinterpret_cast<const float4*>(tile + cp.rd[i0 + b]);
            }
        }
        __syncwarp();
#pragma unroll
        for (int b = 0; b < kConvBatch; ++b) {
            const int i = i0 + b;
            if (i < kConvMax && i < cp.n) {
                if (kZero && cp.row[i] >= zero_from) x[b] = make_float4(0.f, 0.f, 0.f, 0.f);
                uint32_t a0, a1, b0, b1;
                split2(x[b].x, x[b].y, a0, a1);
                split2(x[b].z, x[b].w, b0, b1);
                *reinterpret_cast<uint2*>(tile + cp.wr[i]) = make_uint2(a0, b0);
                *reinterpret_cast<uint2*>(tile + kTermBytes + cp.wr[i]) = make_uint2(a1, b1);
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1)
prefill_tc_kernel(const AttnParams p, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap) {
    // a decode kernel launched as this kernel's programmatic dependent may start
    // on the SMs this grid leaves free (it reads nothing this kernel writes)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sKV = base + kOffKV;
    Control* ctl = reinterpret_cast<Control*>(base + kOffBar);
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&ctl->kv_full[i], 1);
            mbar_init(&ctl->kc_full[i], kConvThreads);
            mbar_init(&ctl->vc_full[i], kConvThreads);
            mbar_init(&ctl->st_free[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&ctl->s_full[i], 1);
            mbar_init(&ctl->p_full[i], kSoftmaxThreads);
            mbar_init(&ctl->p_free[i], 1);
        }
        mbar_init(&ctl->drain, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&ctl->item_full[i], 1);
            mbar_init(&ctl->item_free[i], kItemReaders);
        }
        mbar_init(&ctl->q_full, kSoftmaxThreads);
        ctl->abort = 0;
    }
    fence_barrier_init();
    if (warp == kMmaWarp) {
        tc::tmem_alloc(&ctl->tmem_base, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = ctl->tmem_base;
    const uint32_t tO = tmem + kColO;

    const ArenaGeom& g = p.g;
    const int H = g.num_heads;
    const int total = p.counters->prefill_items * H;
    uint32_t tile_seq = 0;    // key tiles processed by this CTA (ring position)
    uint32_t next_load = 0;   // loader: ring index of the next K/V load to issue
    bool issued_mma = false;  // MMA warp

    auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
        const bool got = wait_or_abort(bar, parity, ctl);
        return __all_sync(0xffffffffu, got);
    };
    // Work items: the loader's lane 0 takes each from the global cursor (the
    // loader needs an item first and runs ahead of the rest by up to the
    // ring's depth) and publishes it in the queue slot j % 2; every other warp
    // reads the items in the same order and frees the slot. -1 ends the loop.
    // No role waits for the others at an item boundary: the loader and the
    // converters go on into the next item's tiles while the softmax warps
    // finish the last one.
    auto publish = [&](uint32_t j, int it) -> bool {
        const uint32_t slot = j & 1u;
        if (j >= 2 && !wait_or_abort(&ctl->item_free[slot], ((j >> 1) - 1) & 1u, ctl)) return false;
        ctl->items[slot] = it;
        mbar_arrive(&ctl->item_full[slot]);
        return true;
    };
    auto take = [&](uint32_t j) -> int {
        const uint32_t slot = j & 1u;
        if (!wait_all(&ctl->item_full[slot], (j >> 1) & 1u)) return -1;
        const int it = *reinterpret_cast<volatile int32_t*>(&ctl->items[slot]);
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->item_free[slot]);
        return it;
    };

    for (uint32_t j = 0;; ++j) {
        int it = -1;
        if (warp == kLoaderWarp) {
            if (lane == 0) {
                if (!*reinterpret_cast<volatile int32_t*>(&ctl->abort)) {
                    it = atomicAdd(&p.counters->prefill_next, 1);
                    if (it >= total) it = -1;
                }
                if (!publish(j, it)) it = -1;
            }
            it = __shfl_sync(0xffffffffu, it, 0);
        } else {
            it = take(j);
        }
        if (it < 0 || *reinterpret_cast<volatile int32_t*>(&ctl->abort)) break;

        const WorkItem wi = p.prefill_items[it / H];
        const int h = it % H;
        const int s = wi.seq;
        const int q0 = p.cu_seqlens_q[s];
        const int qlen = p.cu_seqlens_q[s + 1] - q0;
        const int first_pos = p.context_lens[s] - qlen;
        const int r0 = wi.part * kQT;
        const int nrows = min(kQT, qlen - r0);
        const int nk = first_pos + r0 + nrows;  // keys 0..nk-1 visible to this tile
        const int ntiles = (nk + kKT - 1) / kKT;
        const uint32_t n0 = tile_seq;

        if (warp == kLoaderWarp) {
            // ------------------------------------------------------------------ loader
            // A tile's 32 boxes (4 blocks x 4 atoms x K, V) go one to a lane,
            // so that they leave as one warp instruction (a thread issuing its
            // copies one after another pays the issue cost of each): lane l
            // copies block l / 8, tensor (l / 4) % 2, atom l % 4. The block ids
            // of the item's next tiles are read a tile ahead. The stage is free
            // once O of its earlier tile completed (S read its K before).
            const int32_t* table = p.block_tables + int64_t(s) * p.max_blocks;
            const int lb = lane >> 3, lt = (lane >> 2) & 1, la = lane & 3;
            auto block_of = [&](int t) -> int64_t {
                const int kb = t * kKT;
                const int nb = t < ntiles ? (min(kKT, nk - kb) + 15) / 16 : 0;
                return lb < nb ? int64_t(table[kb / 16 + lb]) : int64_t(-1);
            };
            int64_t blk_next = block_of(0);
            for (int t = 0; t < ntiles; ++t) {
                const uint32_t n = n0 + t;
                const uint32_t st = stage_of(n);
                const int64_t blk = blk_next;
                blk_next = block_of(t + 1);
                if (n >= uint32_t(kStages) && !wait_all(&ctl->st_free[st], stage_parity(n - kStages))) {
                    break;
                }
                const int kbase = t * kKT;
                const int nblk = (min(kKT, nk - kbase) + 15) / 16;
                const bool valid = lb < nblk && blk >= 0 && blk < g.num_blocks;
                // a block's 8 boxes are 16 KiB; the lanes of one block agree
                const uint32_t vmask = __ballot_sync(0xffffffffu, valid);
                if (lane == 0) mbar_arrive_expect_tx(&ctl->kv_full[st], uint32_t(__popc(vmask)) * 2048u);
                __syncwarp();
                if (lb < nblk && !valid && (lane & 7) == 0) raise_status(kStatusBounds);
                if (valid) {
                    unsigned char* dst = sKV + st * kStageBytes + lt * kTileBytes +
                                         f32_atom_offset(la) + uint32_t(lb) * 2048u;
                    const int y = int((blk * g.num_layers + p.layer) * 16);
                    tc::tma_load_2d(dst, lt ? &vmap : &kmap, h * kHD + la * 32, y, &ctl->kv_full[st]);
                }
                __syncwarp();
                next_load = n + 1;
            }
        } else if (warp == kMmaWarp) {
            // -------------------------------------------------------------------- MMAs
            // once the converters have split K of tile n:
            // S(n) = Q1 K0^T + Q0 K1^T + Q0 K0^T, 16 dims per MMA; dims 16k..
            // start 32 k bytes into the rows of atom k / 4 (K-major, 8-row
            // groups 1 KiB apart)
            auto issue_s = [&](uint32_t n) -> bool {
                if (!wait_all(&ctl->kc_full[stage_of(n)], stage_parity(n))) return false;
                if (lane == 0) {
                    tc::fence_after_sync();
                    const uint32_t k0 = smem_addr(sKV + stage_of(n) * kStageBytes);
                    const uint32_t k1 = k0 + kTermBytes;
                    const uint32_t ts = tmem + (n & 1u) * kKT;
#pragma unroll
                    for (int k = 0; k < kHD / 16; ++k) {
                        const uint32_t off = (k >> 2) * kB16Atom + (k & 3) * 32u;
                        const uint64_t d0 = tc::sw128_desc(k0 + off, 16, 1024);
                        const uint64_t d1 = tc::sw128_desc(k1 + off, 16, 1024);
                        const uint32_t q0c = tmem + kColQ + 8u * k;
                        const uint32_t q1c = q0c + 64u;
                        tc::mma_f16_ts(ts, q1c, d0, kIdescS, k > 0);
                        tc::mma_f16_ts(ts, q0c, d1, kIdescS, true);
                        tc::mma_f16_ts(ts, q0c, d0, kIdescS, true);
                    }
                    tc::commit(&ctl->s_full[n & 1u]);
                    issued_mma = true;
                }
                __syncwarp();
                return true;
            };
            // O(n) += P1 V0 + P0 V1 + P0 V0, P from its TMEM buffer, V's terms
            // MN-major: keys 16k.. start 2 KiB into each 64-dim atom, the two
            // atoms of the 128 dims 8 KiB apart (leading byte offset), 8-key
            // groups 1 KiB apart (stride byte offset)
            auto issue_o = [&](uint32_t n, bool first) -> bool {
                if (!wait_all(&ctl->vc_full[stage_of(n)], stage_parity(n))) return false;
                if (lane == 0) {
                    tc::fence_after_sync();
                    const uint32_t v0 = smem_addr(sKV + stage_of(n) * kStageBytes + kTileBytes);
                    const uint32_t v1 = v0 + kTermBytes;
                    const uint32_t pb = tmem + kColP + (n & 1u) * 64u;
#pragma unroll
                    for (int k = 0; k < kKT / 16; ++k) {
                        const uint64_t d0 = tc::sw128_desc(v0 + k * 2048u, kB16Atom, 1024);
                        const uint64_t d1 = tc::sw128_desc(v1 + k * 2048u, kB16Atom, 1024);
                        tc::mma_f16_ts(tO, pb + 32u + 8u * k, d0, kIdescO, k > 0 || !first);
                        tc::mma_f16_ts(tO, pb + 8u * k, d1, kIdescO, true);
                        tc::mma_f16_ts(tO, pb + 8u * k, d0, kIdescO, true);
                    }
                    tc::commit(&ctl->p_free[n & 1u]);
                    tc::commit(&ctl->st_free[stage_of(n)]);
                }
                __syncwarp();
                return true;
            };
            // S(n+1) is queued while the softmax works on S(n); the first S of
            // an item waits for its Q tile in TMEM
            bool ok = wait_all(&ctl->q_full, j & 1u) && issue_s(n0);
            for (int t = 0; ok && t < ntiles; ++t) {
                const uint32_t n = n0 + t;
                if (t + 1 < ntiles && !issue_s(n + 1)) break;
                ok = wait_all(&ctl->p_full[n & 1u], (n >> 1) & 1u) && issue_o(n, t == 0);
            }
        } else if (warp >= kConvWarp0) {
            // -------------------------------------------------------------- converters
            // (the plan is rebuilt per item so that its registers are not live
            // in the other roles' code)
            ConvPlan cp;
            make_conv_plan(cp, warp - kConvWarp0, lane);
            for (int t = 0; t < ntiles; ++t) {
                const uint32_t n = n0 + t;
                // wait outcomes are made warp-uniform, so that no lane is left
                // alone in a warp-collective step after another gave up
                if (!__all_sync(0xffffffffu,
                                wait_or_abort(&ctl->kv_full[stage_of(n)], stage_parity(n), ctl))) {
                    break;
                }
                unsigned char* stage = sKV + stage_of(n) * kStageBytes;
                // K rows past the visible keys are masked by the softmax; V's
                // are zeroed, for their zero weights to cancel
                convert_tile<false>(stage, cp, kKT);
                tc::fence_async_smem();
                mbar_arrive(&ctl->kc_full[stage_of(n)]);
                convert_tile<true>(stage + kTileBytes, cp, nk - t * kKT);
                tc::fence_async_smem();
                mbar_arrive(&ctl->vc_full[stage_of(n)]);
            }
        } else {
            // ------------------------------------------------------------ softmax warps
            const int row = tid;  // query row and TMEM lane
            const int qpos = first_pos + r0 + row;
            const uint32_t lane_off = uint32_t(warp * 32) << 16;
            {
                // Q tile, times scale * log2 e (so that S holds log2-domain
                // scores), -> TMEM as the A operand of S = Q K^T: term 0 in
                // columns 384.., term 1 in 448.., one pair of consecutive dims
                // per column. The previous item's S MMAs all completed (this
                // warp waited for its last S).
                const float4* qrow = reinterpret_cast<const float4*>(
                    p.q + int64_t(q0 + r0 + row) * g.row + int64_t(h) * kHD);
#pragma unroll 1
                for (int c = 0; c < 2; ++c) {  // 64 dims -> 32 columns of each term
                    uint32_t t0[32], t1[32];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (row < nrows) v = __ldg(qrow + c * 16 + i);
                        const float qs = p.qk_scale_log2;
                        v = make_float4(v.x * qs, v.y * qs, v.z * qs, v.w * qs);
                        split2(v.x, v.y, t0[2 * i], t1[2 * i]);
                        split2(v.z, v.w, t0[2 * i + 1], t1[2 * i + 1]);
                    }
                    tmem_st32u(tmem + kColQ + c * 32u + lane_off, t0);
                    tmem_st32u(tmem + kColQ + 64u + c * 32u + lane_off, t1);
                }
                tc::tmem_st_wait();
                tc::fence_before_sync();
                mbar_arrive(&ctl->q_full);
            }
            float m_run = -INFINITY, l_run = 0.f;
            bool ok = true;
            for (int t = 0; t < ntiles; ++t) {
                const uint32_t n = n0 + t;
                if (!__all_sync(0xffffffffu,
                                wait_or_abort(&ctl->s_full[n & 1u], (n >> 1) & 1u, ctl))) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                float sc[kKT];
                tc::tmem_ld32(tmem + (n & 1u) * kKT + lane_off, sc);
                tc::tmem_ld32(tmem + (n & 1u) * kKT + 32u + lane_off, sc + 32);
                tc::tmem_ld_wait();
                const int kbase = t * kKT;
                // only tiles that reach past the tile's first query position
                // need the causal mask (keys past nk are past every row's too)
                if (kbase + kKT - 1 > first_pos + r0) {
#pragma unroll
                    for (int j = 0; j < kKT; ++j) {
                        const int kp = kbase + j;
                        sc[j] = (kp <= qpos && kp < nk) ? sc[j] : -INFINITY;
                    }
                }
                float mx[4] = {sc[0], sc[1], sc[2], sc[3]};
#pragma unroll
                for (int j = 4; j < kKT; ++j) mx[j & 3] = fmaxf(mx[j & 3], sc[j]);
                const float cm = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
                const float m_new = cm > m_run + kRescaleMargin ? cm : m_run;
                const float alpha = ex2_ftz(m_run - m_new);
                l_run *= alpha;
                m_run = m_new;
                // the P buffer is free once O of the tile two back completed
                if (n >= 2 && !__all_sync(0xffffffffu,
                                          wait_or_abort(&ctl->p_free[n & 1u],
                                                        ((n >> 1) - 1) & 1u, ctl))) {
                    ok = false;
                    break;
                }
                if (t > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
                    // O must hold the previous tile's P.V before it is rescaled
                    if (!__all_sync(0xffffffffu,
                                    wait_or_abort(&ctl->p_free[(n - 1) & 1u],
                                                  ((n - 1) >> 1) & 1u, ctl))) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
#pragma unroll 1
                    for (int c = 0; c < kHD / 32; ++c) {
                        float ov[32];
                        tc::tmem_ld32(tO + c * 32u + lane_off, ov);
                        tc::tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 32; ++j) ov[j] *= alpha;
                        tc::tmem_st32(tO + c * 32u + lane_off, ov);
                    }
                } else if (n >= 2) {
                    tc::fence_after_sync();
                }
                // P = exp2(s - m) as two bf16 terms, 32 keys (16 columns of each
                // term) at a time
                const uint32_t pb = tmem + kColP + (n & 1u) * 64u + lane_off;
                float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t p0[16], p1[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float a = ex2_ftz(sc[32 * half + 2 * j] - m_new);
                        const float b = ex2_ftz(sc[32 * half + 2 * j + 1] - m_new);
                        ls[j & 3] += a + b;
                        split2(a, b, p0[j], p1[j]);
                    }
                    tc::tmem_st16(pb + 16u * half, p0);
                    tc::tmem_st16(pb + 32u + 16u * half, p1);
                }
                l_run += (ls[0] + ls[1]) + (ls[2] + ls[3]);
                tc::tmem_st_wait();
                tc::fence_before_sync();
                mbar_arrive(&ctl->p_full[n & 1u]);
            }
            if (ok && ntiles > 0) {
                const uint32_t n = n0 + ntiles - 1;
                if (__all_sync(0xffffffffu,
                               wait_or_abort(&ctl->p_free[n & 1u], (n >> 1) & 1u, ctl))) {
                    tc::fence_after_sync();
                    const float inv = 1.0f / fmaxf(l_run, 1e-12f);
                    float4* op = reinterpret_cast<float4*>(
                        p.out + int64_t(q0 + r0 + row) * g.row + int64_t(h) * kHD);
#pragma unroll 1
                    for (int c = 0; c < kHD / 32; ++c) {
                        float ov[32];
                        tc::tmem_ld32(tO + c * 32u + lane_off, ov);
                        tc::tmem_ld_wait();
                        if (row < nrows) {
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                op[c * 8 + j] = make_float4(ov[4 * j] * inv, ov[4 * j + 1] * inv,
                                                            ov[4 * j + 2] * inv, ov[4 * j + 3] * inv);
                            }
                        }
                    }
                }
            }
            tc::fence_before_sync();
        }
        tile_seq += ntiles;
    }

    // Teardown: on an abort, let this CTA's copies and MMAs finish (bounded)
    // before its shared memory and TMEM are released.
    // (only the last load of each stage can still be in flight: a stage is
    // reloaded only after the MMAs that read its previous load completed)
    if (warp == kLoaderWarp && lane == 0) {
        for (uint32_t n = next_load > uint32_t(kStages) ? next_load - kStages : 0; n < next_load; ++n) {
            mbar_wait(&ctl->kv_full[stage_of(n)], stage_parity(n), kStatusInPrefillTc);
        }
    }
    if (warp == kMmaWarp && lane == 0) {
        if (issued_mma) {
            tc::commit(&ctl->drain);
            mbar_wait(&ctl->drain, 0, kStatusInPrefillTc);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
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

// 2D view of an arena: rows (block, layer, slot) x columns H*hd, box = one
// block's 16 rows x 32 columns, 128-byte swizzle.
bool make_arena_map(CUtensorMap* map, const float* arena, const ArenaGeom& g) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t dims[2] = {cuuint64_t(g.row),
                                cuuint64_t(g.num_blocks) * g.num_layers * g.block_size};
    const cuuint64_t strides[1] = {cuuint64_t(g.row) * sizeof(float)};
    const cuuint32_t box[2] = {32, 16};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(arena), dims, strides,
              box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool prefill_tc_supported(const ArenaGeom& g) { return g.head_dim == kHD && g.block_size == 16; }

int32_t prefill_tc_tile_rows() { return kQT; }

cudaError_t launch_prefill_tc(const AttnParams& p, cudaStream_t stream, int max_sms) {
    CUtensorMap kmap, vmap;
    if (!make_arena_map(&kmap, p.k_arena, p.g) || !make_arena_map(&vmap, p.v_arena, p.g)) {
        return cudaErrorInvalidValue;
    }
    static int grid_per_device[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (grid_per_device[dev] == 0) {
        e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(kSmemBytes));
        if (e != cudaSuccess) return e;
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        grid_per_device[dev] = sms;  // one CTA per SM (shared memory and TMEM sized for it)
    }
    const int grid = max_sms > 0 ? std::min(max_sms, grid_per_device[dev]) : grid_per_device[dev];
    prefill_tc_kernel<<<grid, kThreads, kSmemBytes, stream>>>(p, kmap, vmap);
    return cudaGetLastError();
}

}  // namespace nvllm
