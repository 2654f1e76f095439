// K3 (TF32 tensor cores): causal paged prefill attention on tcgen05.
//
// Same mathematics as src/model.cpp:204-260 for sequences with more than one
// query row, with the two dense products QK^T and PV on the 5th-generation
// tensor cores (kind::tf32, fp32 accumulation in TMEM); softmax in fp32.
// Geometry: head_dim 128, block size 16 (one TMA box = the 16 rows of one
// physical block and 32 columns of one head).
//
// One CTA per SM (persistent), 13 warps:
//   warps 0-3  softmax / epilogue: thread t owns query row t of a 128-row tile
//              and TMEM lane t. Per key tile (32 keys) it reads its row of S
//              from TMEM (tcgen05.ld), applies the causal mask, updates the
//              online max and sum, rescales its row of the O accumulator in
//              TMEM by exp(m_old - m_new) (skipped when no row of the warp saw
//              its maximum grow: the factor is then exactly 1), and stores P as
//              tf32 hi / lo parts into its own TMEM lane (the A operand of P.V).
//   warp 4     producer: one thread issues the TMA gathers of the K and V
//              tiles (2 physical blocks x 4 swizzle atoms per tensor) into a
//              3-stage ring and all tcgen05.mma: S(t+1) = Q K(t+1)^T is issued
//              while the softmax warps work on S(t); O(t) = P(t) V(t) once P(t)
//              is in TMEM, accumulating into O in TMEM.
//   warps 5-12 converters, working ahead of the MMAs: write the lo parts of the
//              landed K and V tiles next to them, and zero the V rows of keys
//              past the visible ones.
// Both products run as 3xTF32 (A_hi B_hi + A_lo B_hi + A_hi B_lo), which keeps
// them at fp32 accuracy: a single tf32 pass errs by ~1e-3 in the output at
// these magnitudes (one visible key => the output is that key's V row, carried
// at tf32 precision). The tensor core reads a tf32 operand as the top 19 bits
// of its fp32 container, so hi is the value itself and lo = x - (x with its low
// 13 bits cleared), exact in fp32; the terms left out (lo*lo and lo's own low
// bits) are ~2^-20 of the product. Q_hi and Q_lo live in TMEM as the A operand
// of S, P_hi and P_lo in TMEM as the A operand of O.
// The shared-memory operands are the tiles as TMA lands them and their lo
// parts in the same layout: K read K-major for S (128-byte swizzle, the 32
// dims of an atom row contiguous along the reduction), V read MN-major for O
// (the same rows, the reduction running down the keys; an MN-major tf32
// operand takes the 128-byte swizzle with 32-byte granules, which V's tensor
// map asks TMA for), so V needs no transpose on chip. TMEM (512 columns): S twice (2 x 32), P_hi and P_lo (32
// each), O (128), Q_hi and Q_lo (128 each).
// Every wait is bounded; on a timeout the CTA records NVLLM_ERR_TIMEOUT, lets
// its outstanding copies and MMAs finish and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace nvllm {

namespace {

constexpr int kQT = 128;  // query rows per tile (= TMEM lanes)
constexpr int kKT = 32;   // keys per tile
constexpr int kHD = 128;
constexpr int kStages = 3;
constexpr int kSoftmaxThreads = 128;  // warps 0-3
constexpr int kProducerWarp = 4;
constexpr int kConvThreads = 256;     // warps 5-12
constexpr int kThreads = kSoftmaxThreads + 32 + kConvThreads;
// TMEM columns: S[0] 0..31, S[1] 32..63, P_hi 64..95, P_lo 96..127, O 128..255,
// Q_hi 256..383, Q_lo 384..511
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColPhi = 64;
constexpr uint32_t kColPlo = 96;
constexpr uint32_t kColO = 128;
constexpr uint32_t kColQhi = 256;
constexpr uint32_t kColQlo = 384;

constexpr uint32_t kKVAtom = kKT * 128;         // 32 rows x 32 fp32
constexpr uint32_t kKBytes = 4 * kKVAtom;       // 16 KiB per tensor tile
constexpr uint32_t kStageBytes = 4 * kKBytes;   // K (= K_hi), K_lo, V (= V_hi), V_lo
constexpr uint32_t kOffKV = 0;
constexpr uint32_t kOffBar = kOffKV + kStages * kStageBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + control block + alignment slack
static_assert(kSmemBytes <= 227u * 1024u, "shared memory");

constexpr uint32_t kIdescS = tc::tf32_idesc(kQT, kKT, false, false);
// O's B operand is V as TMA lands it: MN-major (the 32 dims of an atom row
// contiguous, keys down the rows)
constexpr uint32_t kIdescO = tc::tf32_idesc(kQT, kHD, false, true);

struct Control {
    uint64_t kv_full[kStages];   // TMA landed (transaction count)
    uint64_t cv_full[kStages];   // converters wrote the stage's K_lo and V_lo (256 arrivals)
    uint64_t st_free[kStages];   // O of the stage's tile complete: its K and V read
    uint64_t s_full[2];
    uint64_t p_full;             // P in TMEM, previous O folded (128 arrivals)
    uint64_t o_full;
    uint64_t drain;
    uint32_t tmem_base;
    int32_t item;
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

// x = x_hi + lo exactly, with x_hi = x with its low 13 bits cleared (what the
// tensor core reads of a tf32 operand)
__device__ __forceinline__ float tf32_lo(float x) {
    return x - __uint_as_float(__float_as_uint(x) & 0xffffe000u);
}

#ifndef NVLLM_RESCALE_MARGIN
#define NVLLM_RESCALE_MARGIN 8.0f
#endif
constexpr float kRescaleMargin = NVLLM_RESCALE_MARGIN;

__device__ __forceinline__ uint32_t stage_of(uint32_t n) { return n % kStages; }
__device__ __forceinline__ uint32_t stage_parity(uint32_t n) { return (n / kStages) & 1u; }

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
            mbar_init(&ctl->cv_full[i], kConvThreads);
            mbar_init(&ctl->st_free[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&ctl->s_full[i], 1);
        }
        mbar_init(&ctl->p_full, kSoftmaxThreads);
        mbar_init(&ctl->o_full, 1);
        mbar_init(&ctl->drain, 1);
        ctl->abort = 0;
    }
    fence_barrier_init();
    if (warp == kProducerWarp) {
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
    uint32_t tile_seq = 0;   // key tiles processed by this CTA (ring position)
    uint32_t next_load = 0;  // producer: ring index of the next K/V load to issue
    uint32_t next_wait = 0;  // producer: ring index of the next load not known to have landed
    bool issued_mma = false;

    for (;;) {
        if (tid == 0) ctl->item = atomicAdd(&p.counters->prefill_next, 1);
        __syncthreads();
        const int it = ctl->item;
        const bool stop = it >= total || *reinterpret_cast<volatile int32_t*>(&ctl->abort);
        __syncthreads();
        if (stop) break;

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

        if (tid < kSoftmaxThreads) {
            // Q tile -> TMEM as the A operand of S = Q K^T, split for 3xTF32
            // (q_hi = q as read by the tensor core, q_lo = the rest).
            const int row = tid;
            const uint32_t lane_off = uint32_t(warp * 32) << 16;
            const float4* qrow = reinterpret_cast<const float4*>(
                p.q + int64_t(q0 + r0 + row) * g.row + int64_t(h) * kHD);
#pragma unroll 1
            for (int c = 0; c < kHD / 32; ++c) {
                float hi[32], lo[32];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (row < nrows) v = __ldg(qrow + c * 8 + i);
                    const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        hi[4 * i + e] = x[e];
                        lo[4 * i + e] = tf32_lo(x[e]);
                    }
                }
                tc::tmem_st32(tmem + kColQhi + c * 32u + lane_off, hi);
                tc::tmem_st32(tmem + kColQlo + c * 32u + lane_off, lo);
            }
            tc::tmem_st_wait();
            tc::fence_before_sync();
        }
        __syncthreads();

        if (warp == kProducerWarp) {
            // ---------------------------------------------------------------- producer
            // Lane 0 issues the TMA copies, the MMAs and their commits; the whole
            // warp takes part in the waits.
            const int32_t* table = p.block_tables + int64_t(s) * p.max_blocks;
            auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
                const bool got = wait_or_abort(bar, parity, ctl);
                return __all_sync(0xffffffffu, got);
            };
            // the stage is free once O of its earlier tile completed (S read
            // its K before)
            auto load = [&](uint32_t n, int t) -> bool {
                const uint32_t st = stage_of(n);
                if (n >= uint32_t(kStages) &&
                    !wait_all(&ctl->st_free[st], stage_parity(n - kStages))) {
                    return false;
                }
                if (lane == 0) {
                    unsigned char* sK = sKV + st * kStageBytes;
                    unsigned char* sV = sK + 2 * kKBytes;
                    const int kbase = t * kKT;
                    const int nvalid = min(kKT, nk - kbase);
                    const int nblk = (nvalid + 15) / 16;
                    uint32_t bytes = 0;
                    for (int j = 0; j < nblk; ++j) {
                        const int64_t blk = table[kbase / 16 + j];
                        if (blk >= 0 && blk < g.num_blocks) bytes += 2u * 4u * 2048u;
                    }
                    mbar_arrive_expect_tx(&ctl->kv_full[st], bytes);
                    for (int j = 0; j < nblk; ++j) {
                        const int64_t blk = table[kbase / 16 + j];
                        if (blk < 0 || blk >= g.num_blocks) {
                            raise_status(kStatusBounds);
                            continue;
                        }
                        const int y = int((blk * g.num_layers + p.layer) * 16);
#pragma unroll
                        for (int a = 0; a < 4; ++a) {
                            const int x = h * kHD + a * 32;
                            tc::tma_load_2d(sK + a * kKVAtom + j * 2048, &kmap, x, y, &ctl->kv_full[st]);
                            tc::tma_load_2d(sV + a * kKVAtom + j * 2048, &vmap, x, y, &ctl->kv_full[st]);
                        }
                    }
                }
                __syncwarp();
                next_load = n + 1;
                return true;
            };
            // once the converters have split tile n's K and V:
            // S(n) = Q_hi K_hi^T + Q_lo K_hi^T + Q_hi K_lo^T
            auto issue_s = [&](uint32_t n) -> bool {
                if (!wait_all(&ctl->cv_full[stage_of(n)], stage_parity(n))) return false;
                next_wait = n + 1;
                if (lane == 0) {
                    tc::fence_after_sync();
                    const uint32_t ka = smem_addr(sKV + stage_of(n) * kStageBytes);
                    const uint32_t kla = ka + kKBytes;
                    const uint32_t ts = tmem + (n & 1u) * kKT;
#pragma unroll
                    for (int k = 0; k < kHD / 8; ++k) {
                        const uint32_t off = (k >> 2) * kKVAtom + (k & 3) * 32u;  // 8 tf32 = 32 B
                        const uint64_t bhi = tc::sw128_desc(ka + off, 16, 1024);
                        const uint64_t blo = tc::sw128_desc(kla + off, 16, 1024);
                        tc::mma_tf32_ts(ts, tmem + kColQlo + 8u * k, bhi, kIdescS, k > 0);
                        tc::mma_tf32_ts(ts, tmem + kColQhi + 8u * k, blo, kIdescS, true);
                        tc::mma_tf32_ts(ts, tmem + kColQhi + 8u * k, bhi, kIdescS, true);
                    }
                    tc::commit(&ctl->s_full[n & 1u]);
                    issued_mma = true;
                }
                __syncwarp();
                return true;
            };
            // O(n) = P_hi V_hi + P_lo V_hi + P_hi V_lo, P from TMEM, V and V_lo
            // from the stage, read MN-major (V lands in the 128-byte swizzle
            // with 32-byte granules): keys 8k..8k+7 start 1 KiB into each
            // 32-dim atom, the atoms of the 128 dims lie 4 KiB apart (leading
            // byte offset), rows go in fours 512 bytes apart (stride byte offset)
            auto issue_o = [&](uint32_t n, bool first) {
                if (lane == 0) {
                    tc::fence_after_sync();
                    const uint32_t va = smem_addr(sKV + stage_of(n) * kStageBytes + 2 * kKBytes);
                    const uint32_t vla = va + kKBytes;
#pragma unroll
                    for (int k = 0; k < kKT / 8; ++k) {
                        const uint64_t vhi = tc::sw128_32b_desc(va + k * 1024u, kKVAtom, 512);
                        const uint64_t vlo = tc::sw128_32b_desc(vla + k * 1024u, kKVAtom, 512);
                        tc::mma_tf32_ts(tO, tmem + kColPlo + 8u * k, vhi, kIdescO, k > 0 || !first);
                        tc::mma_tf32_ts(tO, tmem + kColPhi + 8u * k, vlo, kIdescO, true);
                        tc::mma_tf32_ts(tO, tmem + kColPhi + 8u * k, vhi, kIdescO, true);
                    }
                    tc::commit(&ctl->o_full);
                    tc::commit(&ctl->st_free[stage_of(n)]);
                }
                __syncwarp();
            };

            // S(n+1) is queued while the softmax works on S(n); the stage of
            // tile n-1 is refilled (with tile n+2) once O(n-1) has completed,
            // which it has by then or soon, so that the wait never holds back
            // an MMA that could be queued.
            bool ok = true;
            for (int t = 0; ok && t < min(ntiles, kStages); ++t) ok = load(n0 + t, t);
            if (ok) ok = issue_s(n0);
            for (int t = 0; ok && t < ntiles; ++t) {
                const uint32_t n = n0 + t;
                if (t + 1 < ntiles) {
                    ok = issue_s(n + 1);
                    if (!ok) break;
                }
                if (t >= 1 && t - 1 + kStages < ntiles) {
                    ok = load(n - 1 + kStages, t - 1 + kStages);
                    if (!ok) break;
                }
                ok = wait_all(&ctl->p_full, n & 1u);
                if (!ok) break;
                issue_o(n, t == 0);
            }
        } else if (warp > kProducerWarp) {
            // -------------------------------------------------------------- converters
            // thread c: 4 float4 of K_lo, then 4 float4 of V_lo; V rows of keys
            // past the visible ones (stale rows of the last block, or blocks
            // not loaded) are zeroed in V and V_lo
            const int c = tid - (kSoftmaxThreads + 32);
            for (int t = 0; t < ntiles; ++t) {
                const uint32_t n = n0 + t;
                // wait outcomes are made warp-uniform, so that no lane is left
                // alone in a warp-collective step after another gave up
                if (!__all_sync(0xffffffffu,
                                wait_or_abort(&ctl->kv_full[stage_of(n)], stage_parity(n), ctl))) {
                    break;
                }
                unsigned char* stage = sKV + stage_of(n) * kStageBytes;
                const int nvk = nk - t * kKT;
                const float4* kp = reinterpret_cast<const float4*>(stage);
                float4* klp = reinterpret_cast<float4*>(stage + kKBytes);
                float4* vp = reinterpret_cast<float4*>(stage + 2 * kKBytes);
                float4* vlp = reinterpret_cast<float4*>(stage + 3 * kKBytes);
#pragma unroll
                for (int i = 0; i < int(kKBytes / 16) / kConvThreads; ++i) {
                    const int j = c + i * kConvThreads;
                    const float4 k4 = kp[j];
                    klp[j] = make_float4(tf32_lo(k4.x), tf32_lo(k4.y), tf32_lo(k4.z), tf32_lo(k4.w));
                    // float4 j of the V tile: atom j / 256, key row (j % 256) / 8
                    const int key = (j & 255) >> 3;
                    if (key < nvk) {
                        const float4 v4 = vp[j];
                        vlp[j] = make_float4(tf32_lo(v4.x), tf32_lo(v4.y), tf32_lo(v4.z), tf32_lo(v4.w));
                    } else {
                        vp[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                        vlp[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
                tc::fence_async_smem();
                mbar_arrive(&ctl->cv_full[stage_of(n)]);
            }
        } else {
            // ------------------------------------------------------------ softmax warps
            const int row = tid;  // query row and TMEM lane
            const int qpos = first_pos + r0 + row;
            const uint32_t lane_off = uint32_t(warp * 32) << 16;
            float m_run = -INFINITY, l_run = 0.f;
            bool ok = true;
            for (int t = 0; t < ntiles; ++t) {
                const uint32_t n = n0 + t;
                if (!__all_sync(0xffffffffu, wait_or_abort(&ctl->s_full[n & 1u], (n >> 1) & 1u, ctl))) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                float sc[kKT];
                tc::tmem_ld32(tmem + (n & 1u) * kKT + lane_off, sc);
                tc::tmem_ld_wait();
                const int kbase = t * kKT;
                float cm = -INFINITY;
#pragma unroll
                for (int j = 0; j < kKT; ++j) {
                    const int kp = kbase + j;
                    sc[j] = (kp <= qpos && kp < nk) ? sc[j] * p.qk_scale_log2 : -INFINITY;
                    cm = fmaxf(cm, sc[j]);
                }
                // The row's reference maximum moves only when a score exceeds it
                // by more than kRescaleMargin (log2 units): until then the
                // weights exp2(s - m) stay <= 2^margin, O and l keep their
                // scale, and the rescale of O (a TMEM round trip between one
                // tile's P.V and the next tile's P) is skipped. The reference
                // cancels in O / l, so only rounding differs.
                const float m_new = cm > m_run + kRescaleMargin ? cm : m_run;
                const float alpha = exp2f(m_run - m_new);
                float ps = 0.f;
#pragma unroll
                for (int j = 0; j < kKT; ++j) {
                    sc[j] = exp2f(sc[j] - m_new);
                    ps += sc[j];
                }
                l_run = fmaf(l_run, alpha, ps);
                m_run = m_new;
                if (t > 0) {
                    // previous tile's P.V is in O: P's TMEM columns are free, and O
                    // can be rescaled to the new maximum before this tile's P.V
                    if (!__all_sync(0xffffffffu, wait_or_abort(&ctl->o_full, (n - 1) & 1u, ctl))) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
                        for (int c = 0; c < kHD / 32; ++c) {
                            float ov[32];
                            tc::tmem_ld32(tO + c * 32u + lane_off, ov);
                            tc::tmem_ld_wait();
#pragma unroll
                            for (int j = 0; j < 32; ++j) ov[j] *= alpha;
                            tc::tmem_st32(tO + c * 32u + lane_off, ov);
                        }
                    }
                }
                // P -> this row's TMEM lane as tf32 hi / lo parts (A operand of O)
                {
                    float lo[kKT];
#pragma unroll
                    for (int j = 0; j < kKT; ++j) lo[j] = tf32_lo(sc[j]);
                    tc::tmem_st32(tmem + kColPhi + lane_off, sc);
                    tc::tmem_st32(tmem + kColPlo + lane_off, lo);
                    tc::tmem_st_wait();
                }
                tc::fence_before_sync();
                mbar_arrive(&ctl->p_full);
            }
            if (ok && ntiles > 0) {
                const uint32_t n = n0 + ntiles - 1;
                if (__all_sync(0xffffffffu, wait_or_abort(&ctl->o_full, n & 1u, ctl))) {
                    tc::fence_after_sync();
                    const float inv = 1.0f / fmaxf(l_run, 1e-12f);
                    float4* op = reinterpret_cast<float4*>(p.out + int64_t(q0 + r0 + row) * g.row +
                                                           int64_t(h) * kHD);
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
    if (warp == kProducerWarp && lane == 0) {
        for (uint32_t n = next_wait; n < next_load; ++n) {
            mbar_wait(&ctl->kv_full[stage_of(n)], stage_parity(n), kStatusInPrefillTc);
        }
        if (issued_mma) {
            tc::commit(&ctl->drain);
            mbar_wait(&ctl->drain, 0, kStatusInPrefillTc);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == kProducerWarp) {
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
// block's 16 rows x 32 columns, 128-byte swizzle (16-byte granules for K, the
// K-major operand; 32-byte granules for V, the MN-major one).
bool make_arena_map(CUtensorMap* map, const float* arena, const ArenaGeom& g,
                    CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t dims[2] = {cuuint64_t(g.row),
                                cuuint64_t(g.num_blocks) * g.num_layers * g.block_size};
    const cuuint64_t strides[1] = {cuuint64_t(g.row) * sizeof(float)};
    const cuuint32_t box[2] = {32, 16};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(arena), dims, strides,
              box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool prefill_tc_supported(const ArenaGeom& g) { return g.head_dim == kHD && g.block_size == 16; }

int32_t prefill_tc_tile_rows() { return kQT; }

cudaError_t launch_prefill_tc(const AttnParams& p, cudaStream_t stream, int max_sms) {
    CUtensorMap kmap, vmap;
    if (!make_arena_map(&kmap, p.k_arena, p.g, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_arena_map(&vmap, p.v_arena, p.g, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)) {
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
