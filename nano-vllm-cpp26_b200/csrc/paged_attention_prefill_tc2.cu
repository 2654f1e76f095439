// K3 (TF32 tensor cores, CTA pairs): causal paged prefill attention on
// tcgen05 with cta_group::2.
//
// Same mathematics as src/model.cpp:204-260 for sequences with more than one
// query row, and the same 3xTF32 products as the one-CTA kernel
// (paged_attention_prefill_tc.cu): S = Q_hi K_hi + Q_lo K_hi + Q_hi K_lo and
// O += P_hi V_hi + P_lo V_hi + P_hi V_lo, fp32 accumulation in TMEM, softmax
// in fp32. Geometry: head_dim 128, block size 16.
//
// Why pairs. At one CTA per tile the S tile could only be 32 keys wide (Q hi /
// lo, S, P and O fill the 512 TMEM columns), and a 128 x 32 x 8 MMA costs
// nearly what a 128 x 64 x 8 one does. Two CTAs on two SMs (a cluster of two)
// share one 256-row query tile: CTA r holds rows [128 r, 128 r + 128) in its
// TMEM lanes, and the pair's MMAs, issued by one thread of CTA 0, split the B
// operand by columns, so that each CTA holds only half of every key tile:
//   S  = Q K^T : M 256 x N 64 keys x K 8; CTA r holds keys [32 r, 32 r + 32)
//                of the tile's K (all 128 dims);
//   O += P V   : M 256 x N 128 dims x K 8; CTA r holds dims [64 r, 64 r + 64)
//                of V^T for all 64 keys.
// Each pair MMA does four times the work of the one-CTA kernel's S MMA, and
// each SM stages half of K and half of V per tile. Q_hi moves to shared
// memory (the A operand by descriptor), which frees the TMEM for a 64-wide S.
// TMEM (both CTAs alike): S x2 (2 x 64), P_hi and P_lo (64 each), O (128),
// Q_lo (128). Shared memory: Q_hi 64 KiB, two K / K_lo / V stages of 48 KiB,
// two V^T hi / lo buffers of 32 KiB.
//
// One persistent pair per two SMs, 13 warps per CTA as in the one-CTA kernel:
//   warps 0-3  softmax / epilogue (thread t: query row 128 r + t, TMEM lane t);
//   warp 4     producer: TMA loads of this CTA's K and V boxes into its ring;
//              in CTA 0 also the pair's MMAs and their commits, which arrive
//              on the barriers of both CTAs (tcgen05.commit multicast);
//   warps 5-12 converters: K_lo, and V^T hi / lo of this CTA's dimensions.
// Cross-CTA hand-offs: every converter and softmax warp of both CTAs (one
// lane, after the warp synchronised, so one cluster-scope release per warp)
// arrives on CTA 0's kc_full / vc_full / p_full (K_lo for S,
// V^T for O, P for O, kept apart so that S never waits on a V^T conversion,
// which itself waits for the previous O); the MMA commits come
// back to both CTAs' barriers. No named barrier is used: a thread that gives
// up on a wait must not leave the rest of its group blocked. Every wait is
// bounded (2 s);
// a timeout marks both CTAs aborted, both finish their copies and MMAs, meet
// at a cluster barrier and free their TMEM. No TMA multicast is used.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace nvllm {

namespace {

constexpr int kRows = 128;        // query rows per CTA (TMEM lanes)
constexpr int kQT = 2 * kRows;    // query rows per pair tile
constexpr int kKT = 64;           // keys per tile
constexpr int kKH = kKT / 2;      // keys of K per CTA
constexpr int kHD = 128;
constexpr int kDH = kHD / 2;      // dims of V per CTA
constexpr int kStages = 2;
constexpr int kSoftmaxThreads = 128;  // warps 0-3
constexpr int kProducerWarp = 4;
constexpr int kConvThreads = 256;     // warps 5-12
constexpr int kThreads = kSoftmaxThreads + 32 + kConvThreads;

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;      // S[0] 0..63, S[1] 64..127
constexpr uint32_t kColPhi = 128;
constexpr uint32_t kColPlo = 192;
constexpr uint32_t kColO = 256;
constexpr uint32_t kColQlo = 384;

// Shared memory: 128-byte swizzled K-major atoms (32 fp32 of a row).
constexpr uint32_t kQAtom = kRows * 128;       // 128 rows x 32 dims
constexpr uint32_t kQBytes = 4 * kQAtom;       // Q_hi, 64 KiB
constexpr uint32_t kKAtom = kKH * 128;         // 32 keys x 32 dims
constexpr uint32_t kKBytes = 4 * kKAtom;       // 16 KiB (K or K_lo)
constexpr uint32_t kVAtom = kKT * 128;         // 64 keys x 32 dims
constexpr uint32_t kVBytes = 2 * kVAtom;       // 64 keys x this CTA's 64 dims
constexpr uint32_t kStageBytes = 2 * kKBytes + kVBytes;
constexpr uint32_t kVtAtom = kDH * 128;        // 64 dims x 32 keys
constexpr uint32_t kVtBytes = 2 * kVtAtom;     // 64 dims x 64 keys (hi or lo)
constexpr uint32_t kVtBufBytes = 2 * kVtBytes;
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffKV = kOffQ + kQBytes;
constexpr uint32_t kOffVt = kOffKV + kStages * kStageBytes;
constexpr uint32_t kOffBar = kOffVt + 2 * kVtBufBytes;
constexpr uint32_t kSmemBytes = kOffBar + 512 + 1024;  // + control block + alignment slack
static_assert(kSmemBytes <= 227u * 1024u, "shared memory");

constexpr uint32_t kIdescS = tc::tf32_idesc(kQT, kKT, false, false);
constexpr uint32_t kIdescO = tc::tf32_idesc(kQT, kHD, false, false);
constexpr uint16_t kBoth = 0x3;  // commit to the barriers of both CTAs

struct Control {
    uint64_t kv_full[kStages];  // this CTA's TMA boxes of the stage landed
    uint64_t kc_full[kStages];  // CTA 0: K_lo of the stage written by every converter warp of both CTAs
    uint64_t vread[kStages];    // this CTA's converters done reading the stage's V
    uint64_t pv_done[kStages];  // both: S of the stage's tile done (its K read)
    uint64_t vc_full[2];        // CTA 0: V^T of the buffer written by every converter warp of both CTAs
    uint64_t vt_free[2];        // both: O done with the V^T buffer
    uint64_t s_full[2];         // both: S tile in TMEM
    uint64_t p_full;            // CTA 0: every softmax warp of both CTAs wrote P
    uint64_t o_full;            // both: O of the tile done
    uint64_t drain;             // CTA 0: teardown
    uint32_t tmem_base;
    int32_t item;
    int32_t abort;
};
static_assert(sizeof(Control) <= 512, "control block");

// Marks both CTAs of the pair aborted.
__device__ __forceinline__ void abort_pair(Control* ctl, uint32_t rank) {
    atomicExch(&ctl->abort, 1);
    tc::st_rank_u32(reinterpret_cast<uint32_t*>(&ctl->abort), rank ^ 1u, 1u);
}

// Bounded wait (arrivals may come from the other CTA) that also gives up once
// the pair has aborted.
__device__ __forceinline__ bool wait_pair(uint64_t* bar, uint32_t parity, Control* ctl,
                                          uint32_t rank) {
    if (tc::mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (tc::mbar_try_wait_cluster(bar, parity)) return true;
        if (*reinterpret_cast<volatile int32_t*>(&ctl->abort)) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            raise_status(kStatusTimeout | kStatusInPrefillTc);
            abort_pair(ctl, rank);
            return false;
        }
    }
}

__device__ __forceinline__ float tf32_lo(float x) {
    return x - __uint_as_float(__float_as_uint(x) & 0xffffe000u);
}

#ifndef NVLLM_RESCALE_MARGIN
#define NVLLM_RESCALE_MARGIN 8.0f
#endif
constexpr float kRescaleMargin = NVLLM_RESCALE_MARGIN;

__device__ __forceinline__ uint32_t stage_of(uint32_t n) { return n % kStages; }
__device__ __forceinline__ uint32_t stage_parity(uint32_t n) { return (n / kStages) & 1u; }

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
prefill_tc2_kernel(const AttnParams p, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap) {
    // a decode kernel launched as this kernel's programmatic dependent may start
    // on the SMs this grid leaves free (it reads nothing this kernel writes)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sQ = base + kOffQ;
    unsigned char* sKV = base + kOffKV;
    unsigned char* sVt = base + kOffVt;
    Control* ctl = reinterpret_cast<Control*>(base + kOffBar);
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const uint32_t rank = tc::cluster_rank();
    const bool lead = rank == 0;

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&ctl->kv_full[i], 1);
            mbar_init(&ctl->kc_full[i], 2 * kConvThreads / 32);
            mbar_init(&ctl->vread[i], kConvThreads);
            mbar_init(&ctl->pv_done[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&ctl->vc_full[i], 2 * kConvThreads / 32);
            mbar_init(&ctl->vt_free[i], 1);
            mbar_init(&ctl->s_full[i], 1);
        }
        mbar_init(&ctl->p_full, 2 * kSoftmaxThreads / 32);
        mbar_init(&ctl->o_full, 1);
        mbar_init(&ctl->drain, 1);
        ctl->abort = 0;
    }
    fence_barrier_init();
    if (warp == kProducerWarp) {
        tc::tmem_alloc_pair(&ctl->tmem_base, kTmemCols);
        tc::tmem_relinquish_pair();
    }
    tc::fence_before_sync();
    tc::cluster_sync();  // barriers and TMEM of both CTAs exist before any use
    tc::fence_after_sync();
    const uint32_t tmem = ctl->tmem_base;
    const uint32_t tO = tmem + kColO;

    const ArenaGeom& g = p.g;
    const int H = g.num_heads;
    const int total = p.counters->prefill_items * H;
    uint32_t tile_seq = 0;   // key tiles processed by this pair (ring position)
    uint32_t next_load = 0;  // producer: ring index of the next load to issue
    uint32_t next_wait = 0;  // producer: first load not known to have landed
    bool issued_mma = false;

    for (;;) {
        if (lead && tid == 0) {
            const int it = atomicAdd(&p.counters->prefill_next, 1);
            ctl->item = it;
            tc::st_rank_u32(reinterpret_cast<uint32_t*>(&ctl->item), 1u, uint32_t(it));
        }
        tc::cluster_sync();
        const int it = ctl->item;
        const bool stop = it >= total || *reinterpret_cast<volatile int32_t*>(&ctl->abort);
        if (stop) break;

        const WorkItem wi = p.prefill_items[it / H];
        const int h = it % H;
        const int s = wi.seq;
        const int q0 = p.cu_seqlens_q[s];
        const int qlen = p.cu_seqlens_q[s + 1] - q0;
        const int first_pos = p.context_lens[s] - qlen;
        const int r0 = wi.part * kQT;
        const int nrows = min(kQT, qlen - r0);
        const int nk = first_pos + r0 + nrows;  // keys 0..nk-1 visible to the tile
        const int ntiles = (nk + kKT - 1) / kKT;
        const uint32_t n0 = tile_seq;

        if (tid < kSoftmaxThreads) {
            // This CTA's 128 query rows: Q_hi into the swizzled A atoms, Q_lo
            // into TMEM (rows past the sequence are zero).
            const int row = int(rank) * kRows + tid;
            const uint32_t lane_off = uint32_t(warp * 32) << 16;
            const float4* qrow = reinterpret_cast<const float4*>(
                p.q + int64_t(q0 + r0 + row) * g.row + int64_t(h) * kHD);
#pragma unroll 1
            for (int c = 0; c < kHD / 32; ++c) {
                float lo[32];
                unsigned char* atom = sQ + c * kQAtom + tid * 128;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (row < nrows) v = __ldg(qrow + c * 8 + i);
                    *reinterpret_cast<float4*>(atom + ((i ^ (tid & 7)) * 16)) = v;
                    lo[4 * i + 0] = tf32_lo(v.x);
                    lo[4 * i + 1] = tf32_lo(v.y);
                    lo[4 * i + 2] = tf32_lo(v.z);
                    lo[4 * i + 3] = tf32_lo(v.w);
                }
                tc::tmem_st32(tmem + kColQlo + c * 32u + lane_off, lo);
            }
            tc::tmem_st_wait();
            tc::fence_async_smem();
            tc::fence_before_sync();
        }
        tc::cluster_sync();  // both CTAs' Q in place before the pair's first S
        tc::fence_after_sync();

        if (warp == kProducerWarp) {
            // ---------------------------------------------------------------- producer
            const int32_t* table = p.block_tables + int64_t(s) * p.max_blocks;
            auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
                const bool got = wait_pair(bar, parity, ctl, rank);
                return __all_sync(0xffffffffu, got);
            };
            // This CTA's boxes of key tile t: K of keys [64 t + 32 r, +32) (all
            // dims), V of keys [64 t, +64) (dims [64 r, 64 r + 64)).
            // The stage is free once S read the previous tile's K and this CTA's
            // converters read its V.
            auto load = [&](uint32_t n, int t) -> bool {
                const uint32_t st = stage_of(n);
                if (n >= uint32_t(kStages)) {
                    if (!wait_all(&ctl->pv_done[st], stage_parity(n - kStages))) return false;
                    if (!wait_all(&ctl->vread[st], stage_parity(n - kStages))) return false;
                    next_wait = n - kStages + 1;  // its load had landed (S read it)
                }
                if (lane == 0) {
                    unsigned char* sK = sKV + st * kStageBytes;
                    unsigned char* sV = sK + 2 * kKBytes;
                    const int kb = t * kKT + int(rank) * kKH;
                    const int nkb = max(0, min(kKH, nk - kb) + 15) / 16;
                    const int vb = t * kKT;
                    const int nvb = (min(kKT, nk - vb) + 15) / 16;
                    uint32_t bytes = 0;
                    for (int j = 0; j < nkb; ++j) {
                        const int64_t blk = table[kb / 16 + j];
                        if (blk >= 0 && blk < g.num_blocks) bytes += 4u * 2048u;
                    }
                    for (int j = 0; j < nvb; ++j) {
                        const int64_t blk = table[vb / 16 + j];
                        if (blk >= 0 && blk < g.num_blocks) bytes += 2u * 2048u;
                    }
                    mbar_arrive_expect_tx(&ctl->kv_full[st], bytes);
                    for (int j = 0; j < nkb; ++j) {
                        const int64_t blk = table[kb / 16 + j];
                        if (blk < 0 || blk >= g.num_blocks) {
                            raise_status(kStatusBounds);
                            continue;
                        }
                        const int y = int((blk * g.num_layers + p.layer) * 16);
#pragma unroll
                        for (int a = 0; a < 4; ++a) {
                            tc::tma_load_2d(sK + a * kKAtom + j * 2048, &kmap, h * kHD + a * 32, y,
                                            &ctl->kv_full[st]);
                        }
                    }
                    for (int j = 0; j < nvb; ++j) {
                        const int64_t blk = table[vb / 16 + j];
                        if (blk < 0 || blk >= g.num_blocks) {
                            raise_status(kStatusBounds);
                            continue;
                        }
                        const int y = int((blk * g.num_layers + p.layer) * 16);
#pragma unroll
                        for (int a = 0; a < 2; ++a) {
                            tc::tma_load_2d(sV + a * kVAtom + j * 2048, &vmap,
                                            h * kHD + int(rank) * kDH + a * 32, y, &ctl->kv_full[st]);
                        }
                    }
                }
                __syncwarp();
                next_load = n + 1;
                return true;
            };
            // S(n) = Q_lo K_hi + Q_hi K_lo + Q_hi K_hi, once both CTAs wrote tile
            // n's K_lo (the V^T conversion runs on beside it)
            auto issue_s = [&](uint32_t n) -> bool {
                if (!wait_all(&ctl->kc_full[stage_of(n)], stage_parity(n))) return false;
                if (lane == 0) {
                    tc::fence_after_sync();
                    const uint32_t qa = smem_addr(sQ);
                    const uint32_t ka = smem_addr(sKV + stage_of(n) * kStageBytes);
                    const uint32_t kla = ka + kKBytes;
                    const uint32_t ts = tmem + kColS + (n & 1u) * kKT;
#pragma unroll
                    for (int k = 0; k < kHD / 8; ++k) {
                        const uint32_t off_q = (k >> 2) * kQAtom + (k & 3) * 32u;
                        const uint32_t off_k = (k >> 2) * kKAtom + (k & 3) * 32u;
                        const uint64_t qhi = tc::sw128_desc(qa + off_q, 16, 1024);
                        const uint64_t khi = tc::sw128_desc(ka + off_k, 16, 1024);
                        const uint64_t klo = tc::sw128_desc(kla + off_k, 16, 1024);
                        tc::mma_tf32_pair_ts(ts, tmem + kColQlo + 8u * k, khi, kIdescS, k > 0);
                        tc::mma_tf32_pair(ts, qhi, klo, kIdescS, true);
                        tc::mma_tf32_pair(ts, qhi, khi, kIdescS, true);
                    }
                    tc::commit_pair(&ctl->s_full[n & 1u], kBoth);
                    tc::commit_pair(&ctl->pv_done[stage_of(n)], kBoth);
                    issued_mma = true;
                }
                __syncwarp();
                return true;
            };
            // O(n) += P_lo V_hi + P_hi V_lo + P_hi V_hi, P from TMEM, V^T from
            // the buffer the converters filled for tile n
            auto issue_o = [&](uint32_t n, bool first) {
                if (lane == 0) {
                    tc::fence_after_sync();
                    const uint32_t va = smem_addr(sVt + (n & 1u) * kVtBufBytes);
#pragma unroll
                    for (int k = 0; k < kKT / 8; ++k) {
                        const uint32_t off = (k >> 2) * kVtAtom + (k & 3) * 32u;
                        const uint64_t vhi = tc::sw128_desc(va + off, 16, 1024);
                        const uint64_t vlo = tc::sw128_desc(va + kVtBytes + off, 16, 1024);
                        tc::mma_tf32_pair_ts(tO, tmem + kColPlo + 8u * k, vhi, kIdescO,
                                             k > 0 || !first);
                        tc::mma_tf32_pair_ts(tO, tmem + kColPhi + 8u * k, vlo, kIdescO, true);
                        tc::mma_tf32_pair_ts(tO, tmem + kColPhi + 8u * k, vhi, kIdescO, true);
                    }
                    tc::commit_pair(&ctl->o_full, kBoth);
                    tc::commit_pair(&ctl->vt_free[n & 1u], kBoth);
                }
                __syncwarp();
            };

            bool ok = true;
            for (int t = 0; ok && t < min(ntiles, kStages); ++t) ok = load(n0 + t, t);
            if (lead) {
                // S(n+1) is queued behind S(n), the load of tile n+2 goes out as
                // soon as its stage is free (while the softmax works on S(n)),
                // then O(n) once P(n) and V^T(n) are in place.
                if (ok) ok = issue_s(n0);
                for (int t = 0; ok && t < ntiles; ++t) {
                    const uint32_t n = n0 + t;
                    if (t + 1 < ntiles) {
                        ok = issue_s(n + 1);
                        if (!ok) break;
                    }
                    if (t + kStages < ntiles) {
                        ok = load(n + kStages, t + kStages);
                        if (!ok) break;
                    }
                    ok = wait_all(&ctl->vc_full[n & 1u], (n >> 1) & 1u) &&
                         wait_all(&ctl->p_full, n & 1u);
                    if (!ok) break;
                    issue_o(n, t == 0);
                }
            } else {
                for (int t = kStages; ok && t < ntiles; ++t) ok = load(n0 + t, t);
            }
            if (ok) next_wait = next_load;  // every load of the item was consumed
        } else if (warp > kProducerWarp) {
            // -------------------------------------------------------------- converters
            // thread c: 4 float4 of K_lo; then dim d = c % 64 of this CTA's V
            // half, keys 16 * (c / 64) .. +15 of V^T row d
            const int c = tid - (kSoftmaxThreads + 32);
            const int d = c & (kDH - 1);
            const int kq = c >> 6;
            const int dd = d & 31;
            bool ok = true;
            for (int t = 0; t < ntiles; ++t) {
                const uint32_t n = n0 + t;
                // every wait's outcome is made warp-uniform, so that no lane
                // is left alone in a warp-collective step after another gave up
                if (!__all_sync(0xffffffffu,
                                wait_pair(&ctl->kv_full[stage_of(n)], stage_parity(n), ctl, rank))) {
                    ok = false;
                    break;
                }
                unsigned char* stage = sKV + stage_of(n) * kStageBytes;
                {
                    const float4* kp = reinterpret_cast<const float4*>(stage);
                    float4* klp = reinterpret_cast<float4*>(stage + kKBytes);
#pragma unroll
                    for (int i = 0; i < int(kKBytes / 16) / kConvThreads; ++i) {
                        const int j = c + i * kConvThreads;
                        const float4 v = kp[j];
                        klp[j] = make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
                    }
                }
                tc::fence_async_smem();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive_rank(&ctl->kc_full[stage_of(n)], 0);
                if (n >= 2 && !__all_sync(0xffffffffu, wait_pair(&ctl->vt_free[n & 1u],
                                                                  ((n >> 1) - 1) & 1u, ctl, rank))) {
                    ok = false;
                    break;
                }
                unsigned char* vt = sVt + (n & 1u) * kVtBufBytes;
                const int nvk = nk - t * kKT;  // keys of this tile that are visible
                const unsigned char* sV = stage + 2 * kKBytes + (d >> 5) * kVAtom + (dd & 3) * 4;
#pragma unroll
                for (int q = 4 * kq; q < 4 * kq + 4; ++q) {
                    float hi[4], lo[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int k = 4 * q + e;
                        const float x = k < nvk ? *reinterpret_cast<const float*>(
                                                      sV + k * 128 + (((dd >> 2) ^ (k & 7)) * 16))
                                                : 0.f;
                        hi[e] = x;
                        lo[e] = tf32_lo(x);
                    }
                    unsigned char* row = vt + (q >> 3) * kVtAtom + d * 128;
                    const int pos = (q & 7) ^ (d & 7);
                    *reinterpret_cast<float4*>(row + pos * 16) = make_float4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<float4*>(row + kVtBytes + pos * 16) =
                        make_float4(lo[0], lo[1], lo[2], lo[3]);
                }
                mbar_arrive(&ctl->vread[stage_of(n)]);  // this stage's V is no longer read
                tc::fence_async_smem();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive_rank(&ctl->vc_full[n & 1u], 0);
            }
            (void)ok;
        } else {
            // ------------------------------------------------------------ softmax warps
            const int row = int(rank) * kRows + tid;  // query row of the tile; TMEM lane tid
            const int qpos = first_pos + r0 + row;
            const uint32_t lane_off = uint32_t(warp * 32) << 16;
            float m_run = -INFINITY, l_run = 0.f;
            bool ok = true;
            for (int t = 0; t < ntiles; ++t) {
                const uint32_t n = n0 + t;
                if (!__all_sync(0xffffffffu,
                                wait_pair(&ctl->s_full[n & 1u], (n >> 1) & 1u, ctl, rank))) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                float sc[kKT];
                tc::tmem_ld32(tmem + kColS + (n & 1u) * kKT + lane_off, sc);
                tc::tmem_ld32(tmem + kColS + (n & 1u) * kKT + 32u + lane_off, sc + 32);
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
                    // the previous tile's P.V is in O: P's TMEM columns are free,
                    // and O can be rescaled to the new maximum
                    if (!__all_sync(0xffffffffu, wait_pair(&ctl->o_full, (n - 1) & 1u, ctl, rank))) {
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
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float lo[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) lo[j] = tf32_lo(sc[32 * half + j]);
                    tc::tmem_st32(tmem + kColPhi + 32u * half + lane_off, sc + 32 * half);
                    tc::tmem_st32(tmem + kColPlo + 32u * half + lane_off, lo);
                }
                tc::tmem_st_wait();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive_rank(&ctl->p_full, 0);
            }
            if (ok && ntiles > 0) {
                const uint32_t n = n0 + ntiles - 1;
                if (__all_sync(0xffffffffu, wait_pair(&ctl->o_full, n & 1u, ctl, rank))) {
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

    // Teardown: on an abort, let this CTA's copies and the pair's MMAs finish
    // (bounded) before either CTA's shared memory and TMEM are released.
    if (warp == kProducerWarp && lane == 0) {
        for (uint32_t n = next_wait; n < next_load; ++n) {
            mbar_wait(&ctl->kv_full[stage_of(n)], stage_parity(n), kStatusInPrefillTc);
        }
        if (lead && issued_mma) {
            tc::commit_pair(&ctl->drain, 0x1);
            mbar_wait(&ctl->drain, 0, kStatusInPrefillTc);
        }
    }
    tc::fence_before_sync();
    tc::cluster_sync();
    if (warp == kProducerWarp) {
        __syncwarp();
        tc::fence_after_sync();
        tc::tmem_dealloc_pair(tmem, kTmemCols);
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

int32_t prefill_tc2_tile_rows() { return kQT; }

cudaError_t launch_prefill_tc2(const AttnParams& p, cudaStream_t stream, int max_sms) {
    CUtensorMap kmap, vmap;
    if (!make_arena_map(&kmap, p.k_arena, p.g) || !make_arena_map(&vmap, p.v_arena, p.g)) {
        return cudaErrorInvalidValue;
    }
    static int pairs_per_device[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (pairs_per_device[dev] == 0) {
        e = cudaFuncSetAttribute(prefill_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(kSmemBytes));
        if (e != cudaSuccess) return e;
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        pairs_per_device[dev] = std::max(1, sms / 2);  // one CTA per SM
    }
    int pairs = pairs_per_device[dev];
    if (max_sms > 0) pairs = std::max(1, std::min(pairs, max_sms / 2));
    prefill_tc2_kernel<<<2 * pairs, kThreads, kSmemBytes, stream>>>(p, kmap, vmap);
    return cudaGetLastError();
}

}  // namespace nvllm
