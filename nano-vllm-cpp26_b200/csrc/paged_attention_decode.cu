// K0 plan + K2 split-K paged decode attention + merge (sm_100a).
//
// Replaces step 3d of TransformerModel::forward_batch (src/model.cpp:204-260)
// for sequences with one query row. For token t of sequence s at position
// p = ctx - 1 and head h the reference walks the block table
// (:225-253): score = (q . k) * scale, online max / sum rescaling, V
// accumulation, then out /= max(sum, 1e-12) (:255-258).
//
// B200 design (HBM-bound, ~0.25 FLOP/byte):
//  * The context of each (sequence, head) is cut into items of P positions
//    (decode_split_tokens); a persistent grid of warps pulls (item, head)
//    pairs from a global cursor, so every SM streams until the whole batch is
//    done and ragged contexts balance themselves.
//  * Each warp owns a ring of NS shared-memory stages and streams chunks of
//    T = 2048 / hd consecutive positions through it without a bubble between
//    items: while it computes item i it already fetches item i + 1's index and
//    metadata and issues its first chunks. A chunk's K rows and V rows arrive
//    by bulk asynchronous copies (TMA engine, cp.async.bulk, one arena row of
//    hd floats each) completing on the stage's mbarrier; an item's Q row rides
//    on its first chunk's barrier. With block size 16 at hd 128 a chunk is one
//    physical block, so one block-table entry per chunk is held in a lane
//    register for the whole item.
//  * Rows are padded by 16 bytes in shared memory so both the row-per-lane
//    QK^T reads and the column-per-lane PV reads are free of bank conflicts.
//  * QK^T: each lane computes 64-dim partial dots of its rows (two lanes per
//    row at hd 128), shuffles complete them. Softmax runs in the log2 domain
//    (scores times scale*log2 e, exp2f). PV: each lane owns 4 (or 8) output
//    columns.
//  * Latency, not bandwidth, bounds a single warp (one chunk's dependent
//    shuffle / exp / FMA chain), so a CTA holds several warps with shallow
//    rings (NVLLM_DECODE_NW x NVLLM_DECODE_NS) rather than one deep ring.
//  * An item that covers the whole context writes the normalised output; other
//    items write (m, l, acc) partials that the merge kernel combines with the
//    usual max-rescaled sum.
#include <algorithm>
#include <cfloat>

#include "common.cuh"
#include "kernels.cuh"

namespace nvllm {

__device__ uint32_t g_status = 0;
__device__ uint32_t g_timeout_info[4] = {0, 0, 0, 0};

namespace {

template <int HD>
struct DecodeShape {
    static constexpr int T = 2048 / HD;                      // positions per chunk
    static constexpr int ROW = HD + 4;                       // padded smem row (floats)
    static constexpr int PPR = HD >= 128 ? HD / 64 : 1;      // QK lanes per row
    static constexpr int RLANES = 32 / PPR;                  // rows covered per pass
    static constexpr int RPL = T / RLANES;                   // rows per lane (QK)
    static constexpr int DPP = HD / PPR;                     // dims per lane per row
    static constexpr int G = HD >= 128 ? 32 : HD / 4;        // PV lanes per row
    static constexpr int RG = 32 / G;                        // PV row groups
    static constexpr int CPL = HD >= 256 ? HD / 128 : 1;     // float4 columns per lane
    static constexpr int RPG = T / RG;                       // rows per PV group
    static constexpr int COPY_FLOATS = HD < 128 ? HD : 128;  // one bulk copy
    static constexpr int COPY_BYTES = COPY_FLOATS * 4;
    static constexpr int CPR = HD / COPY_FLOATS;             // copies per row
    static constexpr int NCOPIES = 2 * T * CPR;              // K + V copies per chunk
    static constexpr int COPIES_PER_LANE = NCOPIES / 32;
    static constexpr int STAGE_FLOATS = 2 * T * ROW + T;     // K, V, P
    static_assert(NCOPIES % 32 == 0, "copy count must fill the warp");
    static_assert(RPG % 4 == 0, "P reads are float4");
    static_assert((STAGE_FLOATS * 4) % 16 == 0, "stage alignment");
};

constexpr int kBarBytes = 1024;  // mbarriers live in the first KiB of shared memory

// Per-warp shared memory: NS stages plus two Q rows (current / next item).
template <int HD, int NS>
constexpr size_t decode_warp_floats() {
    return size_t(NS) * DecodeShape<HD>::STAGE_FLOATS + 2 * HD;
}

template <int HD, int NW, int NS>
constexpr size_t decode_smem_bytes() {
    return kBarBytes + size_t(NW) * decode_warp_floats<HD, NS>() * sizeof(float);
}

// One decode work item: positions [pos0, pos1) of head h of sequence s.
struct DecodeItem {
    int s;  // < 0: none
    int h;
    int part;
    int pos0;
    int pos1;
    int nchunks;
    int tok;
    bool whole;  // covers the whole context: write the normalised output
};

template <int HD>
__device__ __forceinline__ DecodeItem load_decode_item(const AttnParams& p, int it, int total) {
    using S = DecodeShape<HD>;
    DecodeItem d;
    d.s = -1;
    if (it >= total) return d;
    const int H = p.g.num_heads;
    const WorkItem wi = p.decode_items[it / H];
    d.s = wi.seq;
    d.h = it % H;
    d.part = wi.part;
    const int ctx = p.context_lens[d.s];
    d.pos0 = wi.part * p.split_tokens;
    d.pos1 = min(d.pos0 + p.split_tokens, ctx);
    d.nchunks = (d.pos1 - d.pos0 + S::T - 1) / S::T;
    d.tok = p.cu_seqlens_q[d.s];
    d.whole = d.pos0 == 0 && d.pos1 == ctx;
    return d;
}

// kB16: the arena's block size is 16 and equals the chunk (hd 128), so a chunk
// is one physical block: one table entry per chunk, held in a lane register
// for the whole item. Otherwise every row looks its block up.
template <int HD, int NW, int NS, bool kB16>
__global__ void __launch_bounds__(NW * 32, 1) decode_kernel(const AttnParams p) {
    using S = DecodeShape<HD>;
    static_assert(NW * NS * 8 <= kBarBytes, "barrier area");
    static_assert(!kB16 || S::T == 16, "block-16 path needs 16-position chunks");
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw) + warp * NS;
    float* wbuf = reinterpret_cast<float*>(smem_raw + kBarBytes) +
                  size_t(warp) * decode_warp_floats<HD, NS>();
    float* qbuf = wbuf + NS * S::STAGE_FLOATS;  // two Q rows

    // Zero this warp's stages once: rows past the end of a chunk then always
    // hold finite data (zeros or an earlier chunk), so their zero softmax
    // weight cancels them exactly in PV.
    for (int i = lane * 4; i < NS * S::STAGE_FLOATS; i += 128) {
        *reinterpret_cast<float4*>(wbuf + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (lane == 0) {
        for (int i = 0; i < NS; ++i) mbar_init(&bars[i], 1);
    }
    fence_barrier_init();
    __syncwarp();
    pdl_release();
    // the work list, the arena rows and the queries come from the kernels
    // before (beside a prefill, which writes none of them, the plan completed
    // before the prefill started)
    if (!p.beside_prefill) pdl_wait();

    const uint64_t pol = l2_evict_first();
    const ArenaGeom& g = p.g;
    const int H = g.num_heads;
    const int total = p.counters->decode_items * H;
    const int part = lane / S::RLANES;
    const int rl = lane % S::RLANES;
    const int rg = lane / S::G;
    const int cg = lane % S::G;

    auto fetch_index = [&]() {
        int v = 0;
        if (lane == 0) v = atomicAdd(&p.counters->decode_next, 1);
        return __shfl_sync(0xffffffffu, v, 0);
    };
    auto table_of = [&](const DecodeItem& d) -> const int32_t* {
        return p.block_tables + int64_t(d.s) * p.max_blocks;
    };
    // lane l holds the block id of chunk l of the item (block-16 path)
    auto load_lane_block = [&](const DecodeItem& d) -> int {
        if (!kB16 || lane >= d.nchunks) return 0;
        return table_of(d)[d.pos0 / 16 + lane];
    };

    // Issue chunk c of item d into stage `stage`; the item's Q row rides on
    // the first chunk's barrier.
    auto issue = [&](const DecodeItem& d, int c, int stage, int lane_blk, int qslot) {
        float* sK = wbuf + stage * S::STAGE_FLOATS;
        float* sV = sK + S::T * S::ROW;
        const int cpos = d.pos0 + c * S::T;
        const int nvalid = min(S::T, d.pos1 - cpos);
        const int64_t head_off = int64_t(p.layer) * g.layer_stride + int64_t(d.h) * HD;
        const bool first = c == 0;
        if constexpr (kB16) {
            const int64_t blk = __shfl_sync(0xffffffffu, lane_blk, c);
            const bool blk_ok = blk >= 0 && blk < g.num_blocks;
            if (!blk_ok && lane == 0) raise_status(kStatusBounds);
            const uint32_t bytes = (blk_ok ? uint32_t(nvalid) * HD * 4u * 2u : 0u) +
                                   (first ? HD * 4u : 0u);
            if (lane == 0) mbar_arrive_expect_tx(&bars[stage], bytes);
            __syncwarp();
            if (first && lane == 0) {
                bulk_copy_g2s(qbuf + qslot * HD, p.q + int64_t(d.tok) * g.row + int64_t(d.h) * HD,
                              HD * 4, &bars[stage], pol);
            }
            // lanes 0..15: K rows, lanes 16..31: V rows
            const int tensor = lane / S::T;
            const int row = lane % S::T;
            if (blk_ok && row < nvalid) {
                const int64_t off = blk * g.block_stride + head_off + int64_t(row) * g.row;
                bulk_copy_g2s((tensor ? sV : sK) + row * S::ROW, (tensor ? p.v_arena : p.k_arena) + off,
                              HD * 4, &bars[stage], pol);
            }
        } else {
            const int32_t* table = table_of(d);
            const float* src[S::COPIES_PER_LANE];
            float* dst[S::COPIES_PER_LANE];
            bool ok[S::COPIES_PER_LANE];
            uint32_t bytes = 0;
#pragma unroll
            for (int k = 0; k < S::COPIES_PER_LANE; ++k) {
                const int ci = lane + 32 * k;
                const int tensor = ci / (S::T * S::CPR);
                const int rem = ci % (S::T * S::CPR);
                const int row = rem / S::CPR;
                const int piece = rem % S::CPR;
                const int pos = cpos + row;
                ok[k] = row < nvalid;
                int64_t blk = 0;
                if (ok[k]) {
                    blk = table[pos / g.block_size];
                    if (blk < 0 || blk >= g.num_blocks) {
                        ok[k] = false;
                        raise_status(kStatusBounds);
                    }
                }
                const int64_t off = blk * g.block_stride + head_off +
                                    int64_t(pos % g.block_size) * g.row + piece * S::COPY_FLOATS;
                src[k] = (tensor ? p.v_arena : p.k_arena) + off;
                dst[k] = (tensor ? sV : sK) + row * S::ROW + piece * S::COPY_FLOATS;
                bytes += ok[k] ? S::COPY_BYTES : 0u;
            }
            bytes = __reduce_add_sync(0xffffffffu, bytes) + (first ? HD * 4u : 0u);
            if (lane == 0) mbar_arrive_expect_tx(&bars[stage], bytes);
            __syncwarp();
            if (first && lane == 0) {
                bulk_copy_g2s(qbuf + qslot * HD, p.q + int64_t(d.tok) * g.row + int64_t(d.h) * HD,
                              HD * 4, &bars[stage], pol);
            }
#pragma unroll
            for (int k = 0; k < S::COPIES_PER_LANE; ++k) {
                if (ok[k]) bulk_copy_g2s(dst[k], src[k], S::COPY_BYTES, &bars[stage], pol);
            }
        }
    };

    // ---- streaming state ---------------------------------------------------
    int next_it = fetch_index();
    DecodeItem L = load_decode_item<HD>(p, next_it, total);  // item being issued
    if (L.s < 0) return;
    next_it = fetch_index();
    int lane_blk = load_lane_block(L);
    DecodeItem C = L;          // item being computed
    bool c_live = true;        // C still has chunks to compute
    bool ahead = false;        // L is the item after C
    bool exhausted = false;    // no further items
    int lc = 0;                // next chunk of L to issue
    int cc = 0;                // next chunk of C to compute
    uint32_t issued = 0, consumed = 0;
    uint32_t l_index = 0, c_index = 0;  // items fetched / computed (Q slot parity)

    float m_run = -INFINITY;
    float l_run = 0.f;
    float4 acc[S::CPL];
#pragma unroll
    for (int c = 0; c < S::CPL; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 qv[S::DPP / 4];

    for (;;) {
        // keep the ring full, running at most one item ahead of the compute
        while (issued - consumed < uint32_t(NS)) {
            if (lc == L.nchunks) {
                if (ahead || exhausted) break;
                const DecodeItem nx = load_decode_item<HD>(p, next_it, total);
                if (nx.s < 0) {
                    exhausted = true;
                    break;
                }
                next_it = fetch_index();
                L = nx;
                lane_blk = load_lane_block(L);
                lc = 0;
                ++l_index;
                if (c_live) {
                    ahead = true;
                } else {
                    C = L;
                    c_live = true;
                }
            }
            issue(L, lc, int(issued % NS), lane_blk, int(l_index & 1u));
            ++lc;
            ++issued;
        }
        if (consumed == issued) break;

        const int stage = int(consumed % NS);
        if (!mbar_wait(&bars[stage], (consumed / NS) & 1u, kStatusInDecode)) {
            // let this warp's other copies land (bounded), then stop
            for (uint32_t n = consumed + 1; n < issued; ++n) mbar_wait(&bars[n % NS], (n / NS) & 1u, kStatusInDecode);
            return;
        }
        if (cc == 0) {
            const float4* qs = reinterpret_cast<const float4*>(qbuf + (c_index & 1u) * HD + part * S::DPP);
#pragma unroll
            for (int i = 0; i < S::DPP / 4; ++i) qv[i] = qs[i];
        }
        const float* sK = wbuf + stage * S::STAGE_FLOATS;
        const float* sV = sK + S::T * S::ROW;
        float* sP = const_cast<float*>(sV) + S::T * S::ROW;
        const int nvalid = min(S::T, C.pos1 - (C.pos0 + cc * S::T));

        // scores of this chunk (log2 domain)
        float sc[S::RPL];
#pragma unroll
        for (int k = 0; k < S::RPL; ++k) {
            const int r = rl + k * S::RLANES;
            const float* kr = sK + r * S::ROW + part * S::DPP;
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
            for (int i = 0; i < S::DPP / 4; ++i) {
                const float4 kv = ld_shared4(kr + 4 * i);
                a0 = fmaf(qv[i].x, kv.x, a0);
                a1 = fmaf(qv[i].y, kv.y, a1);
                a2 = fmaf(qv[i].z, kv.z, a2);
                a3 = fmaf(qv[i].w, kv.w, a3);
            }
            float d = (a0 + a1) + (a2 + a3);
#pragma unroll
            for (int o = S::RLANES; o < 32; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            sc[k] = r < nvalid ? d * p.qk_scale_log2 : -INFINITY;
        }
        float cm = sc[0];
#pragma unroll
        for (int k = 1; k < S::RPL; ++k) cm = fmaxf(cm, sc[k]);
        cm = warp_max_xor(cm, S::RLANES);
        const float m_new = fmaxf(m_run, cm);
        const float alpha = exp2f(m_run - m_new);
        float psum = 0.f;
#pragma unroll
        for (int k = 0; k < S::RPL; ++k) {
            const float pk = exp2f(sc[k] - m_new);
            psum += pk;
            if (part == 0) {
                const int r = rl + k * S::RLANES;
                sP[(r % S::RG) * S::RPG + r / S::RG] = pk;
            }
        }
        l_run = fmaf(l_run, alpha, psum);
        __syncwarp();
#pragma unroll
        for (int c = 0; c < S::CPL; ++c) {
            acc[c].x *= alpha;
            acc[c].y *= alpha;
            acc[c].z *= alpha;
            acc[c].w *= alpha;
        }
#pragma unroll
        for (int i4 = 0; i4 < S::RPG / 4; ++i4) {
            const float4 pp = ld_shared4(sP + rg * S::RPG + 4 * i4);
            const float pj[4] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = rg + S::RG * (4 * i4 + j);
#pragma unroll
                for (int c = 0; c < S::CPL; ++c) {
                    const float4 vv = ld_shared4(sV + r * S::ROW + (cg + 32 * c) * 4);
                    acc[c].x = fmaf(pj[j], vv.x, acc[c].x);
                    acc[c].y = fmaf(pj[j], vv.y, acc[c].y);
                    acc[c].z = fmaf(pj[j], vv.z, acc[c].z);
                    acc[c].w = fmaf(pj[j], vv.w, acc[c].w);
                }
            }
        }
        m_run = m_new;
        __syncwarp();  // stage free for the next issue
        ++consumed;
        ++cc;
        if (cc < C.nchunks) continue;

        // ---- item epilogue ---------------------------------------------------
        const float l_tot = warp_sum_xor(l_run, S::RLANES);
#pragma unroll
        for (int o = S::G; o < 32; o <<= 1) {
#pragma unroll
            for (int c = 0; c < S::CPL; ++c) {
                acc[c].x += __shfl_xor_sync(0xffffffffu, acc[c].x, o);
                acc[c].y += __shfl_xor_sync(0xffffffffu, acc[c].y, o);
                acc[c].z += __shfl_xor_sync(0xffffffffu, acc[c].z, o);
                acc[c].w += __shfl_xor_sync(0xffffffffu, acc[c].w, o);
            }
        }
        if (rg == 0) {
            if (C.whole && p.num_outs == 0) {
                const float inv = 1.0f / fmaxf(l_tot, 1e-12f);
                float* op = p.out + int64_t(C.tok) * g.row + int64_t(C.h) * HD;
#pragma unroll
                for (int c = 0; c < S::CPL; ++c) {
                    const float4 v = make_float4(acc[c].x * inv, acc[c].y * inv, acc[c].z * inv,
                                                 acc[c].w * inv);
                    reinterpret_cast<float4*>(op)[cg + 32 * c] = v;
                }
            } else {
                const int64_t pi = (int64_t(C.s) * H + C.h) * p.max_splits + C.part;
                float* ap = p.part_acc + pi * HD;
#pragma unroll
                for (int c = 0; c < S::CPL; ++c) reinterpret_cast<float4*>(ap)[cg + 32 * c] = acc[c];
                if (lane == 0) p.part_ml[pi] = make_float2(m_run, l_tot);
            }
        }
        m_run = -INFINITY;
        l_run = 0.f;
#pragma unroll
        for (int c = 0; c < S::CPL; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
        cc = 0;
        ++c_index;
        if (ahead) {
            C = L;
            ahead = false;
        } else {
            c_live = false;
        }
    }
}

// Combines the split partials of each (decode sequence, head):
// M = max m_j, L = sum l_j 2^(m_j - M), out = sum acc_j 2^(m_j - M) / L.
// A CTA of 8 warps serves 8 / wpr rows; the wpr warps of a row take
// contiguous runs of its splits (loads unrolled four deep, so that a long run
// is not a chain of dependent global loads) and combine their sums through
// shared memory. wpr grows with the split count (merge_warps_per_row), and
// the arithmetic depends only on it and the split size, not on the number of
// heads or sequences in the batch.
template <int HD>
__global__ void __launch_bounds__(256) merge_kernel(const AttnParams p, int wpr) {
    constexpr int PER_LANE = HD / 32;
    __shared__ float sm_m[8], sm_l[8];
    __shared__ float sm_o[8][HD];
    pdl_release();
    pdl_wait();  // the partials of the decode kernel
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int H = p.g.num_heads;
    const int row = blockIdx.x * (8 / wpr) + warp / wpr;
    const int sub = warp % wpr;
    const int lead = warp - sub;  // first warp of this row
    bool active = row < p.num_seqs * H;
    int s = 0, h = 0, q0 = 0, nsplit = 0;
    if (active) {
        s = row / H;
        h = row % H;
        q0 = p.cu_seqlens_q[s];
        const int ctx = p.context_lens[s];
        active = q0 >= 0 && p.cu_seqlens_q[s + 1] - q0 == 1 && ctx >= 1 &&
                 ctx <= p.max_context_len &&
                 int64_t(ctx) <= int64_t(p.max_blocks) * p.g.block_size;
        if (active) nsplit = (ctx + p.split_tokens - 1) / p.split_tokens;
        // one split: the decode kernel wrote the row itself, unless it must go to peers
        if (nsplit <= 1 && p.num_outs == 0) active = false;
    }
    const int per = (nsplit + wpr - 1) / wpr;
    const int j0 = min(nsplit, sub * per);
    const int j1 = min(nsplit, j0 + per);
    const int64_t pbase = (int64_t(s) * H + h) * p.max_splits;
    float M = -INFINITY;
    if (active) {
        for (int j = j0 + lane; j < j1; j += 32) M = fmaxf(M, __ldcg(&p.part_ml[pbase + j].x));
        M = warp_max_xor(M, 32);
    }
    if (lane == 0) sm_m[warp] = M;
    __syncthreads();
    if (active) {
        for (int w = lead; w < lead + wpr; ++w) M = fmaxf(M, sm_m[w]);
    }
    float L = 0.f;
    float o[PER_LANE];
#pragma unroll
    for (int k = 0; k < PER_LANE; ++k) o[k] = 0.f;
    if (active) {
        for (int j = j0 + lane; j < j1; j += 32) {
            const float2 ml = __ldcg(&p.part_ml[pbase + j]);
            L += ml.y * exp2f(ml.x - M);
        }
        L = warp_sum_xor(L, 32);
        int j = j0;
        for (; j + 4 <= j1; j += 4) {
            float w[4];
            float a[4][PER_LANE];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                w[u] = __ldcg(&p.part_ml[pbase + j + u].x);
                const float* ap = p.part_acc + (pbase + j + u) * HD;
#pragma unroll
                for (int k = 0; k < PER_LANE; ++k) a[u][k] = __ldcg(ap + lane + 32 * k);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float wu = exp2f(w[u] - M);
#pragma unroll
                for (int k = 0; k < PER_LANE; ++k) o[k] = fmaf(wu, a[u][k], o[k]);
            }
        }
        for (; j < j1; ++j) {
            const float wu = exp2f(__ldcg(&p.part_ml[pbase + j].x) - M);
            const float* ap = p.part_acc + (pbase + j) * HD;
#pragma unroll
            for (int k = 0; k < PER_LANE; ++k) o[k] = fmaf(wu, __ldcg(ap + lane + 32 * k), o[k]);
        }
    }
    if (wpr > 1) {
        if (lane == 0) sm_l[warp] = L;
#pragma unroll
        for (int k = 0; k < PER_LANE; ++k) sm_o[warp][lane + 32 * k] = o[k];
        __syncthreads();
        if (sub != 0) return;
        for (int w = lead + 1; w < lead + wpr; ++w) {
            L += sm_l[w];
#pragma unroll
            for (int k = 0; k < PER_LANE; ++k) o[k] += sm_o[w][lane + 32 * k];
        }
    }
    if (!active) return;
    const float inv = 1.0f / fmaxf(L, 1e-12f);
    if (p.num_outs == 0) {
        float* op = p.out + int64_t(q0) * p.g.row + int64_t(h) * HD;
#pragma unroll
        for (int k = 0; k < PER_LANE; ++k) op[lane + 32 * k] = o[k] * inv;
        return;
    }
    // head split: store the row into every rank's output buffer (peer memory
    // over NVLink), then the writer of this rank's last row signals all ranks
    for (int r = 0; r < p.num_outs; ++r) {
        float* op = p.outs[r] + int64_t(q0) * p.out_stride + p.out_col + int64_t(h) * HD;
#pragma unroll
        for (int k = 0; k < PER_LANE; ++k) op[lane + 32 * k] = o[k] * inv;
    }
    __threadfence_system();
    __syncwarp();
    if (lane == 0) {
        const int prev = atomicAdd(&p.counters->rows_done, 1);
        if (prev + 1 == p.counters->decode_seqs * H) {
            __threadfence_system();
            for (int r = 0; r < p.num_outs; ++r) atomicAdd_system(p.flags[r], 1u);
        }
    }
}

// Warps that share one row's partials in the merge: 1 up to 16 splits, then
// doubling up to 8 (a CTA's warps) from 128 splits.
int merge_warps_per_row(int max_splits) {
    int w = 1;
    while (w < 8 && max_splits > 16 * w) w *= 2;
    return w;
}

// Head split with nothing to store: signal every rank directly.
__global__ void signal_kernel(AttnParams p) {
    if (threadIdx.x != 0) return;
    __threadfence_system();
    for (int r = 0; r < p.num_outs; ++r) atomicAdd_system(p.flags[r], 1u);
}

// Head split: the call completes once every rank has signalled this rank.
// It may start while this rank's merge still runs (the flag only reaches the
// target once that merge has signalled too), and completes after it.
__global__ void flag_wait_kernel(const uint32_t* flag, uint32_t target) {
    if (threadIdx.x == 0) {
        const uint64_t t0 = global_ns();
        for (;;) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
            if (int32_t(v - target) >= 0) break;
            if (global_ns() - t0 > kWaitLimitNs) {
                record_flag_timeout(kStatusInHeadSplit, target, v);
                raise_status(kStatusTimeout | kStatusInHeadSplit);
                break;
            }
            __nanosleep(200);
        }
    }
    pdl_wait();
}

// Builds the decode and prefill work lists from the batch metadata (one CTA).
constexpr int kPlanThreads = 1024;

__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot, int& total) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < (kPlanThreads / 32) ? warp_tot[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        warp_tot[lane] = w;  // inclusive warp prefix
    }
    __syncthreads();
    const int before = (warp > 0 ? warp_tot[warp - 1] : 0) + x - v;
    total = warp_tot[kPlanThreads / 32 - 1];
    __syncthreads();
    return before;
}

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const AttnParams p) {
    __shared__ int warp_tot[32];
    pdl_release();
    pdl_wait();  // the metadata may come from the kernel before
    int run_d = 0, run_p = 0, run_s = 0;
    const int B = p.g.block_size;
    for (int base = 0; base < p.num_seqs; base += kPlanThreads) {
        const int s = base + threadIdx.x;
        int nd = 0, np = 0;
        if (s < p.num_seqs) {
            const int q0 = p.cu_seqlens_q[s];
            const int qlen = p.cu_seqlens_q[s + 1] - q0;
            const int ctx = p.context_lens[s];
            const bool ok = q0 >= 0 && qlen >= 0 && qlen <= ctx && qlen <= p.max_query_len &&
                            ctx <= p.max_context_len &&
                            int64_t(ctx) <= int64_t(p.max_blocks) * B;
            if (!ok) {
                raise_status(kStatusMetadata);
            } else if (qlen == 1) {
                nd = (ctx + p.split_tokens - 1) / p.split_tokens;
            } else if (qlen > 1) {
                np = (qlen + p.prefill_tile - 1) / p.prefill_tile;
            }
        }
        run_s += __syncthreads_count(nd > 0);
        int tot_d = 0, tot_p = 0;
        const int off_d = block_exclusive_scan(nd, warp_tot, tot_d);
        const int off_p = block_exclusive_scan(np, warp_tot, tot_p);
        for (int j = 0; j < nd; ++j) p.decode_items[run_d + off_d + j] = WorkItem{s, j};
        // Prefill tiles of a sequence go out last-tile first (they see the most keys).
        for (int j = 0; j < np; ++j) p.prefill_items[run_p + off_p + j] = WorkItem{s, np - 1 - j};
        run_d += tot_d;
        run_p += tot_p;
    }
    if (threadIdx.x == 0) {
        p.counters->decode_next = 0;
        p.counters->decode_items = run_d;
        p.counters->prefill_next = 0;
        p.counters->prefill_items = run_p;
        p.counters->decode_seqs = run_s;
        p.counters->rows_done = 0;
        if (p.num_outs > 0 && run_s == 0) {
            // no row will reach the merge kernel: signal the ranks from here
            __threadfence_system();
            for (int r = 0; r < p.num_outs; ++r) atomicAdd_system(p.flags[r], 1u);
        }
    }
}

template <int HD, int NW, int NS, bool kB16>
cudaError_t launch_decode_t(const AttnParams& p, cudaStream_t stream, bool overlap_previous) {
    constexpr size_t smem = decode_smem_bytes<HD, NW, NS>();
    static int grid_per_device[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (grid_per_device[dev] == 0) {
        e = cudaFuncSetAttribute(decode_kernel<HD, NW, NS, kB16>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return e;
        int sms = 0, per_sm = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel<HD, NW, NS, kB16>,
                                                          NW * 32, smem);
        if (e != cudaSuccess) return e;
        grid_per_device[dev] = sms * (per_sm > 0 ? per_sm : 1);
    }
    // Equal rounds: at most U = sequences x heads x splits units, which the
    // full grid's W warps would take in k = ceil(U / W) rounds, some warps one
    // round short; ceil(U / k) warps take the same k rounds with every warp
    // busy in each (a batch with few (sequence, head) pairs otherwise leaves
    // most warps idle during its last round).
    int grid = grid_per_device[dev];
    {
        const int64_t units = int64_t(p.num_seqs) * p.g.num_heads *
                              ((int64_t(p.max_context_len) + p.split_tokens - 1) / p.split_tokens);
        const int64_t full = int64_t(grid) * NW;
        const int64_t rounds = std::max<int64_t>(1, (units + full - 1) / full);
        const int64_t warps = (units + rounds - 1) / rounds;
        grid = int(std::clamp<int64_t>((warps + NW - 1) / NW, 1, grid));
    }
    AttnParams q = p;
    q.beside_prefill = overlap_previous ? 1 : 0;
    e = launch_programmatic(decode_kernel<HD, NW, NS, kB16>, dim3(unsigned(grid)), dim3(NW * 32),
                            smem, stream, q);
    if (e != cudaSuccess) return e;
    const int rows = p.num_seqs * p.g.num_heads;
    const int wpr = merge_warps_per_row(p.max_splits);
    const int rows_per_cta = 8 / wpr;
    return launch_programmatic(merge_kernel<HD>, dim3(unsigned((rows + rows_per_cta - 1) / rows_per_cta)),
                               dim3(256), 0, stream, q, wpr);
}

}  // namespace

int32_t decode_split_tokens(int32_t head_dim) {
    // 16 chunks of 2048/hd positions: 256 KiB of K+V per item at any head_dim.
    // (Finer items for batches with few (sequence, head) pairs measured no
    // faster: the longer plan and merge ate what the better balance gained.)
    return 16 * (2048 / head_dim);
}

cudaError_t launch_signal(uint32_t* const* flags, int n, cudaStream_t stream) {
    AttnParams p{};
    p.num_outs = n;
    for (int r = 0; r < n && r < kMaxRanks; ++r) p.flags[r] = flags[r];
    signal_kernel<<<1, 32, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_flag_wait(const uint32_t* flag, uint32_t target, cudaStream_t stream) {
    return launch_programmatic(flag_wait_kernel, dim3(1), dim3(32), 0, stream, flag, target);
}

cudaError_t launch_plan(const AttnParams& p, cudaStream_t stream) {
    return launch_programmatic(plan_kernel, dim3(1), dim3(kPlanThreads), 0, stream, p);
}

// Warps per CTA and stages per warp of the decode kernel (build-time tunables).
#ifndef NVLLM_DECODE_NW
#define NVLLM_DECODE_NW 6
#endif
#ifndef NVLLM_DECODE_NS
#define NVLLM_DECODE_NS 2
#endif

cudaError_t launch_decode(const AttnParams& p, cudaStream_t stream, bool overlap_previous) {
    constexpr int NW = NVLLM_DECODE_NW;
    constexpr int NS = NVLLM_DECODE_NS;
    const bool o = overlap_previous;
    switch (p.g.head_dim) {
        case 32: return launch_decode_t<32, NW, NS, false>(p, stream, o);
        case 64: return launch_decode_t<64, NW, NS, false>(p, stream, o);
        case 128:
            return p.g.block_size == 16 ? launch_decode_t<128, NW, NS, true>(p, stream, o)
                                        : launch_decode_t<128, NW, NS, false>(p, stream, o);
        case 256: return launch_decode_t<256, NW, NS, false>(p, stream, o);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace nvllm
