// K3 (strict fp32): causal paged prefill attention for sequences with more
// than one query row.
//
// Same mathematics as src/model.cpp:204-260 (each query row at position p sees
// positions 0..p through the block table, online softmax, out /= sum), computed
// flash-attention style over tiles: a CTA owns QT query rows of one
// (sequence, head) and walks key tiles of KT positions up to the tile's last
// query position. K and V tiles are gathered from the paged arena by bulk
// asynchronous copies (one arena row per copy) into a double-buffered
// shared-memory ring completing on mbarriers; QK^T and PV run on the FP32
// pipes (FFMA) so results stay within fp32 rounding of the reference.
//
// Persistent grid: CTAs pull (item, head) pairs from the plan kernel's
// prefill list (tiles with the most keys first within a sequence).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace nvllm {

namespace {

constexpr int kPrefillThreads = 256;  // 16 x 16 thread grid
constexpr int QT = 64;                // query rows per tile

template <int HD>
struct PrefillShape {
    static constexpr int KT = HD >= 256 ? 32 : 64;  // keys per tile
    static constexpr int ROW = HD + 4;               // padded Q/K/V row (floats)
    static constexpr int PROW = KT + 16;             // padded P row
    static constexpr int RPT = QT / 16;              // rows per thread
    static constexpr int KPT = KT / 16;              // keys per thread
    static constexpr int VW = HD >= 64 ? 4 : 2;      // output vector width
    static constexpr int NC = HD / (16 * VW);        // output vectors per row per thread
    static constexpr int COPY_FLOATS = HD < 128 ? HD : 128;
    static constexpr int CPR = HD / COPY_FLOATS;
    static constexpr int Q_FLOATS = QT * ROW;
    static constexpr int KV_FLOATS = KT * ROW;
    static constexpr int P_FLOATS = QT * PROW;
    static constexpr size_t SMEM = 128 + sizeof(float) * (Q_FLOATS + 4 * KV_FLOATS + P_FLOATS);
};

template <int HD>
__global__ void __launch_bounds__(kPrefillThreads, 1) prefill_fp32_kernel(const AttnParams p) {
    using S = PrefillShape<HD>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // a decode kernel launched as this kernel's programmatic dependent may start
    // on the SMs this grid leaves free (it reads nothing this kernel writes)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);  // 2 stages
    __shared__ int s_item;
    float* sQ = reinterpret_cast<float*>(smem_raw + 128);
    float* sKV = sQ + S::Q_FLOATS;  // [stage][K|V][KT][ROW]
    float* sP = sKV + 4 * S::KV_FLOATS;

    const int tid = threadIdx.x;
    const int tx = tid & 15;
    const int ty = tid >> 4;
    const int warp = tid >> 5;
    const int lane = tid & 31;

    for (int i = tid * 4; i < 4 * S::KV_FLOATS; i += kPrefillThreads * 4) {
        *reinterpret_cast<float4*>(sKV + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
    }
    fence_barrier_init();
    __syncthreads();

    const uint64_t pol = l2_evict_first();
    const ArenaGeom& g = p.g;
    const int H = g.num_heads;
    const int total = p.counters->prefill_items * H;
    uint32_t tile_seq = 0;  // K/V tiles consumed by this CTA (ring position)

    for (;;) {
        if (tid == 0) s_item = atomicAdd(&p.counters->prefill_next, 1);
        __syncthreads();
        const int it = s_item;
        __syncthreads();
        if (it >= total) break;
        const WorkItem wi = p.prefill_items[it / H];
        const int h = it % H;
        const int s = wi.seq;
        const int q0 = p.cu_seqlens_q[s];
        const int qlen = p.cu_seqlens_q[s + 1] - q0;
        const int ctx = p.context_lens[s];
        const int first_pos = ctx - qlen;
        const int r0 = wi.part * QT;
        const int nrows = min(QT, qlen - r0);
        const int nk = first_pos + r0 + nrows;  // keys 0..nk-1 are visible to this tile
        const int ntiles = (nk + S::KT - 1) / S::KT;
        const int32_t* table = p.block_tables + int64_t(s) * p.max_blocks;
        const int64_t head_off = int64_t(p.layer) * g.layer_stride + int64_t(h) * HD;

        // Q tile -> smem (rows past nrows zero)
        for (int i = tid; i < QT * (HD / 4); i += kPrefillThreads) {
            const int r = i / (HD / 4);
            const int c4 = i % (HD / 4);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < nrows) {
                v = __ldg(reinterpret_cast<const float4*>(p.q + int64_t(q0 + r0 + r) * g.row +
                                                          int64_t(h) * HD) + c4);
            }
            *reinterpret_cast<float4*>(sQ + r * S::ROW + c4 * 4) = v;
        }

        // Warp 0 gathers key tile t into ring stage (tile_seq + t) % 2.
        auto issue = [&](int t) {
            const uint32_t n = tile_seq + t;
            const int stage = int(n & 1u);
            float* sK = sKV + stage * 2 * S::KV_FLOATS;
            float* sV = sK + S::KV_FLOATS;
            const int kbase = t * S::KT;
            const int nvalid = min(S::KT, nk - kbase);
            constexpr int NCOP = 2 * S::KT * S::CPR;
            uint32_t bytes = 0;
            for (int ci = lane; ci < NCOP; ci += 32) {
                const int row = (ci % (S::KT * S::CPR)) / S::CPR;
                if (row < nvalid) {
                    const int64_t blk = table[(kbase + row) / g.block_size];
                    if (blk >= 0 && blk < g.num_blocks) bytes += S::COPY_FLOATS * 4;
                }
            }
            bytes = __reduce_add_sync(0xffffffffu, bytes);
            if (lane == 0) mbar_arrive_expect_tx(&bars[stage], bytes);
            __syncwarp();
            for (int ci = lane; ci < NCOP; ci += 32) {
                const int tensor = ci / (S::KT * S::CPR);
                const int rem = ci % (S::KT * S::CPR);
                const int row = rem / S::CPR;
                const int piece = rem % S::CPR;
                if (row >= nvalid) continue;
                const int pos = kbase + row;
                const int64_t blk = table[pos / g.block_size];
                if (blk < 0 || blk >= g.num_blocks) {
                    raise_status(kStatusBounds);
                    continue;
                }
                const int64_t off = blk * g.block_stride + head_off +
                                    int64_t(pos % g.block_size) * g.row + piece * S::COPY_FLOATS;
                bulk_copy_g2s((tensor ? sV : sK) + row * S::ROW + piece * S::COPY_FLOATS,
                              (tensor ? p.v_arena : p.k_arena) + off, S::COPY_FLOATS * 4,
                              &bars[stage], pol);
            }
        };
        if (warp == 0) issue(0);

        float o[S::RPT][S::NC][S::VW];
        float m_run[S::RPT], l_run[S::RPT];
#pragma unroll
        for (int i = 0; i < S::RPT; ++i) {
            m_run[i] = -INFINITY;
            l_run[i] = 0.f;
#pragma unroll
            for (int c = 0; c < S::NC; ++c)
#pragma unroll
                for (int v = 0; v < S::VW; ++v) o[i][c][v] = 0.f;
        }
        __syncthreads();  // sQ ready

        bool timed_out = false;
        int t = 0;
        for (; t < ntiles; ++t) {
            if (warp == 0 && t + 1 < ntiles) issue(t + 1);
            const uint32_t n = tile_seq + t;
            const int stage = int(n & 1u);
            if (!mbar_wait(&bars[stage], (n >> 1) & 1u, kStatusInPrefill)) timed_out = true;
            if (__syncthreads_or(timed_out)) {
                timed_out = true;
                break;
            }
            const float* sK = sKV + stage * 2 * S::KV_FLOATS;
            const float* sV = sK + S::KV_FLOATS;
            const int kbase = t * S::KT;

            // S = Q K^T for rows ty + 16 i, keys tx + 16 j
            float sc[S::RPT][S::KPT];
#pragma unroll
            for (int i = 0; i < S::RPT; ++i)
#pragma unroll
                for (int j = 0; j < S::KPT; ++j) sc[i][j] = 0.f;
#pragma unroll 4
            for (int d = 0; d < HD; d += 4) {
                float4 qf[S::RPT], kf[S::KPT];
#pragma unroll
                for (int i = 0; i < S::RPT; ++i) qf[i] = ld_shared4(sQ + (ty + 16 * i) * S::ROW + d);
#pragma unroll
                for (int j = 0; j < S::KPT; ++j) kf[j] = ld_shared4(sK + (tx + 16 * j) * S::ROW + d);
#pragma unroll
                for (int i = 0; i < S::RPT; ++i)
#pragma unroll
                    for (int j = 0; j < S::KPT; ++j) {
                        sc[i][j] = fmaf(qf[i].x, kf[j].x, sc[i][j]);
                        sc[i][j] = fmaf(qf[i].y, kf[j].y, sc[i][j]);
                        sc[i][j] = fmaf(qf[i].z, kf[j].z, sc[i][j]);
                        sc[i][j] = fmaf(qf[i].w, kf[j].w, sc[i][j]);
                    }
            }
            // mask, online softmax per row, P -> smem
#pragma unroll
            for (int i = 0; i < S::RPT; ++i) {
                const int row = ty + 16 * i;
                const int qpos = first_pos + r0 + row;
                float cm = -INFINITY;
#pragma unroll
                for (int j = 0; j < S::KPT; ++j) {
                    const int kpos = kbase + tx + 16 * j;
                    sc[i][j] = (kpos <= qpos && kpos < nk) ? sc[i][j] * p.qk_scale_log2 : -INFINITY;
                    cm = fmaxf(cm, sc[i][j]);
                }
                cm = warp_max_xor(cm, 16);
                const float m_new = fmaxf(m_run[i], cm);
                const float alpha = exp2f(m_run[i] - m_new);
                float ps = 0.f;
#pragma unroll
                for (int j = 0; j < S::KPT; ++j) {
                    const float pj = exp2f(sc[i][j] - m_new);
                    ps += pj;
                    sP[row * S::PROW + tx + 16 * j] = pj;
                }
                l_run[i] = fmaf(l_run[i], alpha, ps);
                m_run[i] = m_new;
#pragma unroll
                for (int c = 0; c < S::NC; ++c)
#pragma unroll
                    for (int v = 0; v < S::VW; ++v) o[i][c][v] *= alpha;
            }
            __syncthreads();
            // O += P V
#pragma unroll 2
            for (int k = 0; k < S::KT; k += 4) {
                float4 pf[S::RPT];
#pragma unroll
                for (int i = 0; i < S::RPT; ++i) pf[i] = ld_shared4(sP + (ty + 16 * i) * S::PROW + k);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    float vf[S::NC][S::VW];
#pragma unroll
                    for (int c = 0; c < S::NC; ++c) {
                        const float* vp = sV + (k + kk) * S::ROW + S::VW * tx + 16 * S::VW * c;
                        if constexpr (S::VW == 4) {
                            const float4 t4 = ld_shared4(vp);
                            vf[c][0] = t4.x; vf[c][1] = t4.y; vf[c][2] = t4.z; vf[c][3] = t4.w;
                        } else {
                            const float2 t2 = *reinterpret_cast<const float2*>(vp);
                            vf[c][0] = t2.x; vf[c][1] = t2.y;
                        }
                    }
#pragma unroll
                    for (int i = 0; i < S::RPT; ++i) {
                        const float pv = kk == 0 ? pf[i].x : kk == 1 ? pf[i].y : kk == 2 ? pf[i].z : pf[i].w;
#pragma unroll
                        for (int c = 0; c < S::NC; ++c)
#pragma unroll
                            for (int v = 0; v < S::VW; ++v) o[i][c][v] = fmaf(pv, vf[c][v], o[i][c][v]);
                    }
                }
            }
            __syncthreads();  // stage and sP free for reuse
        }
        if (timed_out) {
            // Tile t never completed; let the copies of tile t + 1 (already
            // issued) land, bounded, before the CTA's shared memory is released.
            if (t + 1 < ntiles) {
                const uint32_t n = tile_seq + t + 1;
                mbar_wait(&bars[n & 1u], (n >> 1) & 1u, kStatusInPrefill);
            }
            return;
        }
        tile_seq += ntiles;

        // epilogue: normalise and store rows < nrows
#pragma unroll
        for (int i = 0; i < S::RPT; ++i) {
            const int row = ty + 16 * i;
            const float l = warp_sum_xor(l_run[i], 16);
            const float inv = 1.0f / fmaxf(l, 1e-12f);
            if (row < nrows) {
                float* op = p.out + int64_t(q0 + r0 + row) * g.row + int64_t(h) * HD;
#pragma unroll
                for (int c = 0; c < S::NC; ++c) {
                    float* dst = op + S::VW * tx + 16 * S::VW * c;
                    if constexpr (S::VW == 4) {
                        *reinterpret_cast<float4*>(dst) =
                            make_float4(o[i][c][0] * inv, o[i][c][1] * inv, o[i][c][2] * inv,
                                        o[i][c][3] * inv);
                    } else {
                        *reinterpret_cast<float2*>(dst) = make_float2(o[i][c][0] * inv, o[i][c][1] * inv);
                    }
                }
            }
        }
    }
}

template <int HD>
cudaError_t launch_prefill_t(const AttnParams& p, cudaStream_t stream, int max_sms) {
    constexpr size_t smem = PrefillShape<HD>::SMEM;
    static int grid_per_device[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (grid_per_device[dev] == 0) {
        e = cudaFuncSetAttribute(prefill_fp32_kernel<HD>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return e;
        int sms = 0, per_sm = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, prefill_fp32_kernel<HD>,
                                                          kPrefillThreads, smem);
        if (e != cudaSuccess) return e;
        grid_per_device[dev] = sms * (per_sm > 0 ? per_sm : 1);
    }
    int grid = grid_per_device[dev];
    if (max_sms > 0) {
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        if (max_sms < sms) grid = std::max(1, grid / sms * max_sms);
    }
    prefill_fp32_kernel<HD><<<grid, kPrefillThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

int32_t prefill_tile_rows(int32_t /*head_dim*/) { return QT; }

cudaError_t launch_prefill_fp32(const AttnParams& p, cudaStream_t stream, int max_sms) {
    switch (p.g.head_dim) {
        case 32: return launch_prefill_t<32>(p, stream, max_sms);
        case 64: return launch_prefill_t<64>(p, stream, max_sms);
        case 128: return launch_prefill_t<128>(p, stream, max_sms);
        case 256: return launch_prefill_t<256>(p, stream, max_sms);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace nvllm
