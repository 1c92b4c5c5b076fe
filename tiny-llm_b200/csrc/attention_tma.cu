// attention_tma.cu — split-K GQA decode attention with the KV chunk staged in
// shared memory by TMA bulk copies and the splits merged through distributed
// shared memory, sm_100a.
//
// Semantics: attention_decode_ref (kernels/attention/attention_decode_ref.cpp:53-143),
// fp16 KV as in the reference's KVCache (runtime/kv_cache.cpp:120-135).  In the
// engine ("fused") mode the kernel also performs the step's QK-norm, RoPE and KV
// append (runtime/qwen_forward_token.cpp:423-446), which removes one launch per
// layer and lets every cached row be fetched before the previous kernel finishes.
//
// Grid (n_kv_heads, ns) in clusters of (1, ns): the ns CTAs of a KV head form one
// thread-block cluster.  CTA rank s owns positions [s*chunk, s*chunk+n) of its KV
// head for the G query heads that share it.  The chunk streams through a ring of
// shared-memory tiles, a tile being the K and V rows of T positions (two
// cp.async.bulk copies, completion on the slot's mbarrier); the last warp done with
// a slot issues its next tile.  Flash-decoding inside the CTA: each warp takes its
// rows of every tile 32/G at a time, forms their G dot products per row with lanes
// over head dimensions and one warp reduce-scatter, and keeps an online softmax and
// o = sum p v per head.  The warps' (m, l, o) are combined in shared memory; each CTA
// then pushes its partial of output slice r, and its (m, l), into cluster rank r's
// shared memory (DSMEM stores), and after one cluster barrier every rank merges its
// own slice (weights exp(m_s - M) per split and head).  No global scratch, no atomics
// on data.
//
// Ordering (programmatic dependent launch): rows [0, seq-1) of the cache were
// written by earlier steps and *pos at the start of this step, both complete once
// the kernel runs (the kernel before it waited on its own predecessor before
// releasing this one), so in fused mode their copies, and those of the constant
// vectors (RoPE row, QK-norm weights), are issued before griddepcontrol.wait; the
// step's q/k/v come from the immediately preceding kernel and are copied after it.
// In plain mode the whole chunk may come from the previous kernel, so every copy is
// issued after the wait.
#include <float.h>

#include <algorithm>
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace tqb200 {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 8;         // max tiles in flight (all of a 4096-context chunk)
constexpr int kTileBytes = 16384;  // target bytes per staged tile
constexpr int kMaxSplit = 16;      // cluster size (non-portable above 8)

struct TmaAttnParams {
    const float *q;                 // [H*HD] (raw projection in fused mode)
    uint8_t *kc, *vc;               // caches [KVH][max_seq][HD] (KV elements)
    const float *k_new, *v_new;     // fused: this step's k, v [KVH*HD]; null = plain
    const float *q_norm, *k_norm;   // fused, optional [HD]
    float eps;
    const float *cos_tab, *sin_tab; // fused: [max_seq][HD/2]
    const int *pos;                 // seq = *pos + 1 (null -> seq_len)
    int seq_len, max_seq, chunk_max;
    float scale;
    int tile_rows, stages, stage_region;  // rows per tile; tiles in the ring; ring bytes
    int bulk_in;                    // q/k/v and constant vectors 16-byte aligned: bulk copies
    float *out;
    int *status;
    Stamp stamp;                    // in-graph timeline (off unless the engine records one)
    const XPut *put;                // tensor parallelism (device descriptor, XCHG instance
                                    // only): out rows also go to every peer
};

template <typename KV>
__device__ __forceinline__ KV to_kv(float v) {
    if constexpr (sizeof(KV) == 2) return f2h_ref(v);
    else return v;
}

// D consecutive KV elements from shared memory as floats (D = 1, 2, 4)
template <int D>
__device__ __forceinline__ void lds_kv(const float *p, float o[D]) {
    if constexpr (D == 4) {
        const float4 v = *reinterpret_cast<const float4 *>(p);
        o[0] = v.x, o[1] = v.y, o[2] = v.z, o[3] = v.w;
    } else if constexpr (D == 2) {
        const float2 v = *reinterpret_cast<const float2 *>(p);
        o[0] = v.x, o[1] = v.y;
    } else {
        o[0] = *p;
    }
}
template <int D>
__device__ __forceinline__ void lds_kv(const uint16_t *p, float o[D]) {
    if constexpr (D == 4) {
        const uint2 v = *reinterpret_cast<const uint2 *>(p);
        o[0] = h2f((uint16_t)(v.x & 0xFFFFu)), o[1] = h2f((uint16_t)(v.x >> 16));
        o[2] = h2f((uint16_t)(v.y & 0xFFFFu)), o[3] = h2f((uint16_t)(v.y >> 16));
    } else if constexpr (D == 2) {
        const uint32_t v = *reinterpret_cast<const uint32_t *>(p);
        o[0] = h2f((uint16_t)(v & 0xFFFFu)), o[1] = h2f((uint16_t)(v >> 16));
    } else {
        o[0] = h2f(*p);
    }
}

// D consecutive 16-bit cache elements as one register load (staged rows)
template <int D> struct Raw16 { using T = uint16_t; };
template <> struct Raw16<2> { using T = uint32_t; };
template <> struct Raw16<4> { using T = uint2; };
template <int D>
__device__ __forceinline__ typename Raw16<D>::T ld_raw16(const uint16_t *p) {
    return *reinterpret_cast<const typename Raw16<D>::T *>(p);
}
template <int D>
__device__ __forceinline__ void raw16_to_f(typename Raw16<D>::T v, float o[D]) {
    if constexpr (D == 4) {
        o[0] = h2f((uint16_t)(v.x & 0xFFFFu)), o[1] = h2f((uint16_t)(v.x >> 16));
        o[2] = h2f((uint16_t)(v.y & 0xFFFFu)), o[3] = h2f((uint16_t)(v.y >> 16));
    } else if constexpr (D == 2) {
        o[0] = h2f((uint16_t)(v & 0xFFFFu)), o[1] = h2f((uint16_t)(v >> 16));
    } else {
        o[0] = h2f(v);
    }
}

// Reduce-scatter of N per-lane values over the warp: after it, v[0] of lane l is
// the warp-wide sum of value (l >> (5 - log2 N)); N is a power of two <= 32.
template <int N, int OFF>
__device__ __forceinline__ void warp_reduce_scatter(float *v, int lane) {
    if constexpr (N > 1) {
        const bool up = (lane & OFF) != 0;
#pragma unroll
        for (int i = 0; i < N / 2; ++i) {
            const float send = up ? v[i] : v[i + N / 2];
            const float keep = up ? v[i + N / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
        }
        warp_reduce_scatter<N / 2, OFF / 2>(v, lane);
    } else {
#pragma unroll
        for (int o = OFF; o > 0; o >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
}

template <int G> struct Pow2 { static constexpr int v = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8; };
template <int N> struct Log2 { static constexpr int v = N <= 1 ? 0 : N <= 2 ? 1 : N <= 4 ? 2 : 3; };

// Scores of RW = 32/GP consecutive cached rows at once (warp-cooperative): every lane
// forms the partial dots of its HD/32 dimensions for all RW rows and G heads (32
// values), and one 5-level reduce-scatter leaves lane l with the full dot of row
// l / GP, head l % GP: 31 shuffles in 5 dependent steps for RW rows.  Each lane returns
// its value scaled, -inf for lanes past `rows` or G.
template <typename KV, int HD, int G>
__device__ __forceinline__ float score_lane(const KV *kr, int rows, const float (&qr)[G][HD / 32],
                                            int lane, float scale) {
    constexpr int D = HD / 32;
    constexpr int GP = Pow2<G>::v;
    constexpr int RW = 32 / GP;
    float acc[32];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        float k[D];
        if (r < rows) {
            lds_kv<D>(kr + (size_t)r * HD + lane * D, k);
        } else {
#pragma unroll
            for (int d = 0; d < D; ++d) k[d] = 0.0f;
        }
#pragma unroll
        for (int g = 0; g < GP; ++g) {
            float a = 0.0f;
            if (g < G) {
#pragma unroll
                for (int d = 0; d < D; ++d) a = fmaf(qr[g][d], k[d], a);
            }
            acc[r * GP + g] = a;
        }
    }
    warp_reduce_scatter<32, 16>(acc, lane);
    const int r = lane / GP, g = lane - r * GP;
    return (r < rows && g < G) ? acc[0] * scale : -INFINITY;
}

// Warp-level QK-norm (optional) + rotate-half RoPE of one head vector, in place in
// shared memory; the same float operations as the per-head engine kernel.
template <int HD>
__device__ __forceinline__ void norm_rope_warp(float *x, const float *nw, float eps,
                                               const float *cs, const float *sn, int lane) {
    if (nw) {
        double ss = 0.0;
        for (int i = lane; i < HD; i += 32) ss += (double)x[i] * (double)x[i];
        ss = warp_sum_d(ss);
        const float mean_sq = (float)(ss / HD);
        const float rs = 1.0f / sqrtf(__fadd_rn(mean_sq, eps));
        for (int i = lane; i < HD; i += 32) x[i] = __fmul_rn(__fmul_rn(x[i], rs), nw[i]);
        __syncwarp();
    }
    constexpr int half = HD / 2;
    constexpr int E = (half + 31) / 32;
    float r0[E], r1[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int i = lane + 32 * e;
        if (i < half) {
            const float x0 = x[i], x1 = x[i + half], c = cs[i], s = sn[i];
            r0[e] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
            r1[e] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
        }
    }
    __syncwarp();
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int i = lane + 32 * e;
        if (i < half) {
            x[i] = r0[e];
            x[i + half] = r1[e];
        }
    }
    __syncwarp();
}

// 16-bit caches: at most 128 registers, so two CTAs fit an SM with the staged rows; the
// fp32 instantiations keep the compiler's choice (all <= 127 but G=8 x HD 128 at 156,
// whose 4-KV-head grids run one CTA per SM anyway).
template <typename KV, int HD, int G, bool STAMP, bool XCHG>
__global__ void __launch_bounds__(kThreads, sizeof(KV) == 2 ? 2 : 1) attn_tma_kernel(const __grid_constant__ TmaAttnParams P) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int RB = HD * (int)sizeof(KV);  // bytes per cached row
    constexpr int D = HD / 32;                // dimensions per lane in the score phase
    constexpr int half = HD / 2;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);  // [stages] tiles
    uint64_t *bar_c = bars + kStages;                      // constant vectors
    uint8_t *ring = smem + 128;
    KV *lastk = reinterpret_cast<KV *>(ring + P.stage_region);  // [HD] new row (fused)
    KV *lastv = lastk + HD;
    float *krow = reinterpret_cast<float *>(
        ((uintptr_t)(lastv + HD) + 15) & ~(uintptr_t)15);       // [HD] new k (fp32)
    float *vrow = krow + HD;                                    // [HD] new v (fp32)
    float *qs = vrow + HD;                                      // [G][HD]
    float *cs = qs + G * HD;                                    // [HD/2] RoPE row
    float *sn = cs + half;                                      // [HD/2]
    float *qn = sn + half;                                      // [HD] QK-norm weights
    float *kn = qn + HD;                                        // [HD]
    float *rcv_o = kn + HD;                                     // [ns][per] pushed partial o
    float *rcv_m = rcv_o + G * HD + kMaxSplit;                  // [ns][G] pushed m
    float *rcv_l = rcv_m + kMaxSplit * G;                       // [ns][G] pushed l
    // after the last tile the ring holds the warps' partials and this CTA's partial
    float *wpo = reinterpret_cast<float *>(ring);               // [warps][G][HD]
    float *wpm = wpo + kWarps * G * HD;                         // [warps][G]
    float *wpl = wpm + kWarps * G;                              // [warps][G]
    float *po = wpl + kWarps * G;                               // [G][HD] partial o
    float *pm = po + G * HD;                                    // [G] partial m
    float *pl = pm + G;                                         // [G] partial l
    float *wgt = pl + G;                                        // [ns][G] merge weights (+ m, l copies)
    __shared__ float s_m[G], s_l[G];
    __shared__ float s_cw[kWarps * G];  // CTA merge weights
    __shared__ __align__(16) float s_p[kWarps][32];  // each warp's p values, read as broadcasts
    __shared__ int s_err, s_issued;
    __shared__ int s_done[kStages];  // warps finished with the slot's current tile

    StampRegs stamp_r;
    stamp_enter<STAMP>(P.stamp, stamp_r);
    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kh = blockIdx.x;
    const int ns = (int)cluster.num_blocks(), split = (int)cluster.block_rank();
    const bool fused = P.k_new != nullptr;
    const int seq = P.pos ? (*P.pos + 1) : P.seq_len;
    if (seq < 1 || seq > P.max_seq) {  // uniform over the grid: no CTA reaches a cluster barrier
        if (tid == 0 && kh == 0 && split == 0 && P.status) atomicExch(P.status, kDevBadPosition);
        return;
    }
    const int chunk = (seq + ns - 1) / ns;
    const int t0 = split * chunk;
    const int n = max(0, min(seq, t0 + chunk) - t0);
    const bool owner = fused && seq - 1 >= t0 && seq - 1 < t0 + n;  // holds the new row
    const int n_copy = owner ? n - 1 : n;
    const int T = P.tile_rows, NST = P.stages;
    const int total = (n_copy + T - 1) / T;  // tiles: K and V of T rows in one slot
    const size_t row0 = (size_t)kh * P.max_seq + t0;
    const bool has_norm = P.q_norm != nullptr;
    auto issue = [&](int i) {
        const int r0 = i * T, rows = min(T, n_copy - r0);
        uint64_t *bar = &bars[i % NST];
        uint8_t *slot = ring + (size_t)(i % NST) * 2 * T * RB;
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(bar, (uint32_t)(2 * rows * RB));
        bulk_g2s(slot, P.kc + (row0 + r0) * RB, (uint32_t)(rows * RB), bar);
        bulk_g2s(slot + (size_t)T * RB, P.vc + (row0 + r0) * RB, (uint32_t)(rows * RB), bar);
        atomicMax(&s_issued, i + 1);
    };
    if (tid == 0) {
        for (int s = 0; s < kStages + 2; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        s_err = 0;
        s_issued = 0;
        for (int s = 0; s < kStages; ++s) s_done[s] = 0;
        if (fused) {
            for (int i = 0; i < min(total, NST); ++i) issue(i);
            if (P.bulk_in) {
                const uint32_t hb = (uint32_t)half * 4u;
                mbar_arrive_expect_tx(bar_c, 2 * hb + (has_norm ? 2u * HD * 4u : 0u));
                bulk_g2s(cs, P.cos_tab + (size_t)(seq - 1) * half, hb, bar_c);
                bulk_g2s(sn, P.sin_tab + (size_t)(seq - 1) * half, hb, bar_c);
                if (has_norm) {
                    bulk_g2s(qn, P.q_norm, HD * 4u, bar_c);
                    bulk_g2s(kn, P.k_norm, HD * 4u, bar_c);
                }
            }
        }
    }
    stamp_step<STAMP>(P.stamp, stamp_r);
    griddep_wait();
    stamp_waited<STAMP>(P.stamp, stamp_r);
    if (tid == 0 && !fused)
        for (int i = 0; i < min(total, NST); ++i) issue(i);
    // q (and the owner's new k, v) were just written by the projection kernel: plain
    // loads by every thread reach them sooner than a bulk copy and its barrier
    for (int i = tid; i < G * HD; i += kThreads) qs[i] = P.q[(size_t)kh * G * HD + i];
    if (owner)
        for (int i = tid; i < HD; i += kThreads)
            krow[i] = P.k_new[(size_t)kh * HD + i], vrow[i] = P.v_new[(size_t)kh * HD + i];
    if (P.bulk_in) {
        if (tid == 0 && fused && !mbar_wait(bar_c, 0, kWaitCycles)) s_err = 1;
    } else {  // unaligned constant vectors: plain loads
        if (fused) {
            for (int i = tid; i < half; i += kThreads) {
                cs[i] = P.cos_tab[(size_t)(seq - 1) * half + i];
                sn[i] = P.sin_tab[(size_t)(seq - 1) * half + i];
            }
            if (has_norm)
                for (int i = tid; i < HD; i += kThreads) qn[i] = P.q_norm[i], kn[i] = P.k_norm[i];
        }
    }
    __syncthreads();

    // ---- fused mode: QK-norm + RoPE of the G query heads and, for the owner, of the
    // new k row; the new k/v rounded to the cache type, kept in shared memory for this
    // step and appended to the cache for the next ones
    if (fused && !s_err) {
        const int jobs = G + (owner ? 2 : 0);
        for (int h = warp; h < jobs; h += kWarps) {
            if (h < G) {
                norm_rope_warp<HD>(qs + h * HD, has_norm ? qn : nullptr, P.eps, cs, sn, lane);
            } else if (h == G) {
                norm_rope_warp<HD>(krow, has_norm ? kn : nullptr, P.eps, cs, sn, lane);
                KV *dst = reinterpret_cast<KV *>(P.kc) + ((size_t)kh * P.max_seq + seq - 1) * HD;
                for (int i = lane; i < HD; i += 32) {
                    const KV v = to_kv<KV>(krow[i]);
                    lastk[i] = v;
                    dst[i] = v;
                }
            } else {
                KV *dst = reinterpret_cast<KV *>(P.vc) + ((size_t)kh * P.max_seq + seq - 1) * HD;
                for (int i = lane; i < HD; i += 32) {
                    const KV v = to_kv<KV>(vrow[i]);
                    lastv[i] = v;
                    dst[i] = v;
                }
            }
        }
        __syncthreads();
    }
    float qr[G][D];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int d = 0; d < D; ++d) qr[g][d] = qs[g * HD + lane * D + d];

    // ---- rows -> (m, l, o) per warp, flash-decoding style: warp w takes rows
    // [w*RPW, (w+1)*RPW) of every tile, RW at a time (one reduce-scatter for their
    // scores), and keeps an online softmax per head.  Lane l serves head l % GP: it holds
    // the head's running max m (the same in all of the head's lanes) and its own share of
    // the head's sum l (the shares are added once, after the last tile); o = sum p v has
    // lanes over head dimensions.  No block barrier per tile: each warp waits for the tile
    // itself and the last warp done with a slot refills it.  With a 16-bit cache (and a
    // group that fits 32 registers) a warp first copies its rows to registers and gives
    // the slot back, so the refill's latency overlaps the arithmetic.
    constexpr int GP = Pow2<G>::v;
    constexpr int RW = 32 / GP;
    constexpr bool kStage = sizeof(KV) == 2 && 2 * RW * ((D + 1) / 2) <= 32;  // <= 32 registers
    const int RPW = T / kWarps;
    const int gl = lane & (GP - 1);
    float m_lane = -INFINITY, l_lane = 0.0f, acc[G][D];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int d = 0; d < D; ++d) acc[g][d] = 0.0f;
    float *pbuf = s_p[warp];
    // the last warp done with slot sl refills it with tile it + NST
    auto release = [&](int sl, int it) {
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            if (atomicAdd(&s_done[sl], 1) == kWarps - 1) {
                s_done[sl] = 0;
                if (it + NST < total) issue(it + NST);
            }
        }
    };
    // online update with this lane's score s (row lane / GP, head gl; -inf: no row):
    // returns p = exp(s - m) and rescales o.  Fast exponentials (ex2.approx, ~2^-21
    // relative): the online softmax's terms only need fp32-level accuracy.
    auto online = [&](float s) -> float {
        float mx = s;
#pragma unroll
        for (int o = GP; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float mn = fmaxf(m_lane, mx);
        const float alpha = m_lane == -INFINITY ? 0.0f : __expf(m_lane - mn);
        const float p = s == -INFINITY ? 0.0f : __expf(s - mn);
        l_lane = fmaf(l_lane, alpha, p);
        m_lane = mn;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float ag = __shfl_sync(0xffffffffu, alpha, g);
#pragma unroll
            for (int d = 0; d < D; ++d) acc[g][d] *= ag;
        }
        __syncwarp();  // the previous group's reads of pbuf are done
        pbuf[lane] = p;
        __syncwarp();
        return p;
    };
    // o += p(row r, g) * v for every head g; p read back from pbuf as broadcasts
    auto pv_row = [&](int r, const float (&v)[D]) {
        float pr[GP];
        if constexpr (GP >= 4) {
#pragma unroll
            for (int j = 0; j < GP; j += 4) {
                const float4 t = *reinterpret_cast<const float4 *>(pbuf + r * GP + j);
                pr[j] = t.x, pr[j + 1] = t.y, pr[j + 2] = t.z, pr[j + 3] = t.w;
            }
        } else if constexpr (GP == 2) {
            const float2 t = *reinterpret_cast<const float2 *>(pbuf + r * 2);
            pr[0] = t.x, pr[1] = t.y;
        } else {
            pr[0] = pbuf[r];
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int d = 0; d < D; ++d) acc[g][d] = fmaf(pr[g], v[d], acc[g][d]);
    };
    // one group of nrows <= RW rows (K rows kr, V rows vr): scores, online update, P.V;
    // rel_sl >= 0: give ring slot rel_sl back (tile rel_it) once the rows are read
    auto group = [&](const KV *kr, const KV *vr, int nrows, int rel_sl, int rel_it) {
        if constexpr (kStage) {
            using R = typename Raw16<D>::T;
            R kw[RW], vw[RW];
#pragma unroll
            for (int r = 0; r < RW; ++r) {
                if (r < nrows) {
                    kw[r] = ld_raw16<D>(reinterpret_cast<const uint16_t *>(kr) + (size_t)r * HD + lane * D);
                    vw[r] = ld_raw16<D>(reinterpret_cast<const uint16_t *>(vr) + (size_t)r * HD + lane * D);
                } else {
                    kw[r] = R{};
                    vw[r] = R{};
                }
            }
            if (rel_sl >= 0) release(rel_sl, rel_it);
            float a32[32];
#pragma unroll
            for (int r = 0; r < RW; ++r) {
                float k[D];
                raw16_to_f<D>(kw[r], k);
#pragma unroll
                for (int g = 0; g < GP; ++g) {
                    float a = 0.0f;
                    if (g < G) {
#pragma unroll
                        for (int d = 0; d < D; ++d) a = fmaf(qr[g][d], k[d], a);
                    }
                    a32[r * GP + g] = a;
                }
            }
            warp_reduce_scatter<32, 16>(a32, lane);
            const float s = (lane / GP < nrows && gl < G) ? a32[0] * P.scale : -INFINITY;
            online(s);
#pragma unroll
            for (int r = 0; r < RW; ++r) {
                if (r < nrows) {
                    float v[D];
                    raw16_to_f<D>(vw[r], v);
                    pv_row(r, v);
                }
            }
        } else {
            const float s = score_lane<KV, HD, G>(kr, nrows, qr, lane, P.scale);  // -inf: no row
            online(s);
            for (int r = 0; r < nrows; ++r) {
                float v[D];
                lds_kv<D>(vr + (size_t)r * HD + lane * D, v);
                pv_row(r, v);
            }
            if (rel_sl >= 0) release(rel_sl, rel_it);
        }
    };
    if (!s_err) {
        for (int it = 0; it < total; ++it) {
            const int sl = it % NST;
            if (!__all_sync(0xffffffffu, mbar_wait(&bars[sl], (uint32_t)(it / NST) & 1u, kWaitCycles))) {
                if (lane == 0) s_err = 1;
                break;
            }
            const KV *kt = reinterpret_cast<const KV *>(ring + (size_t)sl * 2 * T * RB);
            const KV *vt = kt + (size_t)T * HD;
            const int rows = min(T, n_copy - it * T);
            const int r_beg = warp * RPW, r_end = min(rows, (warp + 1) * RPW);
            for (int rb = r_beg; rb < r_end; rb += RW)
                group(kt + (size_t)rb * HD, vt + (size_t)rb * HD, min(RW, r_end - rb),
                      rb + RW >= r_end ? sl : -1, it);
            if (r_beg >= r_end) release(sl, it);  // no rows of this tile for this warp
        }
        if (owner && warp == kWarps - 1 && !s_err) group(lastk, lastv, 1, -1, 0);  // the new row
    }
    // the head's lanes' shares of l; lanes g < G then hold head g's (m, l)
    float l_head = l_lane;
#pragma unroll
    for (int o = GP; o < 32; o <<= 1) l_head += __shfl_xor_sync(0xffffffffu, l_head, o);
    __syncthreads();  // every warp is past the ring: it now holds the partials
    // dependents (the next projection) start their weight prefetch now, not earlier:
    // their copies would compete with this kernel's cache reads
    griddep_launch();
    const bool err = s_err != 0;
    if (err) {
        // drain the copies still in flight and report; this CTA's partial is an empty
        // split's (the merge gives it weight 0), so the cluster stays in step
        if (tid == 0) {
            const int issued = s_issued;
            for (int i = max(0, issued - NST); i < issued; ++i)
                mbar_wait(&bars[i % NST], (uint32_t)(i / NST) & 1u, kWaitCycles);
            if (P.bulk_in && fused) mbar_wait(bar_c, 0, kWaitCycles);
            if (P.status) atomicExch(P.status, kDevTimeoutTma);
        }
        __syncthreads();
    }
    // ---- warps' partials -> this CTA's partial (m, l, o) in its own shared memory
    if (lane < G) {
        wpm[warp * G + lane] = err ? -INFINITY : m_lane;
        wpl[warp * G + lane] = err ? 0.0f : l_head;
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int d = 0; d < D; ++d) wpo[(warp * G + g) * HD + lane * D + d] = err ? 0.0f : acc[g][d];
    __syncthreads();
    if (tid < G) {  // the warps' weights exp(m_w - M) of head g, once
        const int g = tid;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wpm[w * G + g]);
        float Lsum = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float mw = wpm[w * G + g];
            const float e = mw == -INFINITY ? 0.0f : expf(mw - M);
            s_cw[w * G + g] = e;
            Lsum = fmaf(e, wpl[w * G + g], Lsum);
        }
        pm[g] = M;
        pl[g] = Lsum;
    }
    __syncthreads();
    for (int i = tid; i < G * HD; i += kThreads) {
        const int g = i / HD;
        float O = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) O = fmaf(s_cw[w * G + g], wpo[(w * G + g) * HD + (i - g * HD)], O);
        po[i] = O;
    }
    // ---- merge over DSMEM, pushed: output slice r (per values) belongs to rank r; every
    // rank stores its partial of slice r, and its (m, l), into rank r's receive area
    // (remote stores, no round trip), then one cluster barrier (release / acquire) makes
    // them visible and each rank merges its own slice from local shared memory.  Empty
    // splits (m = -inf, o = 0) weigh 0.
    const int per = (G * HD + ns - 1) / ns;
    __syncthreads();  // po, pm, pl complete
    for (int i = tid; i < G * HD; i += kThreads) {
        const int r = i / per;
        *cluster.map_shared_rank(rcv_o + split * per + (i - r * per), r) = po[i];
    }
    for (int i = tid; i < G * ns; i += kThreads) {
        const int r = i / G, g = i - r * G;
        *cluster.map_shared_rank(rcv_m + split * G + g, r) = pm[g];
        *cluster.map_shared_rank(rcv_l + split * G + g, r) = pl[g];
    }
    cluster.sync();  // every push has landed
    // the splits' weights exp(m_s - M) per head: 16 lanes per head (lane s2 = split s2),
    // the max and the weighted sum of l as shuffle trees
    static_assert(kMaxSplit == 16 && G * 16 <= kThreads, "one 16-lane group per head");
    if (tid < ((G * 16 + 31) & ~31)) {  // whole warps: every lane takes the shuffles
        const int g = tid >> 4, s2 = tid & 15;
        const bool ok = g < G && s2 < ns;
        const float m = ok ? rcv_m[s2 * G + g] : -INFINITY;
        float M = m;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float w = m == -INFINITY ? 0.0f : expf(m - M);
        float L = ok ? rcv_l[s2 * G + g] * w : 0.0f;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        if (ok) wgt[s2 * G + g] = w;
        if (g < G && s2 == 0) s_l[g] = L;
    }
    __syncthreads();
    // this rank's slice of the output: 8 lanes per value, each over every 8th split,
    // then a 3-level shuffle sum
    const int cnt = max(0, min(G * HD, (split + 1) * per) - split * per);
    for (int base = 0; base < cnt; base += kThreads / 8) {  // uniform over the CTA
        const int j = base + (tid >> 3), sub = tid & 7;
        const int i = split * per + j;
        const int g = i / HD;
        float O = 0.0f;
        if (j < cnt)
            for (int s2 = sub; s2 < ns; s2 += 8) O = fmaf(rcv_o[s2 * per + j], wgt[s2 * G + g], O);
        O += __shfl_xor_sync(0xffffffffu, O, 4);
        O += __shfl_xor_sync(0xffffffffu, O, 2);
        O += __shfl_xor_sync(0xffffffffu, O, 1);
        if (j < cnt && sub == 0) {
            if constexpr (XCHG) {
                if (P.put) xput_val(*P.put, P.out + (size_t)kh * G * HD + i, O / s_l[g]);
                else P.out[(size_t)kh * G * HD + i] = O / s_l[g];
            } else {
                P.out[(size_t)kh * G * HD + i] = O / s_l[g];
            }
        }
    }
    if constexpr (XCHG)
        if (P.put) xput_arrive(*P.put);
    stamp_exit<STAMP>(P.stamp, stamp_r);
}

template <typename KV, int HD, int G, bool STAMP, bool XCHG>
int launch_t(const AttnArgs &a, cudaStream_t st) {
    constexpr int RB = HD * (int)sizeof(KV);
    auto k = attn_tma_kernel<KV, HD, G, STAMP, XCHG>;
    static KernelSmem attr;
    static std::atomic<unsigned long long> cluster_attr{0};
    int smem_max = 0;
    TQ_CUDA_TRY(smem_limit_once(k, attr, &smem_max));
    {
        int dev = 0;
        TQ_CUDA_TRY(cudaGetDevice(&dev));
        const unsigned long long bit = 1ull << (dev & 63);
        if (!(cluster_attr.load() & bit)) {
            TQ_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
            cluster_attr.fetch_or(bit);
        }
    }
    auto a16 = [](const void *p) { return ((uintptr_t)p & 15u) == 0; };
    // splits = cluster size: about one CTA per SM over all KV heads, at most 16, at
    // least 32 positions per split; halved while a cluster of that size cannot be
    // scheduled (a cluster must fit in one GPC)
    int ns = std::max(1, std::min(kMaxSplit, (num_sms() + a.n_kv_heads - 1) / a.n_kv_heads));
    ns = std::min(ns, std::max(1, (a.max_seq + 31) / 32));
    for (; ns >= 1; ns /= 2) {
        TmaAttnParams P{};
        P.q = a.q;
        P.kc = (uint8_t *)a.k;
        P.vc = (uint8_t *)a.v;
        P.k_new = a.k_new;
        P.v_new = a.v_new;
        P.q_norm = a.q_norm;
        P.k_norm = a.k_norm;
        P.eps = a.eps;
        P.cos_tab = a.cos_tab;
        P.sin_tab = a.sin_tab;
        P.pos = a.pos;
        P.seq_len = a.seq_len;
        P.max_seq = a.max_seq;
        P.chunk_max = (a.max_seq + ns - 1) / ns;
        P.scale = a.scale;
        // a tile is the K and V rows of tile_rows positions (<= 32 KB, a multiple of the
        // warp count: every warp takes the same share of it)
        int T = std::max(kWarps, 2 * kTileBytes / (2 * RB) / kWarps * kWarps);
        T = std::min(T, (P.chunk_max + kWarps - 1) / kWarps * kWarps);
        P.tile_rows = T;
        // at most 64 KB of tiles in flight: two CTAs fit an SM, so the clusters of all
        // KV heads are resident at once
        P.stages = std::max(1, std::min({kStages, 65536 / (2 * T * RB),
                                         (P.chunk_max + T - 1) / T}));
        const size_t ring = (size_t)P.stages * 2 * T * RB;
        const size_t part = ((size_t)kWarps * G * HD + 2 * (size_t)kWarps * G + (size_t)G * HD +
                             2 * G + 3 * (size_t)kMaxSplit * G) * 4;
        P.stage_region = (int)((std::max(ring, part) + 15) & ~(size_t)15);
        P.bulk_in = a16(a.q) && (!a.k_new || (a16(a.k_new) && a16(a.v_new) && a16(a.cos_tab) &&
                                              a16(a.sin_tab) &&
                                              (!a.q_norm || (a16(a.q_norm) && a16(a.k_norm)))));
        P.out = a.out;
        P.status = a.status;
        P.stamp = a.stamp;
        P.put = a.put;
        // barriers | ring | new k, v rows (cache type) | krow, vrow, qs, cs+sn, qn, kn
        const size_t smem = 128 + (size_t)P.stage_region + ((2 * (size_t)RB + 15) & ~(size_t)15) +
                            ((size_t)5 * HD + (size_t)G * HD) * 4 +
                            ((size_t)G * HD + kMaxSplit + 2 * (size_t)kMaxSplit * G) * 4;
        if (smem > (size_t)smem_max) continue;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(a.n_kv_heads, ns);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr_l[2];
        attr_l[0].id = cudaLaunchAttributeClusterDimension;
        attr_l[0].val.clusterDim.x = 1;
        attr_l[0].val.clusterDim.y = ns;
        attr_l[0].val.clusterDim.z = 1;
        attr_l[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr_l[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr_l;
        cfg.numAttrs = 1;
        // prefer a split count whose clusters (one per KV head) are all resident at
        // once; otherwise take the largest schedulable one
        int nclusters = 0;
        if (cudaOccupancyMaxActiveClusters(&nclusters, k, &cfg) != cudaSuccess || nclusters < 1) {
            cudaGetLastError();
            continue;
        }
        if (nclusters < a.n_kv_heads && ns > 4) continue;
        cfg.numAttrs = a.pdl ? 2 : 1;
        TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, k, P));
        return TQB200_OK;
    }
    return TQB200_ERR_UNSUPPORTED;
}

template <typename KV>
int launch_kv(const AttnArgs &a, cudaStream_t st) {
    const int G = a.n_heads / a.n_kv_heads;
#define TQ_TMA_CASE(HDV, GV)                                                              \
    if (a.head_dim == HDV && G == GV)                                                      \
        return a.put ? (a.stamp.base ? launch_t<KV, HDV, GV, true, true>(a, st)                \
                                     : launch_t<KV, HDV, GV, false, true>(a, st))              \
                     : (a.stamp.base ? launch_t<KV, HDV, GV, true, false>(a, st)               \
                                     : launch_t<KV, HDV, GV, false, false>(a, st));
    TQ_TMA_CASE(64, 1) TQ_TMA_CASE(64, 2) TQ_TMA_CASE(64, 4) TQ_TMA_CASE(64, 7)
    TQ_TMA_CASE(64, 8) TQ_TMA_CASE(128, 1) TQ_TMA_CASE(128, 2) TQ_TMA_CASE(128, 4)
    TQ_TMA_CASE(128, 8) TQ_TMA_CASE(32, 1) TQ_TMA_CASE(32, 2) TQ_TMA_CASE(32, 4)
    TQ_TMA_CASE(32, 8)
#undef TQ_TMA_CASE
    return TQB200_ERR_UNSUPPORTED;
}

}  // namespace

int launch_attention_tma(const AttnArgs &a, cudaStream_t st) {
    if (a.n_kv_heads <= 0 || a.n_heads % a.n_kv_heads != 0) return TQB200_ERR_UNSUPPORTED;
    if (((uintptr_t)a.k | (uintptr_t)a.v) & 15u) return TQB200_ERR_UNSUPPORTED;
    return a.kv_fp16 ? launch_kv<uint16_t>(a, st) : launch_kv<float>(a, st);
}

}  // namespace tqb200
