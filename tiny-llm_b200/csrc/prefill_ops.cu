// prefill_ops.cu — the batched (prompt) pieces of the engine that have no decode
// counterpart: causal GQA attention over a block of new tokens, and the per-expert
// bucketing of a MoE layer's token assignments that plans the grouped tensor-core GEMMs.
//
// Reference semantics: a prompt of n tokens at positions p0 .. p0+n-1 gives the same
// hidden states as n calls of QwenModel::forward_token (runtime/qwen_forward_token.cpp:
// 83-742), whose attention for the token at position p reads the keys and values of
// positions 0..p (runtime/qwen_forward_token.cpp:300-380); the MoE layer sends each token
// to its top-k experts and sums their outputs in router order
// (runtime/qwen_forward_token.cpp:478-631; the batched grouping of
// forward_prefill_moe_batch, runtime/qwen_forward_prefill.cpp:425-753).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace tqb200 {

namespace {

// ------------------------------------------------------------------ causal attention
// CTA = one KV head x a block of tokens: its kApRows query rows are (token, head of the
// GQA group) pairs, so every K/V tile staged in shared memory serves all of them.  Per
// 32-key tile: scores as a 64x32 product (thread = 4 rows x 2 keys, 128-bit shared
// loads along the head dimension), causal mask, online softmax across the 16 threads of
// a row group, then P.V (thread = 4 rows x HD/16 dims).  A row group's 16 threads are one
// half-warp, so P passes between the two products with a warp barrier only.
constexpr int kApRows = 64;
constexpr int kApKeys = 32;
constexpr int kApThreads = 256;

// Shared memory: Q [kApRows][HD+4] f32, K/V tiles double-buffered in the cache's own type
// ([2][K|V][kApKeys][HD + 16 B]), P [kApRows][kApKeys+1] f32.  The next tile's K/V rows
// stream in with cp.async (16-byte pieces, zero-filled past the causal end) while the
// current tile is consumed.
template <typename KV, int HD>
struct ApSmem {
    static constexpr int LD = HD + 4;                  // Q row pitch (floats)
    static constexpr int LDK = HD + 16 / (int)sizeof(KV);  // K/V row pitch (elements)
    static constexpr size_t q_bytes = (size_t)kApRows * LD * 4;
    static constexpr size_t kv_bytes = 2 * 2 * (size_t)kApKeys * LDK * sizeof(KV);
    static constexpr size_t bytes = q_bytes + kv_bytes + (size_t)kApRows * (kApKeys + 1) * 4;
};

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

__device__ __forceinline__ float4 ld4(const uint16_t *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    return make_float4(h2f((uint16_t)(u.x & 0xFFFFu)), h2f((uint16_t)(u.x >> 16)),
                       h2f((uint16_t)(u.y & 0xFFFFu)), h2f((uint16_t)(u.y >> 16)));
}

__device__ __forceinline__ void cp16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <typename KV, int HD>
__device__ __forceinline__ void attn_block(const float *__restrict__ q, const KV *__restrict__ kc,
                                           const KV *__restrict__ vc, int p0, int n, int H, int KVH,
                                           int max_seq, float scale, float *__restrict__ out, int qb,
                                           uint8_t *sm) {
    using S = ApSmem<KV, HD>;
    constexpr int LD = S::LD, LDK = S::LDK;
    constexpr int NU = HD / 64;  // float4 column blocks per thread in P.V
    constexpr int CPR = HD * (int)sizeof(KV) / 16;  // 16-byte pieces per K/V row
    float *Qs = reinterpret_cast<float *>(sm);                          // [kApRows][LD]
    KV *Kr = reinterpret_cast<KV *>(sm + S::q_bytes);                   // [2][2][kApKeys][LDK]
    float *Ps = reinterpret_cast<float *>(sm + S::q_bytes + S::kv_bytes);  // [kApRows][kApKeys + 1]
    const int tid = threadIdx.x;
    const int g = H / KVH;
    const int tq = kApRows / g;              // tokens per CTA
    const int kh = blockIdx.y;
    const int t0 = qb * tq;
    const int rows = min(tq, n - t0) * g;    // live rows; row r = token t0 + r/g, head kh*g + r%g
    const size_t qld = (size_t)H * HD;
    const int kv_end = p0 + min(t0 + tq, n);  // keys [0, kv_end)
    const KV *kb_base = kc + (size_t)kh * max_seq * HD;
    const KV *vb_base = vc + (size_t)kh * max_seq * HD;
    const int ntile = (kv_end + kApKeys - 1) / kApKeys;
    auto issue = [&](int t) {  // K/V rows of tile t into buffer t & 1
        KV *Kb = Kr + (size_t)(t & 1) * 2 * kApKeys * LDK;
        KV *Vb = Kb + kApKeys * LDK;
        const int kb = t * kApKeys;
        for (int i = tid; i < kApKeys * CPR; i += kApThreads) {
            const int r = i / CPR, c = (i % CPR) * (16 / (int)sizeof(KV));
            const bool ok = kb + r < kv_end;
            const size_t off = (size_t)(ok ? kb + r : 0) * HD + c;
            cp16(Kb + r * LDK + c, kb_base + off, ok);
            cp16(Vb + r * LDK + c, vb_base + off, ok);
        }
        cp_commit();
    };
    issue(0);
    for (int i = tid; i < kApRows * (HD / 4); i += kApThreads) {
        const int r = i / (HD / 4), c = 4 * (i % (HD / 4));
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < rows) v = ld4(q + (size_t)(t0 + r / g) * qld + (size_t)(kh * g + r % g) * HD + c);
        *reinterpret_cast<float4 *>(Qs + r * LD + c) = v;
    }
    const int tr = tid >> 4, tc = tid & 15;  // rows 4tr..4tr+3
    float m[4], l[4], acc[4][4 * NU];
    int qpos[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
        const int r = 4 * tr + i;
        qpos[i] = r < rows ? p0 + t0 + r / g : -1;  // dead rows see no key
#pragma unroll
        for (int c = 0; c < 4 * NU; ++c) acc[i][c] = 0.0f;
    }
    for (int t = 0; t < ntile; ++t) {
        if (t + 1 < ntile) {
            issue(t + 1);
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();  // tile t (and Q, the first time) visible to every thread
        const KV *Ks = Kr + (size_t)(t & 1) * 2 * kApKeys * LDK;
        const KV *Vs = Ks + kApKeys * LDK;
        const int kb = t * kApKeys;
        float s[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = 0.0f;
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            const float4 k0 = ld4(Ks + tc * LDK + d), k1 = ld4(Ks + (tc + 16) * LDK + d);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 qv = ld4(Qs + (4 * tr + i) * LD + d);
                s[i][0] = fmaf(qv.x, k0.x, s[i][0]);
                s[i][0] = fmaf(qv.y, k0.y, s[i][0]);
                s[i][0] = fmaf(qv.z, k0.z, s[i][0]);
                s[i][0] = fmaf(qv.w, k0.w, s[i][0]);
                s[i][1] = fmaf(qv.x, k1.x, s[i][1]);
                s[i][1] = fmaf(qv.y, k1.y, s[i][1]);
                s[i][1] = fmaf(qv.z, k1.z, s[i][1]);
                s[i][1] = fmaf(qv.w, k1.w, s[i][1]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float v0 = (kb + tc <= qpos[i]) ? s[i][0] * scale : -INFINITY;
            const float v1 = (kb + tc + 16 <= qpos[i]) ? s[i][1] * scale : -INFINITY;
            float tmax = fmaxf(v0, v1);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
            const float mn = fmaxf(m[i], tmax);
            const bool live = mn != -INFINITY;
            const float corr = live ? __expf(m[i] - mn) : 1.0f;
            const float e0 = live ? __expf(v0 - mn) : 0.0f;
            const float e1 = live ? __expf(v1 - mn) : 0.0f;
            float ps = e0 + e1;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            l[i] = l[i] * corr + ps;
            m[i] = mn;
#pragma unroll
            for (int c = 0; c < 4 * NU; ++c) acc[i][c] *= corr;
            Ps[(4 * tr + i) * (kApKeys + 1) + tc] = e0;
            Ps[(4 * tr + i) * (kApKeys + 1) + tc + 16] = e1;
        }
        __syncwarp();
        const int kn = min(kApKeys, kv_end - kb);
        for (int j = 0; j < kn; ++j) {
            float p[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) p[i] = Ps[(4 * tr + i) * (kApKeys + 1) + j];
#pragma unroll
            for (int u = 0; u < NU; ++u) {
                const float4 vv = ld4(Vs + j * LDK + 4 * tc + 64 * u);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    acc[i][4 * u + 0] = fmaf(p[i], vv.x, acc[i][4 * u + 0]);
                    acc[i][4 * u + 1] = fmaf(p[i], vv.y, acc[i][4 * u + 1]);
                    acc[i][4 * u + 2] = fmaf(p[i], vv.z, acc[i][4 * u + 2]);
                    acc[i][4 * u + 3] = fmaf(p[i], vv.w, acc[i][4 * u + 3]);
                }
            }
        }
        __syncthreads();  // buffer t & 1 and P consumed before they are refilled
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = 4 * tr + i;
        if (r >= rows) continue;
        const float inv = 1.0f / l[i];
        float *o = out + (size_t)(t0 + r / g) * qld + (size_t)(kh * g + r % g) * HD;
#pragma unroll
        for (int u = 0; u < NU; ++u)
            *reinterpret_cast<float4 *>(o + 4 * tc + 64 * u) =
                make_float4(acc[i][4 * u] * inv, acc[i][4 * u + 1] * inv, acc[i][4 * u + 2] * inv,
                            acc[i][4 * u + 3] * inv);
    }
}

// Causal work grows with the token index, so CTA j takes query blocks j and nb-1-j.
template <typename KV, int HD>
__global__ void __launch_bounds__(kApThreads, 2)
attn_prefill_kernel(const float *__restrict__ q, const KV *__restrict__ kc, const KV *__restrict__ vc,
                    int p0, int n, int H, int KVH, int max_seq, float scale, float *__restrict__ out) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int nb = (n + kApRows / (H / KVH) - 1) / (kApRows / (H / KVH));
    const int j = blockIdx.x;
    attn_block<KV, HD>(q, kc, vc, p0, n, H, KVH, max_seq, scale, out, j, sm);
    if (nb - 1 - j != j) {
        __syncthreads();  // the first block's shared-memory reads are done
        attn_block<KV, HD>(q, kc, vc, p0, n, H, KVH, max_seq, scale, out, nb - 1 - j, sm);
    }
}

template <typename KV, int HD>
int launch_ap(const AttnPrefillArgs &a, cudaStream_t st) {
    const size_t smem = ApSmem<KV, HD>::bytes;
    static KernelSmem once;
    int limit = 0;
    TQ_CUDA_TRY(smem_limit_once(attn_prefill_kernel<KV, HD>, once, &limit));
    TQ_CHECK_ARG((int)smem <= limit, "attention prefill: %zu B shared memory", smem);
    const int g = a.n_heads / a.n_kv_heads;
    const int tq = kApRows / g;
    const int nb = (a.n + tq - 1) / tq;
    const dim3 grid((nb + 1) / 2, a.n_kv_heads);
    attn_prefill_kernel<KV, HD><<<grid, kApThreads, smem, st>>>(
        a.q, (const KV *)a.k, (const KV *)a.v, a.p0, a.n, a.n_heads, a.n_kv_heads, a.max_seq,
        a.scale, a.out);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

// ------------------------------------------------------------------ MoE grouping plan
// One CTA.  The n*k assignments (token t, choice j) -> expert idx[t*k+j] are bucketed by
// expert, in assignment order inside a bucket; bucket row `row` holds token rows[row],
// and assignment a sits at bucket row slot[a].  From the bucket sizes it writes the
// grouped GEMM jobs (gate and up per expert with tokens, then down), their X-pack jobs
// and the tile -> job maps, all on the device, so a MoE layer needs no host round trip.
constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;

// Exclusive prefix sums over e < E (E <= kPlanThreads) of four per-expert values, by
// every thread of the CTA (thread e holds expert e's values).
__device__ void plan_scan4(int v[4], int tot[4], int (*wt)[4]) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    int inc[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        inc[q] = v[q];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, inc[q], o);
            if (lane >= o) inc[q] += u;
        }
    }
    if (lane == 31)
        for (int q = 0; q < 4; ++q) wt[warp][q] = inc[q];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int x = wt[lane][q];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += u;
            }
            wt[lane][q] = x;  // inclusive over warps
        }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int before = warp ? wt[warp - 1][q] : 0;
        const int excl = before + inc[q] - v[q];
        tot[q] = wt[kPlanWarps - 1][q];
        v[q] = excl;
    }
    __syncthreads();  // wt reusable
}

// One CTA.  The n*k assignments (token t, choice j) -> expert idx[t*k+j] are bucketed by
// expert, in assignment order inside a bucket; bucket row `row` holds token rows[row],
// and assignment a sits at bucket row slot[a].  From the bucket sizes it writes the
// grouped GEMM jobs (gate and up per expert with tokens, then down), their X-pack jobs
// and the tile -> job maps, all on the device, so a MoE layer needs no host round trip.
// Ranking: warp w takes a contiguous slice of the assignments and ranks each within
// (slice, expert) with __match_any_sync 32 at a time; a per-expert scan over the slices
// then places every slice's run after the previous slices' runs.
__global__ void __launch_bounds__(kPlanThreads) moe_plan_kernel(const MoePlanArgs a) {
    extern __shared__ int sm_plan[];
    const int A = a.n * a.k, E = a.E;
    int *s_idx = sm_plan;            // [A] expert of assignment
    int *s_rank = s_idx + A;         // [A] rank inside (slice, expert)
    int *s_wc = s_rank + A;          // [kPlanWarps][E] slice counts, then slice offsets
    __shared__ int s_off[kMoePlanMaxExperts], s_npre[kMoePlanMaxExperts];
    __shared__ int s_tgu[kMoePlanMaxExperts], s_tdn[kMoePlanMaxExperts], s_job[kMoePlanMaxExperts];
    __shared__ int s_wt[kPlanWarps][4];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < A; i += kPlanThreads) {
        int e = a.idx[i];
        if (e < 0 || e >= E) {  // cannot come from the top-k kernel; keep the plan in bounds
            if (a.status) atomicExch(a.status, kDevBadExpert);
            e = 0;
        }
        s_idx[i] = e;
    }
    for (int i = tid; i < kPlanWarps * E; i += kPlanThreads) s_wc[i] = 0;
    __syncthreads();
    const int S = (((A + kPlanWarps - 1) / kPlanWarps) + 31) & ~31;  // slice length
    {
        int *wc = s_wc + warp * E;
        const int i1 = min(A, (warp + 1) * S);
        for (int a0 = warp * S; a0 < i1; a0 += 32) {
            const int i = a0 + lane;
            const int e = i < i1 ? s_idx[i] : -1 - lane;  // idle lanes: keys of their own
            const unsigned peers = __match_any_sync(0xffffffffu, e);
            const int leader = __ffs(peers) - 1;
            int base = 0;
            if (lane == leader && i < i1) {
                base = wc[e];
                wc[e] = base + __popc(peers);
            }
            base = __shfl_sync(0xffffffffu, base, leader);
            if (i < i1) s_rank[i] = base + __popc(peers & ((1u << lane) - 1u));
            __syncwarp();
        }
    }
    __syncthreads();
    int v[4] = {0, 0, 0, 0}, tot[4];
    const int mt_gu = (a.mi + kMmTileRows - 1) / kMmTileRows;
    const int mt_dn = (a.H + kMmTileRows - 1) / kMmTileRows;
    int c = 0;
    const bool loc = tid < E && (a.e_local == 0 || (tid >= a.e0 && tid < a.e0 + a.e_local));
    if (tid < E) {  // slice offsets inside the bucket, and the bucket size
        for (int w = 0; w < kPlanWarps; ++w) {
            const int x = s_wc[w * E + tid];
            s_wc[w * E + tid] = c;
            c += x;
        }
        const int npad = (c + 15) & ~15, ct = (npad + a.nt - 1) / a.nt;
        v[0] = c;
        v[1] = npad;
        v[2] = loc ? 2 * mt_gu * ct : 0;  // another rank's expert: no tiles here
        v[3] = loc ? mt_dn * ct : 0;
    }
    plan_scan4(v, tot, s_wt);
    int jv[4] = {loc && c > 0 ? 1 : 0, 0, 0, 0}, jt[4];
    plan_scan4(jv, jt, s_wt);
    if (tid < E) {
        s_off[tid] = v[0];
        s_npre[tid] = v[1];
        s_tgu[tid] = v[2];
        s_tdn[tid] = v[3];
        s_job[tid] = loc && c > 0 ? jv[0] : -1;
    }
    if (tid == 0) {
        a.ntiles[0] = tot[2];
        a.ntiles[1] = tot[3];
        a.ntiles[2] = tot[1] / 8;
    }
    __syncthreads();
    const long long cs_gu = (long long)((a.H + a.G - 1) / a.G) * (a.G + 16);   // plane elems per column
    const long long cs_dn = (long long)((a.mi + a.G - 1) / a.G) * (a.G + 16);
    for (int e = tid; e < E; e += kPlanThreads) {
        const int off = s_off[e];
        const int cnt = (e + 1 < E ? s_off[e + 1] : tot[0]) - off;
        const long long bgu = cs_gu * s_npre[e], bdn = cs_dn * s_npre[e];
        MmPackJob pg;
        pg.x = a.xn;
        pg.u = nullptr;
        pg.cols = a.rows + off;
        pg.ldx = a.H;
        pg.N = cnt;
        pg.b_off = bgu;
        pg.col0 = s_npre[e];
        a.pack_gu[e] = pg;
        MmPackJob pd;
        pd.x = a.hbuf + (size_t)off * a.mi;
        pd.u = a.ubuf + (size_t)off * a.mi;
        pd.cols = nullptr;
        pd.ldx = a.mi;
        pd.N = cnt;
        pd.b_off = bdn;
        pd.col0 = s_npre[e];
        a.pack_dn[e] = pd;
        for (int b = 0; b < ((cnt + 15) & ~15) / 8; ++b) a.pack_map[s_npre[e] / 8 + b] = e;
        const int jx = s_job[e];
        if (jx < 0) continue;
        const int ct = (((cnt + 15) & ~15) + a.nt - 1) / a.nt;
        for (int h = 0; h < 2; ++h) {
            MmJob j;
            const int el = e - (a.e_local ? a.e0 : 0);  // the rank's copy of expert e
            j.w = (h ? a.wu : a.wg) + (size_t)el * a.wgu_stride;
            j.tmap = h ? a.tmu : a.tmg;
            j.tz = el;
            j.y = (h ? a.ubuf : a.hbuf) + (size_t)off * a.mi;
            j.M = a.mi;
            j.N = cnt;
            j.ldy = a.mi;
            j.tile_begin = s_tgu[e] + h * mt_gu * ct;
            j.b_off = bgu;
            j.resid = nullptr;
            j.bias = nullptr;
            a.jobs_gu[2 * jx + h] = j;
            for (int i = 0; i < mt_gu * ct; ++i) a.tile_gu[j.tile_begin + i] = 2 * jx + h;
        }
        MmJob j;
        const int el = e - (a.e_local ? a.e0 : 0);
        j.w = a.wd + (size_t)el * a.wd_stride;
        j.tmap = a.tmd;
        j.tz = el;
        j.y = a.obuf + (size_t)off * a.H;
        j.M = a.H;
        j.N = cnt;
        j.ldy = a.H;
        j.tile_begin = s_tdn[e];
        j.b_off = bdn;
        j.resid = nullptr;
        j.bias = nullptr;
        a.jobs_dn[jx] = j;
        for (int i = 0; i < mt_dn * ct; ++i) a.tile_dn[j.tile_begin + i] = jx;
    }
    for (int i = tid; i < A; i += kPlanThreads) {  // bucket row of every assignment
        const int e = s_idx[i], w = i / S;
        const int row = s_off[e] + s_wc[w * E + e] + s_rank[i];
        a.rows[row] = i / a.k;
        a.slot[i] = row;
    }
}

}  // namespace

int launch_attn_prefill(const AttnPrefillArgs &a, cudaStream_t st) {
    TQ_CHECK_ARG(a.n > 0 && a.p0 >= 0 && a.p0 + a.n <= a.max_seq, "attention prefill: tokens %d at %d (max %d)",
                 a.n, a.p0, a.max_seq);
    TQ_CHECK_ARG(a.n_kv_heads > 0 && a.n_heads % a.n_kv_heads == 0 &&
                     a.n_heads / a.n_kv_heads <= kApRows && kApRows % (a.n_heads / a.n_kv_heads) == 0,
                 "attention prefill: %d heads over %d KV heads", a.n_heads, a.n_kv_heads);
    TQ_CHECK_ARG(((uintptr_t)a.q & 15) == 0 && ((uintptr_t)a.out & 15) == 0 &&
                     ((uintptr_t)a.k & 15) == 0 && ((uintptr_t)a.v & 15) == 0,
                 "attention prefill: buffers not 16-byte aligned");
    if (a.head_dim == 128)
        return a.kv_fp16 ? launch_ap<uint16_t, 128>(a, st) : launch_ap<float, 128>(a, st);
    if (a.head_dim == 64)
        return a.kv_fp16 ? launch_ap<uint16_t, 64>(a, st) : launch_ap<float, 64>(a, st);
    return set_error(TQB200_ERR_UNSUPPORTED, "attention prefill: head_dim %d (64 or 128)", a.head_dim);
}

bool attn_prefill_supported(int n_heads, int n_kv_heads, int head_dim) {
    if (n_kv_heads <= 0 || n_heads % n_kv_heads) return false;
    const int g = n_heads / n_kv_heads;
    return (head_dim == 64 || head_dim == 128) && g <= kApRows && kApRows % g == 0;
}

size_t moe_plan_smem_bytes(int n, int k, int E) {
    return (size_t)n * k * 8 + (size_t)kPlanWarps * E * 4;
}

int moe_plan_max_cols(int n, int k, int E) {
    const long long A = (long long)n * k, live = std::min<long long>(E, A);
    return (int)(A + 15 * live);
}

int moe_plan_max_tiles(int n, int k, int E, int M, int nt) {
    const long long A = (long long)n * k, live = std::min<long long>(E, A);
    const long long cols = A + 15 * live;  // padded columns over all experts
    const long long mt = (M + kMmTileRows - 1) / kMmTileRows;
    return (int)(mt * (cols / nt + live));
}

long long moe_plan_plane_elems(int n, int k, int E, int K, int G) {
    const long long A = (long long)n * k, live = std::min<long long>(E, A);
    return (long long)((K + G - 1) / G) * (G + 16) * (A + 15 * live);
}

int launch_moe_plan(const MoePlanArgs &a, cudaStream_t st) {
    TQ_CHECK_ARG(a.E > 0 && a.E <= kMoePlanMaxExperts && a.k > 0 && a.n > 0,
                 "moe plan: E %d k %d n %d", a.E, a.k, a.n);
    TQ_CHECK_ARG(a.e_local >= 0 && a.e0 >= 0 && a.e0 + a.e_local <= a.E,
                 "moe plan: local experts [%d, %d) outside %d", a.e0, a.e0 + a.e_local, a.E);
    const size_t smem = moe_plan_smem_bytes(a.n, a.k, a.E);
    TQ_CHECK_ARG(smem <= kMoePlanMaxSmem, "moe plan: %d assignments over %d experts", a.n * a.k, a.E);
    static KernelSmem once;
    int limit = 0;
    TQ_CUDA_TRY(smem_limit_once(moe_plan_kernel, once, &limit));
    moe_plan_kernel<<<1, kPlanThreads, smem, st>>>(a);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

}  // namespace tqb200
