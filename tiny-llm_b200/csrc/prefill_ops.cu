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

template <int HD>
struct ApSmem {
    static constexpr int LD = HD + 4;  // row pitch (floats): conflict-free 128-bit loads
    static constexpr size_t bytes =
        ((size_t)kApRows * LD + 2 * (size_t)kApKeys * LD + (size_t)kApRows * (kApKeys + 1)) * 4;
};

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

__device__ __forceinline__ float4 ld4(const uint16_t *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    return make_float4(h2f((uint16_t)(u.x & 0xFFFFu)), h2f((uint16_t)(u.x >> 16)),
                       h2f((uint16_t)(u.y & 0xFFFFu)), h2f((uint16_t)(u.y >> 16)));
}

template <typename KV, int HD>
__global__ void __launch_bounds__(kApThreads, 2)
attn_prefill_kernel(const float *__restrict__ q, const KV *__restrict__ kc, const KV *__restrict__ vc,
                    int p0, int n, int H, int KVH, int max_seq, float scale, float *__restrict__ out) {
    constexpr int LD = ApSmem<HD>::LD;
    constexpr int NU = HD / 64;  // float4 column blocks per thread in P.V
    extern __shared__ __align__(16) float sm[];
    float *Qs = sm;                          // [kApRows][LD]
    float *Ks = Qs + kApRows * LD;           // [kApKeys][LD]
    float *Vs = Ks + kApKeys * LD;           // [kApKeys][LD]
    float *Ps = Vs + kApKeys * LD;           // [kApRows][kApKeys + 1]
    const int tid = threadIdx.x;
    const int g = H / KVH;
    const int tq = kApRows / g;              // tokens per CTA
    const int kh = blockIdx.y;
    const int t0 = blockIdx.x * tq;
    const int rows = min(tq, n - t0) * g;    // live rows; row r = token t0 + r/g, head kh*g + r%g
    const size_t qld = (size_t)H * HD;
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
    const int kv_end = p0 + min(t0 + tq, n);  // keys [0, kv_end)
    const KV *kb_base = kc + (size_t)kh * max_seq * HD;
    const KV *vb_base = vc + (size_t)kh * max_seq * HD;
    for (int kb = 0; kb < kv_end; kb += kApKeys) {
        __syncthreads();  // previous tile's K/V reads done (and Q staged, first time)
        for (int i = tid; i < kApKeys * (HD / 4); i += kApThreads) {
            const int r = i / (HD / 4), c = 4 * (i % (HD / 4));
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (kb + r < kv_end) {
                kv = ld4(kb_base + (size_t)(kb + r) * HD + c);
                vv = ld4(vb_base + (size_t)(kb + r) * HD + c);
            }
            *reinterpret_cast<float4 *>(Ks + r * LD + c) = kv;
            *reinterpret_cast<float4 *>(Vs + r * LD + c) = vv;
        }
        __syncthreads();
        float s[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = 0.0f;
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            const float4 k0 = ld4(Ks + tc * LD + d), k1 = ld4(Ks + (tc + 16) * LD + d);
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
                const float4 vv = ld4(Vs + j * LD + 4 * tc + 64 * u);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    acc[i][4 * u + 0] = fmaf(p[i], vv.x, acc[i][4 * u + 0]);
                    acc[i][4 * u + 1] = fmaf(p[i], vv.y, acc[i][4 * u + 1]);
                    acc[i][4 * u + 2] = fmaf(p[i], vv.z, acc[i][4 * u + 2]);
                    acc[i][4 * u + 3] = fmaf(p[i], vv.w, acc[i][4 * u + 3]);
                }
            }
        }
        __syncwarp();  // P of this tile read before the next tile rewrites it
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

template <typename KV, int HD>
int launch_ap(const AttnPrefillArgs &a, cudaStream_t st) {
    const size_t smem = ApSmem<HD>::bytes;
    static KernelSmem once;
    int limit = 0;
    TQ_CUDA_TRY(smem_limit_once(attn_prefill_kernel<KV, HD>, once, &limit));
    TQ_CHECK_ARG((int)smem <= limit, "attention prefill: %zu B shared memory", smem);
    const int g = a.n_heads / a.n_kv_heads;
    const int tq = kApRows / g;
    const dim3 grid((a.n + tq - 1) / tq, a.n_kv_heads);
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

__global__ void __launch_bounds__(kPlanThreads) moe_plan_kernel(const MoePlanArgs a) {
    extern __shared__ int s_idx[];  // [A]
    __shared__ int s_cnt[kMoePlanMaxExperts];
    __shared__ int s_off[kMoePlanMaxExperts];
    __shared__ int s_npre[kMoePlanMaxExperts];   // padded columns before expert e
    __shared__ int s_tgu[kMoePlanMaxExperts];    // first gate/up tile of expert e
    __shared__ int s_tdn[kMoePlanMaxExperts];    // first down tile of expert e
    __shared__ int s_job[kMoePlanMaxExperts];    // compacted index of expert e (-1: no tokens)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int A = a.n * a.k, E = a.E;
    for (int e = tid; e < E; e += kPlanThreads) s_cnt[e] = 0;
    __syncthreads();
    for (int i = tid; i < A; i += kPlanThreads) {
        int e = a.idx[i];
        if (e < 0 || e >= E) {  // cannot come from the top-k kernel; keep the plan in bounds
            if (a.status) atomicExch(a.status, kDevBadExpert);
            e = 0;
        }
        s_idx[i] = e;
        atomicAdd(&s_cnt[e], 1);
    }
    __syncthreads();
    const int mt_gu = (a.mi + kMmTileRows - 1) / kMmTileRows;
    const int mt_dn = (a.H + kMmTileRows - 1) / kMmTileRows;
    if (tid == 0) {
        int off = 0, npre = 0, tgu = 0, tdn = 0, nj = 0;
        for (int e = 0; e < E; ++e) {
            const int c = s_cnt[e], npad = (c + 15) & ~15, ct = (npad + a.nt - 1) / a.nt;
            s_off[e] = off;
            s_npre[e] = npre;
            s_tgu[e] = tgu;
            s_tdn[e] = tdn;
            s_job[e] = c > 0 ? nj++ : -1;
            off += c;
            npre += npad;
            tgu += 2 * mt_gu * ct;
            tdn += mt_dn * ct;
        }
        a.ntiles[0] = tgu;
        a.ntiles[1] = tdn;
    }
    __syncthreads();
    const long long cs_gu = (long long)((a.H + a.G - 1) / a.G) * (a.G + 16);   // plane elems per column
    const long long cs_dn = (long long)((a.mi + a.G - 1) / a.G) * (a.G + 16);
    for (int e = tid; e < E; e += kPlanThreads) {
        const int c = s_cnt[e], off = s_off[e];
        const long long bgu = cs_gu * s_npre[e], bdn = cs_dn * s_npre[e];
        MmPackJob pg;
        pg.x = a.xn;
        pg.cols = a.rows + off;
        pg.ldx = a.H;
        pg.N = c;
        pg.b_off = bgu;
        a.pack_gu[e] = pg;
        MmPackJob pd;
        pd.x = a.act + (size_t)off * a.mi;
        pd.cols = nullptr;
        pd.ldx = a.mi;
        pd.N = c;
        pd.b_off = bdn;
        a.pack_dn[e] = pd;
        const int jx = s_job[e];
        if (jx < 0) continue;
        const int ct = (((c + 15) & ~15) + a.nt - 1) / a.nt;
        for (int h = 0; h < 2; ++h) {
            MmJob j;
            j.w = (h ? a.wu : a.wg) + (size_t)e * a.wgu_stride;
            j.y = (h ? a.ubuf : a.hbuf) + (size_t)off * a.mi;
            j.M = a.mi;
            j.N = c;
            j.ldy = a.mi;
            j.tile_begin = s_tgu[e] + h * mt_gu * ct;
            j.b_off = bgu;
            j.resid = nullptr;
            j.bias = nullptr;
            a.jobs_gu[2 * jx + h] = j;
            for (int i = 0; i < mt_gu * ct; ++i) a.tile_gu[j.tile_begin + i] = 2 * jx + h;
        }
        MmJob j;
        j.w = a.wd + (size_t)e * a.wd_stride;
        j.y = a.obuf + (size_t)off * a.H;
        j.M = a.H;
        j.N = c;
        j.ldy = a.H;
        j.tile_begin = s_tdn[e];
        j.b_off = bdn;
        j.resid = nullptr;
        j.bias = nullptr;
        a.jobs_dn[jx] = j;
        for (int i = 0; i < mt_dn * ct; ++i) a.tile_dn[j.tile_begin + i] = jx;
    }
    // stable scatter: a warp per expert, assignments in order, ranks by ballot
    for (int e = warp; e < E; e += kPlanThreads / 32) {
        int run = s_off[e];
        for (int a0 = 0; a0 < A; a0 += 32) {
            const int i = a0 + lane;
            const bool hit = i < A && s_idx[i] == e;
            const unsigned mask = __ballot_sync(0xffffffffu, hit);
            if (hit) {
                const int row = run + __popc(mask & ((1u << lane) - 1u));
                a.rows[row] = i / a.k;
                a.slot[i] = row;
            }
            run += __popc(mask);
        }
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
    const size_t smem = (size_t)a.n * a.k * 4;
    TQ_CHECK_ARG(smem <= 96 * 1024, "moe plan: %d assignments", a.n * a.k);
    static KernelSmem once;
    int limit = 0;
    TQ_CUDA_TRY(smem_limit_once(moe_plan_kernel, once, &limit));
    moe_plan_kernel<<<1, kPlanThreads, smem, st>>>(a);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

}  // namespace tqb200
