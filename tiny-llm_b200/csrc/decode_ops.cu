// decode_ops.cu — the non-matvec ops of one decode step, sm_100a.
//
//   rmsnorm        rmsnorm_ref          kernels/rmsnorm/rmsnorm_ref.cpp:48-78
//   rope           rope_ref             kernels/rope/rope_ref.cpp:56-117
//   qk-norm+rope+kv-append (engine)     runtime/qwen_forward_token.cpp:423-446,
//                                       runtime/kv_cache.cpp:120-135
//   attention      attention_decode_ref kernels/attention/attention_decode_ref.cpp:53-143
//                  (fp16 KV: the same math on decoded halves)
//   swiglu         swiglu_ref           kernels/silu/swiglu_ref.cpp:41-52
//   argmax         argmax_ref           kernels/argmax/argmax_ref.cpp:42-54
//   topk_softmax   topk_softmax_ref     kernels/topk_softmax/topk_softmax_ref.cpp:41-78
//   embed          qwen_forward_token.cpp:121-164 (f32 copy / f16 decode / i4 dequant row)
//
// Rounding: where the reference rounds in fp32 the kernels use the _rn
// intrinsics so nvcc cannot contract a multiply and an add into an FMA the
// reference does not perform; reductions the reference does in double are
// done in double.  Transcendentals call CUDA's expf/powf/cosf/sinf (full
// precision, never the fast intrinsics), so those ops agree to a few ulp.
#include <float.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace tqb200 {

namespace {

__device__ __forceinline__ double block_sum_d(double v, double *sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum_d(v);
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    double r = 0.0;
    if (warp == 0) {
        r = lane < nw ? sh[lane] : 0.0;
        r = warp_sum_d(r);
        if (lane == 0) sh[0] = r;
    }
    __syncthreads();
    return sh[0];
}

// y = rmsnorm(x) * w over `rows` independent rows of n (one CTA per row).
__global__ void rmsnorm_rows_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                    float *__restrict__ y, int n, float eps) {
    __shared__ double sh[32];
    const float *xr = x + (size_t)blockIdx.x * n;
    float *yr = y + (size_t)blockIdx.x * n;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const double v = (double)xr[i];
        ss += v * v;
    }
    ss = block_sum_d(ss, sh);
    const float mean_sq = (float)(ss / n);
    const float scale = 1.0f / sqrtf(__fadd_rn(mean_sq, eps));
    for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], scale), w[i]);
}

// The same with the row held in registers as float4s (n % 4 == 0, n <= 4 * 4 * 256,
// 16-byte aligned rows): x is read once.  Same double sum of squares and float
// operations; in place (y == x) is safe, each thread writing only what it read.
constexpr int kRmsV = 4;  // float4s per thread

__global__ void __launch_bounds__(256) rmsnorm_rows_v4_kernel(const float *__restrict__ x,
                                                              const float *__restrict__ w,
                                                              float *__restrict__ y, int n, float eps) {
    __shared__ double sh[32];
    const int n4 = n >> 2;
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)blockIdx.x * n);
    float4 *yr = reinterpret_cast<float4 *>(y + (size_t)blockIdx.x * n);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    float4 v[kRmsV];
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < kRmsV; ++j) {
        const int i = threadIdx.x + 256 * j;
        v[j] = i < n4 ? xr[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        ss += (double)v[j].x * (double)v[j].x;
        ss += (double)v[j].y * (double)v[j].y;
        ss += (double)v[j].z * (double)v[j].z;
        ss += (double)v[j].w * (double)v[j].w;
    }
    ss = block_sum_d(ss, sh);
    const float mean_sq = (float)(ss / n);
    const float scale = 1.0f / sqrtf(__fadd_rn(mean_sq, eps));
#pragma unroll
    for (int j = 0; j < kRmsV; ++j) {
        const int i = threadIdx.x + 256 * j;
        if (i < n4) {
            const float4 g = w4[i];
            yr[i] = make_float4(__fmul_rn(__fmul_rn(v[j].x, scale), g.x),
                                __fmul_rn(__fmul_rn(v[j].y, scale), g.y),
                                __fmul_rn(__fmul_rn(v[j].z, scale), g.z),
                                __fmul_rn(__fmul_rn(v[j].w, scale), g.w));
        }
    }
}

// Rotate-half RoPE with the position's cos/sin row (per-op entry point).  The row
// comes from rope_row() on the host: the angle pos * powf(theta, -2i/hd) is so
// ill-conditioned at long positions (a 1-ulp difference in powf moves cos by
// ~1e-4 at pos 4095) that the rotation is only bit-exact with the reference's
// own libm values.
__global__ void rope_kernel(float *__restrict__ q, float *__restrict__ k, int n_heads,
                            int n_kv_heads, int head_dim, const float *__restrict__ cs,
                            const float *__restrict__ sn) {
    const int half = head_dim / 2;
    const int h = blockIdx.x;
    float *v = h < n_heads ? q + (size_t)h * head_dim : k + (size_t)(h - n_heads) * head_dim;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float c = cs[i], s = sn[i];
        const float x0 = v[i], x1 = v[i + half];
        v[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        v[i + half] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
    }
}

// Engine: per-head QK-norm (optional), RoPE from a precomputed [max_seq][hd/2]
// cos/sin table (host-computed with the reference's exact powf/cosf/sinf), and
// the KV append at *pos.  One CTA per head: blocks [0, H) = q heads,
// [H, H+KVH) = k heads (rope + store), [H+KVH, H+2KVH) = v heads (store).
template <typename KV>
__global__ void qk_rope_kv_kernel(float *__restrict__ q, const float *__restrict__ k,
                                  const float *__restrict__ v, const float *__restrict__ q_norm,
                                  const float *__restrict__ k_norm, float eps,
                                  const float *__restrict__ cos_tab,
                                  const float *__restrict__ sin_tab, const int *__restrict__ pos_p,
                                  KV *__restrict__ kcache, KV *__restrict__ vcache, int n_heads,
                                  int n_kv_heads, int head_dim, int max_seq) {
    __shared__ double sh[32];
    __shared__ float buf[512];
    const int h = blockIdx.x;
    const int pos = *pos_p + blockIdx.y;  // batched: token blockIdx.y of consecutive rows
    const int half = head_dim / 2;
    q += (size_t)blockIdx.y * n_heads * head_dim;
    k += (size_t)blockIdx.y * n_kv_heads * head_dim;
    v += (size_t)blockIdx.y * n_kv_heads * head_dim;
    if (h >= n_heads + n_kv_heads) {  // value head: plain store
        const int kh = h - n_heads - n_kv_heads;
        KV *dst = vcache + ((size_t)kh * max_seq + pos) * head_dim;
        for (int i = threadIdx.x; i < head_dim; i += blockDim.x) {
            const float val = v[kh * head_dim + i];
            if constexpr (sizeof(KV) == 2) dst[i] = f2h_ref(val);
            else dst[i] = val;
        }
        return;
    }
    const bool is_q = h < n_heads;
    const float *src = is_q ? q + (size_t)h * head_dim : k + (size_t)(h - n_heads) * head_dim;
    const float *nw = is_q ? q_norm : k_norm;
    for (int i = threadIdx.x; i < head_dim; i += blockDim.x) buf[i] = src[i];
    if (nw) {
        double ss = 0.0;
        for (int i = threadIdx.x; i < head_dim; i += blockDim.x) ss += (double)buf[i] * (double)buf[i];
        ss = block_sum_d(ss, sh);
        const float mean_sq = (float)(ss / head_dim);
        const float scale = 1.0f / sqrtf(__fadd_rn(mean_sq, eps));
        for (int i = threadIdx.x; i < head_dim; i += blockDim.x)
            buf[i] = __fmul_rn(__fmul_rn(buf[i], scale), nw[i]);
    }
    __syncthreads();
    const float *cs = cos_tab + (size_t)pos * half;
    const float *sn = sin_tab + (size_t)pos * half;
    float r[2][4];
    int cnt = 0;
    for (int i = threadIdx.x; i < half; i += blockDim.x, ++cnt) {
        const float x0 = buf[i], x1 = buf[i + half], c = cs[i], s = sn[i];
        r[0][cnt & 3] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        r[1][cnt & 3] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
    }
    __syncthreads();
    cnt = 0;
    for (int i = threadIdx.x; i < half; i += blockDim.x, ++cnt) {
        buf[i] = r[0][cnt & 3];
        buf[i + half] = r[1][cnt & 3];
    }
    __syncthreads();
    if (is_q) {
        for (int i = threadIdx.x; i < head_dim; i += blockDim.x) q[(size_t)h * head_dim + i] = buf[i];
    } else {
        const int kh = h - n_heads;
        KV *dst = kcache + ((size_t)kh * max_seq + pos) * head_dim;
        for (int i = threadIdx.x; i < head_dim; i += blockDim.x) {
            if constexpr (sizeof(KV) == 2) dst[i] = f2h_ref(buf[i]);
            else dst[i] = buf[i];
        }
    }
}

// The same step with one warp per head (head_dim <= 256), eight heads per CTA: the
// lane holds elements i and i + head_dim/2 for i = lane + 32e in registers, the
// sum of squares is a warp sum in double, and the norm and rotation are the same
// float operations as the per-CTA form.  Grid (ceil(heads / 8), tokens).
constexpr int kQrWarps = 8, kQrMaxE = 4;

template <typename KV>
__global__ void __launch_bounds__(kQrWarps * 32) qk_rope_kv_warp_kernel(
    float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
    const float *__restrict__ q_norm, const float *__restrict__ k_norm, float eps,
    const float *__restrict__ cos_tab, const float *__restrict__ sin_tab,
    const int *__restrict__ pos_p, KV *__restrict__ kcache, KV *__restrict__ vcache, int n_heads,
    int n_kv_heads, int head_dim, int max_seq) {
    const int lane = threadIdx.x & 31;
    const int h = blockIdx.x * kQrWarps + (threadIdx.x >> 5);
    if (h >= n_heads + 2 * n_kv_heads) return;
    const int pos = *pos_p + blockIdx.y;  // token blockIdx.y of consecutive rows
    q += (size_t)blockIdx.y * n_heads * head_dim;
    k += (size_t)blockIdx.y * n_kv_heads * head_dim;
    v += (size_t)blockIdx.y * n_kv_heads * head_dim;
    if (h >= n_heads + n_kv_heads) {  // value head: plain store
        const int kh = h - n_heads - n_kv_heads;
        KV *dst = vcache + ((size_t)kh * max_seq + pos) * head_dim;
        for (int i = lane; i < head_dim; i += 32) {
            const float val = v[kh * head_dim + i];
            if constexpr (sizeof(KV) == 2) dst[i] = f2h_ref(val);
            else dst[i] = val;
        }
        return;
    }
    const bool is_q = h < n_heads;
    const float *src = is_q ? q + (size_t)h * head_dim : k + (size_t)(h - n_heads) * head_dim;
    const float *nw = is_q ? q_norm : k_norm;
    const int half = head_dim / 2;
    float x0[kQrMaxE], x1[kQrMaxE];
#pragma unroll
    for (int e = 0; e < kQrMaxE; ++e) {
        const int i = lane + 32 * e;
        x0[e] = i < half ? src[i] : 0.0f;
        x1[e] = i < half ? src[i + half] : 0.0f;
    }
    if (nw) {
        double ss = 0.0;
#pragma unroll
        for (int e = 0; e < kQrMaxE; ++e) ss += (double)x0[e] * (double)x0[e] + (double)x1[e] * (double)x1[e];
        ss = warp_sum_d(ss);
        const float mean_sq = (float)(ss / head_dim);
        const float scale = 1.0f / sqrtf(__fadd_rn(mean_sq, eps));
#pragma unroll
        for (int e = 0; e < kQrMaxE; ++e) {
            const int i = lane + 32 * e;
            if (i < half) {
                x0[e] = __fmul_rn(__fmul_rn(x0[e], scale), nw[i]);
                x1[e] = __fmul_rn(__fmul_rn(x1[e], scale), nw[i + half]);
            }
        }
    }
    const float *cs = cos_tab + (size_t)pos * half;
    const float *sn = sin_tab + (size_t)pos * half;
    float *qd = q + (size_t)h * head_dim;
    KV *kd = is_q ? nullptr : kcache + ((size_t)(h - n_heads) * max_seq + pos) * head_dim;
#pragma unroll
    for (int e = 0; e < kQrMaxE; ++e) {
        const int i = lane + 32 * e;
        if (i < half) {
            const float c = cs[i], sv = sn[i];
            const float r0 = __fsub_rn(__fmul_rn(x0[e], c), __fmul_rn(x1[e], sv));
            const float r1 = __fadd_rn(__fmul_rn(x1[e], c), __fmul_rn(x0[e], sv));
            if (is_q) {
                qd[i] = r0;
                qd[i + half] = r1;
            } else if constexpr (sizeof(KV) == 2) {
                kd[i] = f2h_ref(r0);
                kd[i + half] = f2h_ref(r1);
            } else {
                kd[i] = r0;
                kd[i + half] = r1;
            }
        }
    }
}

// ------------------------------------------------------------------ attention
__device__ __forceinline__ void load4(const float *p, float o[4]) {
    const float4 v = *reinterpret_cast<const float4 *>(p);
    o[0] = v.x, o[1] = v.y, o[2] = v.z, o[3] = v.w;
}
__device__ __forceinline__ void load4(const uint16_t *p, float o[4]) {
    const uint2 v = *reinterpret_cast<const uint2 *>(p);
    o[0] = h2f((uint16_t)(v.x & 0xFFFF)), o[1] = h2f((uint16_t)(v.x >> 16));
    o[2] = h2f((uint16_t)(v.y & 0xFFFF)), o[3] = h2f((uint16_t)(v.y >> 16));
}

constexpr int kAttnThreads = 256;

// Split-K (flash-decoding) GQA decode attention.  grid = (n_kv_heads, nsplit).
// CTA (kh, s) handles the G = n_heads/n_kv_heads query heads of KV head kh over
// positions [s*chunk, (s+1)*chunk) of [0, seq): it reads each K/V row once for
// all G heads.  Scores -> smem, exact max/sum softmax over the chunk, P.V, then
// the partial (m, l, o) goes to global scratch; the last CTA of the KV head (an
// atomic ticket) merges the partials and writes out.  seq = *pos_p + 1 when
// pos_p is set (CUDA-graph replays), else seq_len.
template <typename KV, int HD, int G>
__global__ void __launch_bounds__(kAttnThreads)
    attn_split_kernel(const float *__restrict__ q, const KV *__restrict__ kc,
                      const KV *__restrict__ vc, const int *__restrict__ pos_p, int seq_len,
                      int max_seq, int nsplit, float scale, float *__restrict__ part,
                      unsigned int *__restrict__ tickets, float *__restrict__ out) {
    extern __shared__ float sm[];
    float *qs = sm;                              // [G][HD]
    constexpr int kTS = kAttnThreads / (HD / 4);  // position subsets of the P.V phase
    float *red = qs + G * HD;                    // [kTS][G][HD] (P.V partials)
    float *sc = red + kTS * G * HD;              // [chunk_max][G]
    __shared__ float s_m[G], s_l[G];
    __shared__ bool s_last;
    const int kh = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x;
    const int seq = pos_p ? (*pos_p + 1) : seq_len;
    const int chunk = (seq + nsplit - 1) / nsplit;
    const int t0 = split * chunk;
    const int t1 = min(seq, t0 + chunk);
    const int n = max(0, t1 - t0);
    const KV *kbase = kc + (size_t)kh * max_seq * HD;
    const KV *vbase = vc + (size_t)kh * max_seq * HD;

    for (int i = tid; i < G * HD; i += kAttnThreads) qs[i] = q[(size_t)kh * G * HD + i];
    __syncthreads();
    // scores: one position per thread, q broadcast from smem
    for (int tt = tid; tt < n; tt += kAttnThreads) {
        const KV *kr = kbase + (size_t)(t0 + tt) * HD;
        float acc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) acc[g] = 0.0f;
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            float kv[4];
            load4(kr + d, kv);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float4 qv = *reinterpret_cast<const float4 *>(qs + g * HD + d);
                acc[g] = fmaf(qv.x, kv[0], acc[g]);
                acc[g] = fmaf(qv.y, kv[1], acc[g]);
                acc[g] = fmaf(qv.z, kv[2], acc[g]);
                acc[g] = fmaf(qv.w, kv[3], acc[g]);
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) sc[tt * G + g] = acc[g] * scale;
    }
    __syncthreads();
    // softmax statistics per head (warp g)
    const int lane = tid & 31, warp = tid >> 5;
    if (warp < G) {
        float m = -INFINITY;
        for (int tt = lane; tt < n; tt += 32) m = fmaxf(m, sc[tt * G + warp]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int tt = lane; tt < n; tt += 32) {
            const float p = expf(sc[tt * G + warp] - m);
            sc[tt * G + warp] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) {
            s_m[warp] = m;
            s_l[warp] = l;
        }
    }
    __syncthreads();
    // P.V: thread = (dim group of 4, position subset of 8)
    {
        const int dg = tid % (HD / 4), ts = tid / (HD / 4);
        constexpr int TS = kAttnThreads / (HD / 4);
        float acc[G][4];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[g][j] = 0.0f;
        for (int tt = ts; tt < n; tt += TS) {
            float vv[4];
            load4(vbase + (size_t)(t0 + tt) * HD + dg * 4, vv);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float p = sc[tt * G + g];
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[g][j] = fmaf(p, vv[j], acc[g][j]);
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int j = 0; j < 4; ++j) red[(ts * G + g) * HD + dg * 4 + j] = acc[g][j];
        __syncthreads();
        float *my = part + ((size_t)kh * nsplit + split) * G * (HD + 2);
        for (int i = tid; i < G * HD; i += kAttnThreads) {
            float s = 0.0f;
            for (int r = 0; r < TS; ++r) s += red[r * G * HD + i];
            my[2 * G + i] = s;
        }
        if (tid < G) {
            my[tid] = s_m[tid];
            my[G + tid] = s_l[tid];
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned int t = atomicAdd(&tickets[kh], 1u);
        s_last = (t == (unsigned)nsplit - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // merge the nsplit partials of this KV head.  The per-split (m, l) pairs go to
    // shared memory in one parallel pass (red is free now and holds >= 1024*G floats,
    // nsplit <= 296), each (split, head) weight exp(m_s - M) is computed once, and
    // every output element then sums its nsplit weighted partials with independent
    // loads.  Empty splits (m_s = -inf, o = 0) get weight 0.
    const float *pk = part + (size_t)kh * nsplit * G * (HD + 2);
    const size_t PS = (size_t)G * (HD + 2);
    float *wf = red;                        // [nsplit][G] m_s, then the weights
    float *wl = red + (size_t)nsplit * G;   // [nsplit][G] l_s
    for (int i = tid; i < nsplit * G; i += kAttnThreads) {
        const int s = i / G, g = i - s * G;
        wf[i] = __ldcg(pk + s * PS + g);
        wl[i] = __ldcg(pk + s * PS + G + g);
    }
    __syncthreads();
    if (tid < G) {
        float M = -INFINITY;
        for (int s = 0; s < nsplit; ++s) M = fmaxf(M, wf[s * G + tid]);
        s_m[tid] = M;
    }
    __syncthreads();
    for (int i = tid; i < nsplit * G; i += kAttnThreads) {
        const float ms = wf[i];
        wf[i] = ms == -INFINITY ? 0.0f : expf(ms - s_m[i % G]);
    }
    __syncthreads();
    if (tid < G) {
        float L = 0.0f;
        for (int s = 0; s < nsplit; ++s) L = fmaf(wl[s * G + tid], wf[s * G + tid], L);
        s_l[tid] = L;
    }
    __syncthreads();
    for (int i = tid; i < G * HD; i += kAttnThreads) {
        const int g = i / HD;
        const float *po = pk + 2 * G + i;
        float O = 0.0f;
#pragma unroll 8
        for (int s = 0; s < nsplit; ++s) O = fmaf(__ldcg(po + s * PS), wf[s * G + g], O);
        out[(size_t)kh * G * HD + i] = O / s_l[g];
    }
    if (tid == 0) tickets[kh] = 0u;
}

// Any head_dim / group size: one CTA per query head, scores for every position in
// shared memory, exact max/sum softmax, then P.V with one thread per dimension.
template <typename KV>
__global__ void attn_generic_kernel(const float *__restrict__ q, const KV *__restrict__ kc,
                                    const KV *__restrict__ vc, const int *__restrict__ pos_p,
                                    int seq_len, int max_seq, int n_heads, int n_kv_heads,
                                    int head_dim, float scale, float *__restrict__ out) {
    extern __shared__ float sc[];  // [seq]
    __shared__ float s_red[32];
    const int h = blockIdx.x, tid = threadIdx.x;
    const int kvh = h / (n_heads / n_kv_heads);
    const int seq = pos_p ? (*pos_p + 1) : seq_len;
    const float *qh = q + (size_t)h * head_dim;
    const KV *kb = kc + (size_t)kvh * max_seq * head_dim;
    const KV *vb = vc + (size_t)kvh * max_seq * head_dim;
    auto ld = [](const KV *p, size_t i) -> float {
        if constexpr (sizeof(KV) == 2) return h2f(((const uint16_t *)p)[i]);
        else return ((const float *)p)[i];
    };
    float m = -INFINITY;
    for (int t = tid; t < seq; t += blockDim.x) {
        float a = 0.0f;
        for (int i = 0; i < head_dim; ++i) a = fmaf(qh[i], ld(kb, (size_t)t * head_dim + i), a);
        sc[t] = a * scale;
        m = fmaxf(m, sc[t]);
    }
    const int lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_red[warp] = m;
    __syncthreads();
    m = -INFINITY;
    for (int w = 0; w < nw; ++w) m = fmaxf(m, s_red[w]);
    __syncthreads();
    float l = 0.0f;
    for (int t = tid; t < seq; t += blockDim.x) {
        sc[t] = expf(sc[t] - m);
        l += sc[t];
    }
    l = warp_sum(l);
    if (lane == 0) s_red[warp] = l;
    __syncthreads();
    l = 0.0f;
    for (int w = 0; w < nw; ++w) l += s_red[w];
    for (int d = tid; d < head_dim; d += blockDim.x) {
        float o = 0.0f;
        for (int t = 0; t < seq; ++t) o = fmaf(sc[t], ld(vb, (size_t)t * head_dim + d), o);
        out[(size_t)h * head_dim + d] = o / l;
    }
}

// ------------------------------------------------------------------ swiglu
__global__ void swiglu_kernel(float *__restrict__ g, const float *__restrict__ u, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float gv = g[i];
        const float denom = __fadd_rn(1.0f, expf(-gv));
        g[i] = __fmul_rn(__fdiv_rn(gv, denom), u[i]);
    }
}

__global__ void swiglu_out_kernel(const float *__restrict__ g, const float *__restrict__ u,
                                  float *__restrict__ out, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float gv = g[i];
        out[i] = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), u[i]);
    }
}

// ------------------------------------------------------------------ argmax
// (value, index) pairs compare by value, then lower index wins: the first
// maximum, as argmax_ref's strict '>' scan yields.
__device__ __forceinline__ void better(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

__device__ __forceinline__ void block_argmax(float &bv, int &bi, float *sv, int *si) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        better(bv, bi, ov, oi);
    }
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        bv = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : INT_MAX;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            better(bv, bi, ov, oi);
        }
    }
}

__global__ void argmax_kernel(const float *__restrict__ l, int n, float *__restrict__ pv,
                              int *__restrict__ pi, unsigned int *__restrict__ ticket,
                              int *__restrict__ out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ bool last;
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        better(bv, bi, l[i], i);
    block_argmax(bv, bi, sv, si);
    if (threadIdx.x == 0) {
        pv[blockIdx.x] = bv;
        pi[blockIdx.x] = bi;
        __threadfence();
        last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    bv = -INFINITY;
    bi = INT_MAX;
    for (int b = threadIdx.x; b < gridDim.x; b += blockDim.x) better(bv, bi, __ldcg(pv + b), __ldcg(pi + b));
    __syncthreads();
    block_argmax(bv, bi, sv, si);
    if (threadIdx.x == 0) {
        // every value NaN (or n == 0): argmax_ref returns index 0
        *out = bi == INT_MAX ? 0 : bi;
        *ticket = 0u;
    }
}

// Global greedy token from per-rank (max, index) pairs: largest value, then lowest index.
__global__ void argmax_pairs_kernel(const ArgPair *__restrict__ pairs, int n, int *__restrict__ out,
                                    XWait xw, int *status) {
    xwait(xw, status);  // peer exchange: every rank's pair has landed
    if (threadIdx.x != 0) return;
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int r = 0; r < n; ++r) better(bv, bi, __ldcg(&pairs[r].v), __ldcg(&pairs[r].i));
    *out = bi == INT_MAX ? 0 : bi;
}

// ------------------------------------------------------------------ top-k softmax
// n <= 1024, k <= 64; one CTA.  Selection by (value desc, index asc); the
// softmax over the selected logits runs in double exactly as topk_softmax_ref.
__device__ void topk_softmax_block(const float *__restrict__ logits, int n, int k,
                                   int *__restrict__ idx_out, float *__restrict__ w_out) {
    __shared__ float vals[1024];
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ int sel[64];
    for (int i = threadIdx.x; i < n; i += blockDim.x) vals[i] = logits[i];
    __syncthreads();
    const int kk = min(k, n);
    for (int t = 0; t < kk; ++t) {
        float bv = -INFINITY;
        int bi = INT_MAX;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            bool taken = false;
            for (int j = 0; j < t; ++j) taken |= (sel[j] == i);
            if (!taken) {
                const float v = vals[i];
                if (bi == INT_MAX || v > bv || (v == bv && i < bi)) {
                    bv = v;
                    bi = i;
                }
            }
        }
        block_argmax(bv, bi, sv, si);
        if (threadIdx.x == 0) sel[t] = bi;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        float m = vals[sel[0]];
        for (int i = 1; i < kk; ++i) m = fmaxf(m, vals[sel[i]]);
        float e[64];
        double sum = 0.0;
        for (int i = 0; i < kk; ++i) {
            e[i] = (float)exp((double)vals[sel[i]] - (double)m);
            sum += (double)e[i];
        }
        const double inv = sum > 0.0 ? 1.0 / sum : 0.0;
        for (int i = 0; i < kk; ++i) {
            idx_out[i] = sel[i];
            w_out[i] = (float)((double)e[i] * inv);
        }
        for (int i = kk; i < k; ++i) {
            idx_out[i] = -1;
            w_out[i] = 0.0f;
        }
    }
}

__global__ void topk_softmax_kernel(const float *__restrict__ logits, int n, int k,
                                    int *__restrict__ idx_out, float *__restrict__ w_out) {
    topk_softmax_block(logits, n, k, idx_out, w_out);
}

// ------------------------------------------------------------------ MoE router + combine
// Top-k softmax of n <= 32 * kRouterPer logits by one warp: the k largest (value, then
// lowest index, as topk_softmax_ref's partial_sort on distinct values) by k rounds of a
// warp-wide (value, index) maximum, then softmax over them with exp and the sum in double
// (kernels/topk_softmax/topk_softmax_ref.cpp:41-78).
constexpr int kRouterPer = 32;  // logits per lane (n <= 1024)

__device__ void topk_softmax_warp(const float *__restrict__ logits, int n, int k,
                                  int *__restrict__ idx_out, float *__restrict__ w_out) {
    const int lane = threadIdx.x & 31;
    float v[kRouterPer];
#pragma unroll
    for (int j = 0; j < kRouterPer; ++j) {
        const int i = lane + 32 * j;
        v[j] = i < n ? logits[i] : -INFINITY;
    }
    uint32_t taken = 0;  // bit j: v[j] already chosen
    float sel_v = 0.0f, vmax = 0.0f;
    int sel_i = 0;
    const int kk = min(k, n);
    for (int t = 0; t < kk; ++t) {
        float bv = -INFINITY;
        int bi = INT_MAX;
#pragma unroll
        for (int j = 0; j < kRouterPer; ++j) {
            const int i = lane + 32 * j;
            if (i < n && !((taken >> j) & 1u) && (bi == INT_MAX || v[j] > bv)) {
                bv = v[j];
                bi = i;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        if (t == 0) vmax = bv;
        if (lane == t) {
            sel_v = bv;
            sel_i = bi;
        }
    }
    // lane t < kk holds the t-th choice
    const float e = lane < kk ? (float)exp((double)sel_v - (double)vmax) : 0.0f;
    double sum = (double)e;
    for (int t = 1; t < kk; ++t) sum += __shfl_sync(0xffffffffu, (double)e, t) * (lane == 0);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    if (lane < k) {
        const double inv = sum > 0.0 ? 1.0 / sum : 0.0;
        idx_out[lane] = lane < kk ? sel_i : -1;
        w_out[lane] = lane < kk ? (float)((double)e * inv) : 0.0f;
    }
}

// MoE router of one decode step (runtime/qwen_forward_token.cpp:478-491 with an f32
// router): normed = rmsnorm(h) * post_ln (rmsnorm_ref semantics), logits[e] = W[e] . normed
// in double as matvec_f32_ref (kernels/matvec/matvec_f32_ref.cpp), then, in the last CTA
// to finish, top-k softmax.  One warp per router row, its whole row loaded up front
// (float4, many loads in flight); every CTA normalises the (small) hidden vector itself.
constexpr int kRouterWarps = 4;
constexpr int kRouterHid = 16;  // hidden elements per thread and chunk (H <= 2048 in one)
constexpr int kRouterChunk = 32 * 4 * 16;  // floats of a row one warp loads at once

template <bool STAMP>
__global__ void __launch_bounds__(kRouterWarps * 32) moe_router_kernel(
    const float *__restrict__ h, const float *__restrict__ norm_w, float eps, int H,
    const float *__restrict__ W, int E, int k, float *__restrict__ logits, int *__restrict__ idx,
    float *__restrict__ wts, unsigned int *ticket, Stamp stamp, XWait xw, int *status) {
    extern __shared__ __align__(16) float xn[];  // [H]
    StampRegs stamp_r;
    stamp_enter<STAMP>(stamp, stamp_r);
    __shared__ double s_red[kRouterWarps];
    __shared__ bool s_last;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int e = blockIdx.x * kRouterWarps + warp;
    const float *row = W + (size_t)min(e, E - 1) * H;
    const bool vec = (H % 4 == 0) && (((uintptr_t)W & 15) == 0);
    // the router row does not depend on the previous kernel: its first chunk is loaded
    // before the dependency wait
    float4 wv[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int c = 4 * (lane + 32 * j);
        wv[j] = (vec && c < H) ? *reinterpret_cast<const float4 *>(row + c) : make_float4(0, 0, 0, 0);
    }
    stamp_step<STAMP>(stamp, stamp_r);
    griddep_wait();
    stamp_waited<STAMP>(stamp, stamp_r);
    griddep_launch();
    xwait(xw, status);  // tensor parallelism: the peers' rows of h have landed
    // the hidden vector and the norm weights, every load issued before any is used
    // (a chunk of kRouterHid per thread at a time)
    double ss = 0.0;
    for (int c0 = 0; c0 < H; c0 += kRouterHid * kRouterWarps * 32) {
        float hv[kRouterHid];
#pragma unroll
        for (int j = 0; j < kRouterHid; ++j) {
            const int i = c0 + t + j * kRouterWarps * 32;
            hv[j] = i < H ? h[i] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kRouterHid; ++j) ss += (double)hv[j] * (double)hv[j];
    }
    ss = warp_sum_d(ss);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    double tot = 0.0;
    for (int w = 0; w < kRouterWarps; ++w) tot += s_red[w];
    const float scale = 1.0f / sqrtf(__fadd_rn((float)(tot / H), eps));
    for (int c0 = 0; c0 < H; c0 += kRouterHid * kRouterWarps * 32) {
        float hv[kRouterHid], nv[kRouterHid];
#pragma unroll
        for (int j = 0; j < kRouterHid; ++j) {
            const int i = c0 + t + j * kRouterWarps * 32;
            hv[j] = i < H ? h[i] : 0.0f;
            nv[j] = i < H ? norm_w[i] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kRouterHid; ++j) {
            const int i = c0 + t + j * kRouterWarps * 32;
            if (i < H) xn[i] = __fmul_rn(__fmul_rn(hv[j], scale), nv[j]);
        }
    }
    __syncthreads();
    if (e < E) {
        double acc = 0.0;
        if (vec) {
            for (int c0 = 0; c0 < H; c0 += kRouterChunk) {
                if (c0 > 0) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int c = c0 + 4 * (lane + 32 * j);
                        wv[j] = c < H ? *reinterpret_cast<const float4 *>(row + c) : make_float4(0, 0, 0, 0);
                    }
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int c = c0 + 4 * (lane + 32 * j);
                    if (c < H) {
                        const float4 x4 = *reinterpret_cast<const float4 *>(xn + c);
                        acc += (double)wv[j].x * (double)x4.x;
                        acc += (double)wv[j].y * (double)x4.y;
                        acc += (double)wv[j].z * (double)x4.z;
                        acc += (double)wv[j].w * (double)x4.w;
                    }
                }
            }
        } else {
            for (int i = lane; i < H; i += 32) acc += (double)row[i] * (double)xn[i];
        }
        acc = warp_sum_d(acc);
        if (lane == 0) logits[e] = (float)acc;
    }
    __threadfence();
    __syncthreads();
    if (t == 0) s_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) {
        stamp_exit<STAMP>(stamp, stamp_r);
        return;
    }
    __threadfence();
    if (warp == 0) topk_softmax_warp(logits, E, k, idx, wts);
    if (t == 0) *ticket = 0u;  // ready for the next launch (graph replay)
    stamp_exit<STAMP>(stamp, stamp_r);
}

// acc = sum_t w_t * o_t in router order, then h += acc, with the reference's fp32
// rounding points (runtime/qwen_forward_token.cpp:604-609, :627-631).
template <bool STAMP>
__global__ void moe_combine_kernel(float *__restrict__ h, const float *__restrict__ o,
                                   const float *__restrict__ wts, int k, int H, Stamp stamp,
                                   XWait xw, int *status) {
    StampRegs stamp_r;
    stamp_enter<STAMP>(stamp, stamp_r);
    stamp_step<STAMP>(stamp, stamp_r);
    griddep_wait();
    stamp_waited<STAMP>(stamp, stamp_r);
    griddep_launch();
    xwait(xw, status);  // expert parallelism: every owner's slot rows have landed
    constexpr int kMax = 16;  // expert outputs loaded at once (k is at most 32)
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < H; j += gridDim.x * blockDim.x) {
        float acc = 0.0f;
        const float hj = h[j];
        for (int t0 = 0; t0 < k; t0 += kMax) {
            float ov[kMax], wv[kMax];
#pragma unroll
            for (int u = 0; u < kMax; ++u) {
                const int t = t0 + u;
                ov[u] = t < k ? o[(size_t)t * H + j] : 0.0f;
                wv[u] = t < k ? wts[t] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < kMax; ++u)
                if (t0 + u < k) acc = __fadd_rn(acc, __fmul_rn(wv[u], ov[u]));
        }
        h[j] = __fadd_rn(hj, acc);
    }
    stamp_exit<STAMP>(stamp, stamp_r);
}

// Expert parallelism: the chosen experts as this rank's local indices (-1: another
// rank's expert, e outside [e0, e0 + e_local)), and the expert-output slots zeroed so
// that the cross-rank sum of the slots is each slot's owner's value exactly.
__global__ void moe_ep_local_kernel(const int *__restrict__ idx, int k, int e0, int e_local,
                                    int *__restrict__ local, float *__restrict__ o, int n) {
    griddep_wait();
    griddep_launch();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < k) {
        const int e = idx[i] - e0;
        local[i] = (e >= 0 && e < e_local) ? e : -1;
    }
    if (o)
        for (int j = i; j < n; j += gridDim.x * blockDim.x) o[j] = 0.0f;
}

// ------------------------------------------------------------------ embed
__global__ void embed_kernel(const void *__restrict__ table, int dtype, const int *__restrict__ token,
                             int dim, int group_size, float *__restrict__ out,
                             unsigned int *__restrict__ epoch) {
    // the decode step's epoch for the peer exchanges (launched without PDL: every kernel
    // of the previous step has completed, none of this step's has started)
    if (epoch && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *epoch += 1u;
    const int tok = token[blockIdx.y];  // batched: row blockIdx.y
    out += (size_t)blockIdx.y * dim;
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < dim; c += gridDim.x * blockDim.x) {
        if (dtype == TQB200_DT_F32) {
            out[c] = ((const float *)table)[(size_t)tok * dim + c];
        } else if (dtype == TQB200_DT_F16) {
            out[c] = h2f(((const uint16_t *)table)[(size_t)tok * dim + c]);
        } else {
            const int ng = (dim + group_size - 1) / group_size, GB = 4 + group_size / 2;
            const uint8_t *gp = (const uint8_t *)table + ((size_t)tok * ng + c / group_size) * GB;
            const int i = c % group_size;
            const float s = h2f((uint16_t)(gp[0] | (gp[1] << 8)));
            const float z = h2f((uint16_t)(gp[2] | (gp[3] << 8)));
            const uint8_t b = gp[4 + (i >> 1)];
            out[c] = __fmul_rn(__fsub_rn((float)((i & 1) ? (b >> 4) : (b & 15)), z), s);
        }
    }
}

// ------------------------------------------------------------------ MoE prefill
// Router logits of many tokens (f32 router): logits[t][e] = W[e] . xn[t] with the
// products and the sum in double (matvec_f32_ref, kernels/matvec/matvec_f32_ref.cpp),
// xn already normalised.  On the FP64 tensor cores: a product of two floats is exact in
// double and the m8n8k4 f64 MMA accumulates in double, so only the summation order
// differs from the reference's (relative 1e-16 before the final rounding to float).
// CTA = 16 tokens x 32 experts, K staged through shared memory in chunks of 64, widened
// to double once at staging; warp w owns the 8 x 8 output block (tokens (w & 1) * 8,
// experts (w >> 1) * 8) with two accumulator pairs (even and odd k steps).
constexpr int kRrTok = 16, kRrExp = 32, kRrK = 64;
constexpr int kRrPad = kRrK + 4;  // row stride in doubles: the 8 x 4 fragment loads hit 16 bank pairs

__device__ __forceinline__ void dmma_8x8x4(double (&d)[2], double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};\n"
                 : "+d"(d[0]), "+d"(d[1])
                 : "d"(a), "d"(b));
}

__global__ void __launch_bounds__(256) router_rows_kernel(const float *__restrict__ xn, int n, int H,
                                                          const float *__restrict__ W, int E,
                                                          float *__restrict__ logits) {
    __shared__ double xs[kRrTok][kRrPad];
    __shared__ double ws[kRrExp][kRrPad];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t0 = blockIdx.y * kRrTok, e0 = blockIdx.x * kRrExp;
    const int tb = (warp & 1) * 8, eb = (warp >> 1) * 8;
    const int fr = lane >> 2, fc = lane & 3;  // fragment row (token / expert), k column
    constexpr int RX = kRrTok * kRrK / 256, RW = kRrExp * kRrK / 256;
    float px[RX], pw[RW];  // the next chunk, loaded while this one is consumed
    auto fetch = [&](int k0) {
#pragma unroll
        for (int r = 0; r < RX; ++r) {
            const int i = tid + 256 * r, row = i / kRrK, c = i % kRrK;
            px[r] = (t0 + row < n && k0 + c < H) ? xn[(size_t)(t0 + row) * H + k0 + c] : 0.0f;
        }
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            const int i = tid + 256 * r, row = i / kRrK, c = i % kRrK;
            pw[r] = (e0 + row < E && k0 + c < H) ? W[(size_t)(e0 + row) * H + k0 + c] : 0.0f;
        }
    };
    fetch(0);
    double acc0[2] = {0.0, 0.0}, acc1[2] = {0.0, 0.0};
    for (int k0 = 0; k0 < H; k0 += kRrK) {
        __syncthreads();
#pragma unroll
        for (int r = 0; r < RX; ++r) xs[(tid + 256 * r) / kRrK][(tid + 256 * r) % kRrK] = (double)px[r];
#pragma unroll
        for (int r = 0; r < RW; ++r) ws[(tid + 256 * r) / kRrK][(tid + 256 * r) % kRrK] = (double)pw[r];
        __syncthreads();
        if (k0 + kRrK < H) fetch(k0 + kRrK);
#pragma unroll
        for (int kk = 0; kk < kRrK; kk += 8) {
            dmma_8x8x4(acc0, xs[tb + fr][kk + fc], ws[eb + fr][kk + fc]);
            dmma_8x8x4(acc1, xs[tb + fr][kk + 4 + fc], ws[eb + fr][kk + 4 + fc]);
        }
    }
    // D fragment: row lane >> 2 (token), columns (lane & 3) * 2 + {0, 1} (experts)
    const int t = t0 + tb + fr;
    if (t < n) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int e = e0 + eb + fc * 2 + i;
            if (e < E) logits[(size_t)t * E + e] = (float)(acc0[i] + acc1[i]);
        }
    }
}

// Top-k softmax of every token's router logits: one warp per token.
__global__ void topk_rows_kernel(const float *__restrict__ logits, int n, int E, int k,
                                 int *__restrict__ idx, float *__restrict__ wts) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= n) return;
    topk_softmax_warp(logits + (size_t)t * E, E, k, idx + (size_t)t * k, wts + (size_t)t * k);
}

// h[t] += sum_j wts[t][j] * o[slot[t*k + j]] in router order for every token, with the
// decode combine's rounding points (moe_combine_kernel).
__global__ void moe_combine_rows_kernel(float *__restrict__ h, const float *__restrict__ o,
                                        const float *__restrict__ wts, const int *__restrict__ slot,
                                        int k, int H) {
    const int t = blockIdx.y;
    constexpr int kMax = 16;
    for (int jx = blockIdx.x * blockDim.x + threadIdx.x; jx < H; jx += gridDim.x * blockDim.x) {
        float acc = 0.0f;
        const float hj = h[(size_t)t * H + jx];
        for (int u0 = 0; u0 < k; u0 += kMax) {
            float ov[kMax], wv[kMax];
#pragma unroll
            for (int u = 0; u < kMax; ++u) {
                const int a = u0 + u;
                ov[u] = a < k ? o[(size_t)slot[(size_t)t * k + a] * H + jx] : 0.0f;
                wv[u] = a < k ? wts[(size_t)t * k + a] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < kMax; ++u)
                if (u0 + u < k) acc = __fadd_rn(acc, __fmul_rn(wv[u], ov[u]));
        }
        h[(size_t)t * H + jx] = __fadd_rn(hj, acc);
    }
}

template <typename KV, int HD, int G>
int launch_attn_t(const AttnArgs &a, cudaStream_t st) {
    const size_t smem = (size_t)(G * HD + (kAttnThreads / (HD / 4)) * G * HD) * 4 +
                        (size_t)a.chunk_max * G * 4;
    auto k = attn_split_kernel<KV, HD, G>;
    if (smem > 48 * 1024) {
        TQ_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    }
    dim3 grid(a.n_kv_heads, a.nsplit);
    k<<<grid, kAttnThreads, smem, st>>>(a.q, (const KV *)a.k, (const KV *)a.v, a.pos, a.seq_len,
                                        a.max_seq, a.nsplit, a.scale, a.partial, a.tickets, a.out);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

template <typename KV>
int launch_attn_kv(const AttnArgs &a, cudaStream_t st) {
    const int G = a.n_heads / a.n_kv_heads;
#define TQ_ATTN_CASE(HDV, GV) \
    if (a.head_dim == HDV && G == GV) return launch_attn_t<KV, HDV, GV>(a, st);
    TQ_ATTN_CASE(64, 1) TQ_ATTN_CASE(64, 2) TQ_ATTN_CASE(64, 4) TQ_ATTN_CASE(64, 7)
    TQ_ATTN_CASE(64, 8) TQ_ATTN_CASE(128, 1) TQ_ATTN_CASE(128, 2) TQ_ATTN_CASE(128, 4)
    TQ_ATTN_CASE(128, 8) TQ_ATTN_CASE(32, 1) TQ_ATTN_CASE(32, 2) TQ_ATTN_CASE(32, 4)
    TQ_ATTN_CASE(32, 8)
#undef TQ_ATTN_CASE
    // other shapes: the generic one-CTA-per-head kernel (no scratch, any head_dim)
    const size_t smem = (size_t)a.max_seq * 4;
    TQ_CHECK_ARG(smem <= 200 * 1024, "attention: max_seq %d too long for the generic kernel",
                 a.max_seq);
    auto k = attn_generic_kernel<KV>;
    if (smem > 48 * 1024)
        TQ_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k<<<a.n_heads, 128, smem, st>>>(a.q, (const KV *)a.k, (const KV *)a.v, a.pos, a.seq_len,
                                    a.max_seq, a.n_heads, a.n_kv_heads, a.head_dim, a.scale, a.out);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

}  // namespace

// ------------------------------------------------------------------ launchers
int launch_rmsnorm(const float *x, const float *w, float *y, int rows, int n, float eps,
                   cudaStream_t st) {
    TQ_CHECK_ARG(n > 0 && rows > 0, "rmsnorm n %d rows %d", n, rows);
    const bool a16 = (((uintptr_t)x | (uintptr_t)w | (uintptr_t)y) & 15u) == 0;
    if (a16 && n % 4 == 0 && n <= 4 * kRmsV * 256)
        rmsnorm_rows_v4_kernel<<<rows, 256, 0, st>>>(x, w, y, n, eps);
    else
        rmsnorm_rows_kernel<<<rows, 256, 0, st>>>(x, w, y, n, eps);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

void rope_row(float theta, int head_dim, int pos, float *cs, float *sn) {
    // kernels/rope/rope_ref.cpp:74-85, same float operations and libm calls
    for (int i = 0; i < head_dim / 2; ++i) {
        const float exponent = -(float)(2 * i) / (float)head_dim;
        const float inv_freq = powf(theta, exponent);
        volatile float angle = (float)pos * inv_freq;
        cs[i] = cosf(angle);
        sn[i] = sinf(angle);
    }
}

int launch_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim, const float *cs,
                const float *sn, cudaStream_t st) {
    TQ_CHECK_ARG(head_dim > 0 && head_dim % 2 == 0 && head_dim / 2 <= 256,
                 "rope: unsupported head_dim %d", head_dim);
    if (n_heads + n_kv_heads == 0) return TQB200_OK;
    rope_kernel<<<n_heads + n_kv_heads, 128, 0, st>>>(q, k, n_heads, n_kv_heads, head_dim, cs, sn);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_qk_rope_kv(const QkRopeKvArgs &a, cudaStream_t st) {
    TQ_CHECK_ARG(a.head_dim <= 512 && a.head_dim % 2 == 0 && a.head_dim / 2 <= 4 * 128,
                 "head_dim %d", a.head_dim);
    TQ_CHECK_ARG(a.n_tokens >= 1 && a.n_tokens <= 65535, "qk_rope_kv: %d tokens", a.n_tokens);
    const int nh = a.n_heads + 2 * a.n_kv_heads;
    if (a.head_dim / 2 <= 32 * kQrMaxE) {
        const dim3 grid((nh + kQrWarps - 1) / kQrWarps, a.n_tokens);
        if (a.kv_fp16)
            qk_rope_kv_warp_kernel<uint16_t><<<grid, kQrWarps * 32, 0, st>>>(
                a.q, a.k, a.v, a.q_norm, a.k_norm, a.eps, a.cos_tab, a.sin_tab, a.pos,
                (uint16_t *)a.kcache, (uint16_t *)a.vcache, a.n_heads, a.n_kv_heads, a.head_dim,
                a.max_seq);
        else
            qk_rope_kv_warp_kernel<float><<<grid, kQrWarps * 32, 0, st>>>(
                a.q, a.k, a.v, a.q_norm, a.k_norm, a.eps, a.cos_tab, a.sin_tab, a.pos,
                (float *)a.kcache, (float *)a.vcache, a.n_heads, a.n_kv_heads, a.head_dim,
                a.max_seq);
        TQ_CUDA_TRY(cudaGetLastError());
        return TQB200_OK;
    }
    const dim3 blocks(nh, a.n_tokens);
    if (a.kv_fp16)
        qk_rope_kv_kernel<uint16_t><<<blocks, 128, 0, st>>>(
            a.q, a.k, a.v, a.q_norm, a.k_norm, a.eps, a.cos_tab, a.sin_tab, a.pos,
            (uint16_t *)a.kcache, (uint16_t *)a.vcache, a.n_heads, a.n_kv_heads, a.head_dim,
            a.max_seq);
    else
        qk_rope_kv_kernel<float><<<blocks, 128, 0, st>>>(
            a.q, a.k, a.v, a.q_norm, a.k_norm, a.eps, a.cos_tab, a.sin_tab, a.pos,
            (float *)a.kcache, (float *)a.vcache, a.n_heads, a.n_kv_heads, a.head_dim, a.max_seq);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int attn_plan(int n_kv_heads, int max_seq, int *nsplit, int *chunk_max) {
    // aim for >= 2 CTAs per SM at full context, chunks of at least 32 positions
    const int target = 2 * num_sms();
    int ns = std::max(1, (target + n_kv_heads - 1) / n_kv_heads);
    ns = std::min(ns, std::max(1, (max_seq + 31) / 32));
    *nsplit = ns;
    *chunk_max = (max_seq + ns - 1) / ns;
    return TQB200_OK;
}

size_t attn_partial_floats(int n_heads, int head_dim, int nsplit) {
    return (size_t)nsplit * (n_heads * head_dim + 2 * n_heads);
}

int launch_attention(const AttnArgs &a, cudaStream_t st) {
    TQ_CHECK_ARG(a.n_kv_heads > 0 && a.n_heads % a.n_kv_heads == 0, "heads %d / kv %d",
                 a.n_heads, a.n_kv_heads);
    TQ_CHECK_ARG(!a.k_new || (a.pos && a.v_new && a.cos_tab && a.sin_tab), "fused attention args");
    const int rc = launch_attention_tma(a, st);
    if (rc != TQB200_ERR_UNSUPPORTED) return rc;
    TQ_CHECK_ARG(!a.put, "peer exchange needs the TMA attention kernel (head_dim %d, group %d)",
                 a.head_dim, a.n_heads / a.n_kv_heads);
    // no TMA shape: the split kernel (global partials), after the per-head
    // QK-norm / RoPE / KV-append kernel in fused mode
    TQ_CHECK_ARG(a.chunk_max >= (a.max_seq + a.nsplit - 1) / a.nsplit, "chunk plan");
    if (a.k_new) {
        QkRopeKvArgs r{};
        r.q = const_cast<float *>(a.q);
        r.k = a.k_new;
        r.v = a.v_new;
        r.q_norm = a.q_norm;
        r.k_norm = a.k_norm;
        r.eps = a.eps;
        r.cos_tab = a.cos_tab;
        r.sin_tab = a.sin_tab;
        r.pos = a.pos;
        r.kcache = const_cast<void *>(a.k);
        r.vcache = const_cast<void *>(a.v);
        r.kv_fp16 = a.kv_fp16;
        r.n_heads = a.n_heads;
        r.n_kv_heads = a.n_kv_heads;
        r.head_dim = a.head_dim;
        r.max_seq = a.max_seq;
        const int rr = launch_qk_rope_kv(r, st);
        if (rr != TQB200_OK) return rr;
    }
    return a.kv_fp16 ? launch_attn_kv<uint16_t>(a, st) : launch_attn_kv<float>(a, st);
}

int launch_attention_split(const AttnArgs &a, cudaStream_t st) {
    TQ_CHECK_ARG(a.n_kv_heads > 0 && a.n_heads % a.n_kv_heads == 0 && !a.k_new,
                 "split attention: heads %d / kv %d (plain mode only)", a.n_heads, a.n_kv_heads);
    TQ_CHECK_ARG(a.chunk_max >= (a.max_seq + a.nsplit - 1) / a.nsplit, "chunk plan");
    return a.kv_fp16 ? launch_attn_kv<uint16_t>(a, st) : launch_attn_kv<float>(a, st);
}

int launch_swiglu(float *g, const float *u, int n, cudaStream_t st) {
    if (n == 0) return TQB200_OK;
    const int block = 256;
    const int grid = std::min((n + block - 1) / block, num_sms() * 8);
    swiglu_kernel<<<grid, block, 0, st>>>(g, u, n);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_swiglu_out(const float *g, const float *u, float *out, int n, cudaStream_t st) {
    if (n == 0) return TQB200_OK;
    const int block = 256;
    const int grid = std::min((n + block - 1) / block, num_sms() * 8);
    swiglu_out_kernel<<<grid, block, 0, st>>>(g, u, out, n);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_argmax_pairs(const ArgPair *pairs, int n, int *out, cudaStream_t st, const XWait &xw,
                        int *status) {
    argmax_pairs_kernel<<<1, 32, 0, st>>>(pairs, n, out, xw, status);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int argmax_blocks(int n) { return std::max(1, std::min((n + 1023) / 1024, 2 * num_sms())); }

int launch_argmax(const float *l, int n, float *pv, int *pi, unsigned int *ticket, int *out,
                  cudaStream_t st) {
    TQ_CHECK_ARG(n > 0, "argmax n %d", n);
    argmax_kernel<<<argmax_blocks(n), 256, 0, st>>>(l, n, pv, pi, ticket, out);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

template <typename Kern, typename... Args>
int launch_pdl(Kern k, int grid, int block, size_t smem, bool pdl, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, k, args...));
    return TQB200_OK;
}

int launch_moe_router(const float *h, const float *norm_w, float eps, int H, const float *W, int E,
                      int k, float *logits, int *idx, float *wts, unsigned int *ticket, bool pdl,
                      cudaStream_t st, const Stamp &stamp, const XWait &xw, int *status) {
    TQ_CHECK_ARG(E > 0 && E <= 32 * kRouterPer && k > 0 && k <= 32 && k <= E && H > 0,
                 "moe router: E %d k %d H %d", E, k, H);
    const size_t smem = (size_t)H * 4;
    TQ_CHECK_ARG(smem <= 48 * 1024, "moe router: hidden %d too large", H);
    return launch_pdl(stamp.base ? moe_router_kernel<true> : moe_router_kernel<false>,
                      (E + kRouterWarps - 1) / kRouterWarps, kRouterWarps * 32, smem, pdl, st, h,
                      norm_w, eps, H, W, E, k, logits, idx, wts, ticket, stamp, xw, status);
}

int launch_moe_combine(float *h, const float *o, const float *wts, int k, int H, bool pdl,
                       cudaStream_t st, const Stamp &stamp, const XWait &xw, int *status) {
    TQ_CHECK_ARG(k > 0 && H > 0, "moe combine: k %d H %d", k, H);
    const int threads = 256;
    return launch_pdl(stamp.base ? moe_combine_kernel<true> : moe_combine_kernel<false>,
                      (H + threads - 1) / threads, threads, 0, pdl, st, h, o, wts, k, H, stamp, xw,
                      status);
}

int launch_topk_softmax(const float *logits, int n, int k, int *idx, float *w, cudaStream_t st) {
    TQ_CHECK_ARG(n > 0 && n <= 1024 && k > 0 && k <= 64, "topk n %d k %d", n, k);
    topk_softmax_kernel<<<1, 256, 0, st>>>(logits, n, k, idx, w);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_router_rows(const float *xn, int n, int H, const float *W, int E, float *logits,
                       cudaStream_t st) {
    TQ_CHECK_ARG(n > 0 && n <= 65535 * kRrTok && E > 0 && H > 0, "router rows: n %d E %d H %d", n, E, H);
    const dim3 grid((E + kRrExp - 1) / kRrExp, (n + kRrTok - 1) / kRrTok);
    router_rows_kernel<<<grid, 256, 0, st>>>(xn, n, H, W, E, logits);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_topk_rows(const float *logits, int n, int E, int k, int *idx, float *wts, cudaStream_t st) {
    TQ_CHECK_ARG(n > 0 && E > 0 && E <= 32 * kRouterPer && k > 0 && k <= 32 && k <= E,
                 "topk rows: n %d E %d k %d", n, E, k);
    topk_rows_kernel<<<(n + 3) / 4, 128, 0, st>>>(logits, n, E, k, idx, wts);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_moe_combine_rows(float *h, const float *o, const float *wts, const int *slot, int n,
                            int k, int H, cudaStream_t st) {
    TQ_CHECK_ARG(n > 0 && n <= 65535 && k > 0 && H > 0, "moe combine rows: n %d k %d H %d", n, k, H);
    const dim3 grid((H + 255) / 256, n);
    moe_combine_rows_kernel<<<grid, 256, 0, st>>>(h, o, wts, slot, k, H);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_moe_ep_local(const int *idx, int k, int e0, int e_local, int *local, float *o, int H,
                        bool pdl, cudaStream_t st) {
    TQ_CHECK_ARG(k > 0 && k <= 1024 && H > 0 && e_local > 0, "moe ep: k %d H %d", k, H);
    const int n = o ? k * H : k, threads = 256;
    const int grid = std::max(1, std::min((n + threads - 1) / threads, 64));
    return launch_pdl(moe_ep_local_kernel, grid, threads, 0, pdl, st, idx, k, e0, e_local, local, o, n);
}

int launch_embed(const void *table, int dtype, const int *token, int dim, int group_size,
                 float *out, cudaStream_t st, int n_tokens, unsigned int *epoch) {
    TQ_CHECK_ARG(n_tokens >= 1 && n_tokens <= 65535, "embed: %d tokens", n_tokens);
    const dim3 grid(std::max(1, std::min((dim + 255) / 256, 16)), n_tokens);
    embed_kernel<<<grid, 256, 0, st>>>(table, dtype, token, dim, group_size, out, epoch);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

}  // namespace tqb200
