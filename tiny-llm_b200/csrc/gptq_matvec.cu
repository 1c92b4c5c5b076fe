// gptq_matvec.cu — GPTQ-INT4 matvec / matmul and dense f32 / f16 matvec, sm_100a.
//
// GPTQ (reference: kernels/matvec/matvec_gptq_ref.cpp:52-96, matmul_gptq_ref.cpp; tensor
// layout runtime/tiny_format.h:140-182): the weight blob is
//   [u32 magic][u32 flags][scales fp16 [n_groups][out]][qzeros fp16 [n_groups][out]]
//   [g_idx u32 [in] when flags & 1][qweight u32 [in/8][out]]
// with qweight column-major: word (c8, o) holds columns 8 c8 .. 8 c8 + 7 of row o, column
// 8 c8 + k in bits 4k .. 4k + 3, and w = (q - z[g]) * s[g], g = g_idx[c] or c / G.
//   * A CTA is 32 rows x 8 slices of the in / 8 weight words: lane = row, warp = slice,
//     so every weight load of a warp is one 128-byte line (the layout is made for it) and
//     a small matrix still spreads over the SMs (4864 rows: 152 CTAs).  The slices'
//     partial sums are added in slice order at the end (deterministic).
//   * Without g_idx a slice accumulates per run of words in one group s (sum_k q_k x_k -
//     z X), X the run's sum of x (8-column sums precomputed per CTA), in fp32; with g_idx
//     (act-order) every column dequantises on its own, (q - z[g]) * s[g], the CTA rows'
//     scales and zeros staged in shared memory.
//   * The reference accumulates in double; fp32 stays inside the 1e-4 max-relative bound.
// matmul_gptq (MatmulGPTQFn, kernels/dispatch.h:258): the same kernel per column of X
// (blockIdx.y), X and Y column-major.
//
// Dense matvec_f32_ref / matvec_f16_ref (kernels/matvec/matvec_f32_ref.cpp:41,
// matvec_f16_ref.cpp): a warp per row, coalesced loads, double accumulation as the
// reference.  These serve the per-op backend's f32 / f16 tensors (a MoE router, f16
// models); the quantised decode path does not use them.
#include "common.cuh"
#include "kernels.h"

namespace tqb200 {
namespace {

constexpr int kGqRows = 32;    // rows per CTA (a lane per row)
constexpr int kGqSlices = 8;   // warps per CTA, each over one slice of the weight words
constexpr int kGqThreads = kGqRows * kGqSlices;

__device__ __forceinline__ uint32_t ldg_u32_nc(const uint8_t *p) {
    return __ldg(reinterpret_cast<const unsigned int *>(p));
}
__device__ __forceinline__ float ld_f16(const uint8_t *p) {
    return h2f(__ldg(reinterpret_cast<const unsigned short *>(p)));
}

// dot of one weight word's 8 codes with x[8 c8 .. 8 c8 + 7] (two chains)
__device__ __forceinline__ void word_dot(uint32_t wd, const float *xc, float &a0, float &a1) {
    const float4 xa = reinterpret_cast<const float4 *>(xc)[0];
    const float4 xb = reinterpret_cast<const float4 *>(xc)[1];
    a0 = fmaf((float)(wd & 15u), xa.x, a0);
    a1 = fmaf((float)((wd >> 4) & 15u), xa.y, a1);
    a0 = fmaf((float)((wd >> 8) & 15u), xa.z, a0);
    a1 = fmaf((float)((wd >> 12) & 15u), xa.w, a1);
    a0 = fmaf((float)((wd >> 16) & 15u), xb.x, a0);
    a1 = fmaf((float)((wd >> 20) & 15u), xb.y, a1);
    a0 = fmaf((float)((wd >> 24) & 15u), xb.z, a0);
    a1 = fmaf((float)(wd >> 28), xb.w, a1);
}

// Shared memory: x [in]; then the 8-column sums [in / 8] (no g_idx) or the CTA rows'
// scales and zeros [2][ng][32] (g_idx); then the slices' partials [8][32].
__global__ void __launch_bounds__(kGqThreads) gptq_matvec_kernel(
    const uint8_t *__restrict__ w, const float *__restrict__ x, float *__restrict__ y, int out,
    int in, int G, int ldx, int ldy) {
    extern __shared__ __align__(16) float s_x[];
    x += (size_t)blockIdx.y * ldx;
    y += (size_t)blockIdx.y * ldy;
    const uint32_t flags = __ldg(reinterpret_cast<const unsigned int *>(w) + 1);
    const bool gidx = (flags & 1u) != 0;
    const int ng = in / G, W = in / 8;
    const size_t sq = (size_t)ng * out * 2;
    const uint8_t *scales = w + 8, *qzeros = scales + sq;
    const uint8_t *g_idx = gidx ? qzeros + sq : nullptr;
    const uint8_t *qw = gidx ? g_idx + (size_t)in * 4 : qzeros + sq;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row0 = blockIdx.x * kGqRows, o = row0 + lane;
    for (int i = threadIdx.x; i < in; i += kGqThreads) s_x[i] = x[i];
    float *s_aux = s_x + in;
    float *s_part = s_aux + (gidx ? 2 * (size_t)ng * kGqRows : (size_t)W);
    if (!gidx) {
        __syncthreads();
        for (int c8 = threadIdx.x; c8 < W; c8 += kGqThreads) {
            float X = 0.0f;
#pragma unroll
            for (int k = 0; k < 8; ++k) X += s_x[8 * c8 + k];
            s_aux[c8] = X;
        }
    } else {
        for (int i = threadIdx.x; i < ng * kGqRows; i += kGqThreads) {
            const int g = i / kGqRows, row = row0 + i % kGqRows;
            if (row < out) {
                s_aux[i] = ld_f16(scales + ((size_t)g * out + row) * 2);
                s_aux[(size_t)ng * kGqRows + i] = ld_f16(qzeros + ((size_t)g * out + row) * 2);
            }
        }
    }
    __syncthreads();
    const int wb = (int)((long long)W * warp / kGqSlices);
    const int we = (int)((long long)W * (warp + 1) / kGqSlices);
    float acc = 0.0f;
    if (o < out) {
        const uint8_t *qo = qw + (size_t)o * 4;
        const size_t wstride = (size_t)out * 4;
        if (!gidx) {
            const int wpg = G / 8;
            for (int c8 = wb; c8 < we;) {
                const int g = c8 / wpg;
                const int ge = min(we, (g + 1) * wpg);
                const float sc = ld_f16(scales + ((size_t)g * out + o) * 2);
                const float z = ld_f16(qzeros + ((size_t)g * out + o) * 2);
                float a0 = 0.0f, a1 = 0.0f, X = 0.0f;
                for (; c8 + 4 <= ge; c8 += 4) {  // four independent loads in flight
                    uint32_t wd[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) wd[u] = ldg_u32_nc(qo + (size_t)(c8 + u) * wstride);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        word_dot(wd[u], s_x + 8 * (c8 + u), a0, a1);
                        X += s_aux[c8 + u];
                    }
                }
                for (; c8 < ge; ++c8) {
                    word_dot(ldg_u32_nc(qo + (size_t)c8 * wstride), s_x + 8 * c8, a0, a1);
                    X += s_aux[c8];
                }
                acc = fmaf(sc, fmaf(-z, X, a0 + a1), acc);
            }
        } else {
            const unsigned int *gi = reinterpret_cast<const unsigned int *>(g_idx);
            const float *s_s = s_aux + lane, *s_z = s_aux + (size_t)ng * kGqRows + lane;
            for (int c8 = wb; c8 < we; ++c8) {
                const uint32_t wd = ldg_u32_nc(qo + (size_t)c8 * wstride);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const int c = 8 * c8 + kk;
                    const int g = min((int)__ldg(gi + c), ng - 1);
                    const float sc = s_s[g * kGqRows], z = s_z[g * kGqRows];
                    acc = fmaf(__fmul_rn(__fsub_rn((float)((wd >> (4 * kk)) & 15u), z), sc), s_x[c],
                               acc);
                }
            }
        }
    }
    s_part[warp * kGqRows + lane] = acc;
    __syncthreads();
    if (warp == 0 && o < out) {
        float v = 0.0f;
#pragma unroll
        for (int sl = 0; sl < kGqSlices; ++sl) v += s_part[sl * kGqRows + lane];
        y[o] = v;
    }
}

// Dense matvec, a warp per row, double accumulation (matvec_f32_ref / matvec_f16_ref).
template <typename T>
__global__ void dense_matvec_kernel(const T *__restrict__ w, const float *__restrict__ x,
                                    float *__restrict__ y, int out, int in) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= out) return;
    const T *r = w + (size_t)row * in;
    double acc = 0.0;
    for (int i = lane; i < in; i += 32) {
        float wv;
        if constexpr (sizeof(T) == 2) wv = h2f(r[i]);
        else wv = r[i];
        acc += (double)wv * (double)x[i];
    }
    acc = warp_sum_d(acc);
    if (lane == 0) y[row] = (float)acc;
}

}  // namespace

size_t gptq_bytes(int out, int in, int G, bool g_idx) {
    const size_t ng = (size_t)(in / G);
    return 8 + 2 * ng * out * 2 + (g_idx ? (size_t)in * 4 : 0) + (size_t)(in / 8) * out * 4;
}

int launch_gptq_matmul(const uint8_t *w, bool g_idx, const float *x, float *y, int out, int in,
                       int n, int G, cudaStream_t st) {
    TQ_CHECK_ARG(out > 0 && in > 0 && n > 0 && n <= 65535 && G > 0 && in % G == 0 && G % 8 == 0,
                 "gptq: bad shape %d x %d, %d columns, group %d (in %% G == 0, G %% 8 == 0)", out,
                 in, n, G);
    const int ng = in / G;
    const size_t smem = ((size_t)in + (g_idx ? 2 * (size_t)ng * kGqRows : (size_t)(in / 8)) +
                         (size_t)kGqSlices * kGqRows) * 4;
    static KernelSmem attr;
    int smem_max = 0;
    TQ_CUDA_TRY(smem_limit_once(gptq_matvec_kernel, attr, &smem_max));
    TQ_CHECK_ARG(smem <= (size_t)smem_max, "gptq: in_dim %d / %d groups need too much shared memory",
                 in, ng);
    const dim3 grid((out + kGqRows - 1) / kGqRows, n);
    gptq_matvec_kernel<<<grid, kGqThreads, smem, st>>>(w, x, y, out, in, G, in, out);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_dense_matvec(const void *w, bool f16, const float *x, float *y, int out, int in,
                        cudaStream_t st) {
    TQ_CHECK_ARG(out >= 0 && in > 0, "dense matvec: bad shape %d x %d", out, in);
    if (out == 0) return TQB200_OK;
    const int rows_per_cta = 8;
    const int grid = (out + rows_per_cta - 1) / rows_per_cta;
    if (f16)
        dense_matvec_kernel<uint16_t><<<grid, 32 * rows_per_cta, 0, st>>>((const uint16_t *)w, x, y,
                                                                         out, in);
    else
        dense_matvec_kernel<float><<<grid, 32 * rows_per_cta, 0, st>>>((const float *)w, x, y, out,
                                                                      in);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

}  // namespace tqb200
