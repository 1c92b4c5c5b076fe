// gptq_matvec.cu — GPTQ-INT4 matvec / matmul and dense f32 / f16 matvec, sm_100a.
//
// GPTQ (reference: kernels/matvec/matvec_gptq_ref.cpp:52-96, matmul_gptq_ref.cpp; tensor
// layout runtime/tiny_format.h:140-182): the weight blob is
//   [u32 magic][u32 flags][scales fp16 [n_groups][out]][qzeros fp16 [n_groups][out]]
//   [g_idx u32 [in] when flags & 1][qweight u32 [in/8][out]]
// with qweight column-major: word (c8, o) holds columns 8 c8 .. 8 c8 + 7 of row o, column
// 8 c8 + k in bits 4k .. 4k + 3, and w = (q - z[g]) * s[g], g = g_idx[c] or c / G.
//   * Thread o owns output row o: the words of consecutive rows are consecutive, so every
//     weight load of a warp is one 128-byte line (the layout is made for it).
//   * Without g_idx a group's dot is s (sum_k q_k x_k - z X_g), X_g the group's sum of x
//     (computed once per CTA), in fp32 within the group and across groups; with g_idx
//     (act-order) every column dequantises on its own, (q - z[g]) * s[g], scales and
//     zeros of the CTA's rows staged in shared memory.
//   * The reference accumulates in double; fp32 stays inside the 1e-4 max-relative bound.
// matmul_gptq (MatmulGPTQFn, kernels/dispatch.h:258): the same kernel per column of X
// (blockIdx.y), X and Y column-major.
//
// Dense matvec_f32_ref / matvec_f16_ref (kernels/matvec/matvec_f32_ref.cpp:41,
// matvec_f16_ref.cpp): a warp per row, 16-byte loads, double accumulation as the
// reference.  These serve the per-op backend's f32 / f16 tensors (a MoE router, f16
// models); the quantised decode path does not use them.
#include "common.cuh"
#include "kernels.h"

namespace tqb200 {
namespace {

constexpr int kGptqThreads = 128;

__device__ __forceinline__ uint32_t ldg_u32_nc(const uint8_t *p) {
    return __ldg(reinterpret_cast<const unsigned int *>(p));
}
__device__ __forceinline__ float ld_f16(const uint8_t *p) {
    return h2f(__ldg(reinterpret_cast<const unsigned short *>(p)));
}

// x of column blockIdx.y in shared memory, followed (no g_idx) by the group sums X_g.
__global__ void __launch_bounds__(kGptqThreads) gptq_matvec_kernel(
    const uint8_t *__restrict__ w, const float *__restrict__ x, float *__restrict__ y, int out,
    int in, int G, int ldx, int ldy) {
    extern __shared__ float s_x[];  // [in] x, then [ng] X_g or [ng][blockDim] s, z
    x += (size_t)blockIdx.y * ldx;
    y += (size_t)blockIdx.y * ldy;
    const uint32_t flags = __ldg(reinterpret_cast<const unsigned int *>(w) + 1);
    const bool gidx = (flags & 1u) != 0;
    const int ng = in / G;
    const size_t sq = (size_t)ng * out * 2;
    const uint8_t *scales = w + 8, *qzeros = scales + sq;
    const uint8_t *g_idx = gidx ? qzeros + sq : nullptr;
    const uint8_t *qw = gidx ? g_idx + (size_t)in * 4 : qzeros + sq;
    for (int i = threadIdx.x; i < in; i += blockDim.x) s_x[i] = x[i];
    float *s_aux = s_x + in;
    const int o = blockIdx.x * blockDim.x + threadIdx.x;
    if (!gidx) {
        __syncthreads();
        for (int g = threadIdx.x; g < ng; g += blockDim.x) {
            float X = 0.0f;
            for (int c = g * G; c < (g + 1) * G; ++c) X += s_x[c];
            s_aux[g] = X;
        }
        __syncthreads();
        if (o >= out) return;
        float acc = 0.0f;
        for (int g = 0; g < ng; ++g) {
            const float s = ld_f16(scales + ((size_t)g * out + o) * 2);
            const float z = ld_f16(qzeros + ((size_t)g * out + o) * 2);
            float a0 = 0.0f, a1 = 0.0f;
            for (int c8 = g * G / 8; c8 < (g + 1) * G / 8; ++c8) {
                const uint32_t wd = ldg_u32_nc(qw + ((size_t)c8 * out + o) * 4);
                const float *xc = s_x + 8 * c8;
#pragma unroll
                for (int kk = 0; kk < 8; kk += 2) {
                    a0 = fmaf((float)((wd >> (4 * kk)) & 15u), xc[kk], a0);
                    a1 = fmaf((float)((wd >> (4 * kk + 4)) & 15u), xc[kk + 1], a1);
                }
            }
            acc = fmaf(s, fmaf(-z, s_aux[g], a0 + a1), acc);
        }
        y[o] = acc;
        return;
    }
    // act-order: this CTA's rows' scales and zeros per group in shared memory
    float *s_s = s_aux, *s_z = s_aux + (size_t)ng * blockDim.x;
    for (int g = 0; g < ng; ++g)
        if (o < out) {
            s_s[g * blockDim.x + threadIdx.x] = ld_f16(scales + ((size_t)g * out + o) * 2);
            s_z[g * blockDim.x + threadIdx.x] = ld_f16(qzeros + ((size_t)g * out + o) * 2);
        }
    __syncthreads();
    if (o >= out) return;
    const unsigned int *gi = reinterpret_cast<const unsigned int *>(g_idx);
    float acc = 0.0f;
    for (int c8 = 0; c8 < in / 8; ++c8) {
        const uint32_t wd = ldg_u32_nc(qw + ((size_t)c8 * out + o) * 4);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const int c = 8 * c8 + kk;
            const int g = min((int)__ldg(gi + c), ng - 1);
            const float s = s_s[g * blockDim.x + threadIdx.x], z = s_z[g * blockDim.x + threadIdx.x];
            acc = fmaf(__fmul_rn(__fsub_rn((float)((wd >> (4 * kk)) & 15u), z), s), s_x[c], acc);
        }
    }
    y[o] = acc;
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
    const size_t smem = ((size_t)in + (g_idx ? 2 * (size_t)ng * kGptqThreads : (size_t)ng)) * 4;
    static KernelSmem attr;
    int smem_max = 0;
    TQ_CUDA_TRY(smem_limit_once(gptq_matvec_kernel, attr, &smem_max));
    TQ_CHECK_ARG(smem <= (size_t)smem_max, "gptq: in_dim %d / %d groups need too much shared memory",
                 in, ng);
    const dim3 grid((out + kGptqThreads - 1) / kGptqThreads, n);
    gptq_matvec_kernel<<<grid, kGptqThreads, smem, st>>>(w, x, y, out, in, G, in, out);
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
