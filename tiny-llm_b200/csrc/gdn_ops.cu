// gdn_ops.cu — the Gated DeltaNet (Qwen3.5 linear-attention) decode ops and partial RoPE,
// sm_100a.
//
// Reference semantics (kernels/gdn/gdn_ops_ref.cpp):
//   l2norm_inplace_ref      :44-57   x *= 1 / sqrtf((float)sum(double x^2) + eps)
//   causal_conv1d_update_ref:82-105  per channel: acc = sum_i w_i st_i + w_last x (fp32, in
//                                     order); out = silu(acc); the state shifts left and
//                                     takes x
//   gdn_step_ref            :134-176 S = decay * S; kv = S^T k; delta = beta (v - kv);
//                                     S += k delta^T; o = S^T q (double sum), per head
//   rmsnorm_gated_ref       :203-218 y = ((x * scale) * w) * silu(gate)
//   partial_rope_ref        :233-277 rotate-half RoPE over the first rotary_dim dimensions
//
// Every step keeps the reference's fp32 rounding points (__fmul_rn / __fadd_rn: no FMA
// contraction) and summation order where the reference sums in fp32, so the results are
// bit-exact except where a libm function enters: the SiLU's expf (CUDA's expf, within a
// few ulp of the host's), and the double sums' association in l2norm / rmsnorm_gated
// (summed in a tree here; the double result rounds to the same float except in rare
// ties).  gdn_step's decay = exp(g) is computed on the host with the host libm (the
// launcher takes the decay), so gdn_step is bit-exact.
//
// The decode ops are tiny (one head: 128 x 128 state, 64 KB) and latency-bound.  gdn_step
// on 128 x 128 heads (Qwen3.5's) gives each warp 32 value columns of one head, copies
// them to shared memory with every row's 128 bytes in flight at once, runs both passes
// there and stores each column element once; the grid is heads x ceil(v_dim / 32)
// one-warp CTAs.  Other shapes use the two-pass kernel that reads the column from global
// memory in each pass.
#include "common.cuh"
#include "kernels.h"

namespace tqb200 {
namespace {

constexpr int kGdnThreads = 256;

__device__ __forceinline__ float silu_ref(float x) {
    return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}

// Block-wide double sum of squares (tree order), broadcast to every thread.
__device__ double block_sumsq(const float *x, int n) {
    __shared__ double s_part[32];
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (double)x[i] * (double)x[i];
    ss = warp_sum_d(ss);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    if (lane == 0) s_part[warp] = ss;
    __syncthreads();
    double tot = lane < nw ? s_part[lane] : 0.0;
    tot = warp_sum_d(tot);
    __syncthreads();  // s_part reusable
    return tot;
}

// One vector per CTA (n_vec vectors of n floats, stride n).
__global__ void l2norm_kernel(float *__restrict__ x, int n, float eps) {
    float *v = x + (size_t)blockIdx.x * n;
    const double ss = block_sumsq(v, n);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)ss, eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x) v[i] = __fmul_rn(v[i], inv);
}

__global__ void causal_conv1d_kernel(const float *__restrict__ x, float *__restrict__ state,
                                     const float *__restrict__ weight, float *__restrict__ out,
                                     int dim, int ks) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= dim) return;
    const int sl = ks - 1;
    float *st = state + (size_t)c * sl;
    const float *w = weight + (size_t)c * ks;
    const float xc = x[c];
    float acc = 0.0f;
    for (int i = 0; i < sl; ++i) acc = __fadd_rn(acc, __fmul_rn(w[i], st[i]));
    acc = __fadd_rn(acc, __fmul_rn(w[sl], xc));
    out[c] = silu_ref(acc);
    for (int i = 0; i < sl - 1; ++i) st[i] = st[i + 1];
    st[sl - 1] = xc;
}

// One head per CTA (blockIdx.x), thread d over the value dimension; the head's state S
// [qk_dim][v_dim] is read and written twice (decay + S^T k, then the rank-1 update with
// the output sum of the updated rows, the reference's j order in both).
__global__ void gdn_step_kernel(float *__restrict__ S, const float *__restrict__ q,
                                const float *__restrict__ k, const float *__restrict__ v,
                                const float *__restrict__ decay, const float *__restrict__ beta,
                                float *__restrict__ o, int qk_dim, int v_dim) {
    extern __shared__ float s_qk[];  // [2][qk_dim]: q, k of this head
    const int h = blockIdx.x;
    S += (size_t)h * qk_dim * v_dim;
    q += (size_t)h * qk_dim;
    k += (size_t)h * qk_dim;
    v += (size_t)h * v_dim;
    o += (size_t)h * v_dim;
    for (int j = threadIdx.x; j < qk_dim; j += blockDim.x) {
        s_qk[j] = q[j];
        s_qk[qk_dim + j] = k[j];
    }
    __syncthreads();
    const float dc = decay[h], bt = beta[h];
    for (int d = threadIdx.x; d < v_dim; d += blockDim.x) {
        float kv = 0.0f;
        for (int j = 0; j < qk_dim; ++j) {
            const float sv = __fmul_rn(S[(size_t)j * v_dim + d], dc);
            S[(size_t)j * v_dim + d] = sv;
            kv = __fadd_rn(kv, __fmul_rn(sv, s_qk[qk_dim + j]));
        }
        const float delta = __fmul_rn(bt, __fsub_rn(v[d], kv));
        double acc = 0.0;
        for (int j = 0; j < qk_dim; ++j) {
            const float sv = __fadd_rn(S[(size_t)j * v_dim + d], __fmul_rn(s_qk[qk_dim + j], delta));
            S[(size_t)j * v_dim + d] = sv;
            acc += (double)sv * (double)s_qk[j];
        }
        o[d] = (float)acc;
    }
}

// The same step with the warp's 32 columns of S staged in shared memory by 4-byte
// cp.async copies (all qk_dim rows in flight at once, no registers held), for qk_dim ==
// QK and v_dim == V known at compile time: one warp per 32 value columns of a head,
// identical rounding points and summation order.
template <int QK, int V>
__global__ void __launch_bounds__(32) gdn_step_warp_kernel(
    float *__restrict__ S, const float *__restrict__ q, const float *__restrict__ k,
    const float *__restrict__ v, const float *__restrict__ decay, const float *__restrict__ beta,
    float *__restrict__ o) {
    __shared__ float s_q[QK], s_k[QK];
    __shared__ float s_col[QK * 32];  // [j][lane]
    const int h = blockIdx.x, lane = threadIdx.x, d = blockIdx.y * 32 + lane;
    const bool live = d < V;
    float *const col_p = S + (size_t)h * QK * V + d;
    if (live) {
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(s_col + lane);
#pragma unroll 16
        for (int j = 0; j < QK; ++j)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst + 128u * j),
                         "l"(col_p + (size_t)j * V) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    q += (size_t)h * QK;
    k += (size_t)h * QK;
    for (int j = lane; j < QK; j += 32) {
        s_q[j] = q[j];
        s_k[j] = k[j];
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
    if (!live) return;
    const float dc = decay[h], bt = beta[h];
    float *col = s_col + lane;
    float kv = 0.0f;
#pragma unroll 8
    for (int j = 0; j < QK; ++j) {
        const float sv = __fmul_rn(col[32 * j], dc);
        col[32 * j] = sv;
        kv = __fadd_rn(kv, __fmul_rn(sv, s_k[j]));
    }
    const float delta = __fmul_rn(bt, __fsub_rn(v[(size_t)h * V + d], kv));
    double acc = 0.0;
#pragma unroll 8
    for (int j = 0; j < QK; ++j) {
        const float sv = __fadd_rn(col[32 * j], __fmul_rn(s_k[j], delta));
        col_p[(size_t)j * V] = sv;
        acc += (double)sv * (double)s_q[j];
    }
    o[(size_t)h * V + d] = (float)acc;
}

// One vector per CTA.
__global__ void rmsnorm_gated_kernel(const float *__restrict__ x, const float *__restrict__ gate,
                                     const float *__restrict__ w, float *__restrict__ y, int n,
                                     float eps) {
    x += (size_t)blockIdx.x * n;
    gate += (size_t)blockIdx.x * n;
    y += (size_t)blockIdx.x * n;
    const double ss = block_sumsq(x, n);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(ss / n), eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        y[i] = __fmul_rn(__fmul_rn(__fmul_rn(x[i], scale), w[i]), silu_ref(gate[i]));
}

// Rotate-half over dimensions [0, rotary_dim) of every head; cs/sn = the rotary_dim / 2
// cos/sin values of the position.
__global__ void partial_rope_kernel(float *__restrict__ q, float *__restrict__ k, int n_heads,
                                    int head_dim, int rotary_dim, const float *__restrict__ cs,
                                    const float *__restrict__ sn) {
    const int half = rotary_dim / 2;
    const int h = blockIdx.x;
    float *x = h < n_heads ? q + (size_t)h * head_dim : k + (size_t)(h - n_heads) * head_dim;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float c = cs[i], s = sn[i];
        const float x0 = x[i], x1 = x[i + half];
        x[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        x[i + half] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
    }
}

}  // namespace

int launch_l2norm(float *x, int n_vec, int n, float eps, cudaStream_t st) {
    TQ_CHECK_ARG(n > 0 && n_vec > 0 && n_vec <= 65535, "l2norm: %d vectors of %d", n_vec, n);
    l2norm_kernel<<<n_vec, kGdnThreads, 0, st>>>(x, n, eps);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_causal_conv1d(const float *x, float *state, const float *w, float *out, int dim, int ks,
                         cudaStream_t st) {
    TQ_CHECK_ARG(dim > 0 && ks >= 2, "causal_conv1d_update: dim %d kernel_size %d (< 2)", dim, ks);
    causal_conv1d_kernel<<<(dim + 127) / 128, 128, 0, st>>>(x, state, w, out, dim, ks);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_gdn_step(float *S, const float *q, const float *k, const float *v, const float *decay,
                    const float *beta, float *o, int n_heads, int qk_dim, int v_dim,
                    cudaStream_t st) {
    TQ_CHECK_ARG(n_heads > 0 && n_heads <= 65535 && qk_dim > 0 && qk_dim <= 4096 && v_dim > 0 &&
                     v_dim <= 512,
                 "gdn_step: %d heads, qk_dim %d, v_dim %d (v_dim 1..512)", n_heads, qk_dim, v_dim);
    const dim3 grid(n_heads, (v_dim + 31) / 32);
    if (qk_dim == 128 && v_dim == 128) {  // every Qwen3.5 linear-attention head
        gdn_step_warp_kernel<128, 128><<<grid, 32, 0, st>>>(S, q, k, v, decay, beta, o);
    } else {
        const int threads = ((v_dim + 31) / 32) * 32;
        gdn_step_kernel<<<n_heads, threads, (size_t)2 * qk_dim * 4, st>>>(S, q, k, v, decay, beta,
                                                                          o, qk_dim, v_dim);
    }
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_rmsnorm_gated(const float *x, const float *gate, const float *w, float *y, int n_vec,
                         int n, float eps, cudaStream_t st) {
    TQ_CHECK_ARG(n > 0 && n_vec > 0 && n_vec <= 65535, "rmsnorm_gated: %d vectors of %d", n_vec, n);
    rmsnorm_gated_kernel<<<n_vec, kGdnThreads, 0, st>>>(x, gate, w, y, n, eps);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_partial_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim,
                        int rotary_dim, const float *cs, const float *sn, cudaStream_t st) {
    TQ_CHECK_ARG(rotary_dim > 0 && rotary_dim <= head_dim && rotary_dim % 2 == 0 &&
                     rotary_dim / 2 <= 256,
                 "partial_rope: bad rotary_dim %d (head_dim %d)", rotary_dim, head_dim);
    if (n_heads + n_kv_heads == 0) return TQB200_OK;
    partial_rope_kernel<<<n_heads + n_kv_heads, 128, 0, st>>>(q, k, n_heads, head_dim, rotary_dim,
                                                            cs, sn);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

}  // namespace tqb200
