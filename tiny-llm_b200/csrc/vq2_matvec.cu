// vq2_matvec.cu — VQ2 2-bit codebook matvec and BiIP activation rotation, sm_100a.
//
// Reference semantics:
//   matvec_vq2_ref (kernels/matvec/matvec_vq2_ref.cpp:52-82): the tensor is
//     [codebook 256 x 4 fp16 = 2048 B][one uint8 index per 4 weights, row-major],
//     y[o] = sum_b sum_j cb[idx[o,b]][j] * x[4b+j]
//   biip_rotate_activation_ref (kernels/biip/biip_rotate.cpp:36-69):
//     y = FWHT_bs((x / scale) * sign) / sqrt(bs) per block of bs elements, with the
//     butterfly order h = 1, 2, 4, ... (pairs (j, j+h)); elements past the last full
//     block keep (x / scale) * sign.
//
// Design: VQ2 at batch 1 is gather-bound, not HBM-bound (a weight byte selects a
// 16-byte codebook vector).  The codebook is decoded once per CTA into shared
// memory as 8 interleaved fp32 copies, entry k of copy p at byte k*128 + p*16:
// the 8 lanes of each LDS.128 phase (lane % 8 = p) always hit 8 distinct 16-byte
// bank groups, so the random lookups are conflict free.  Thread (slot, seg) owns
// 16 columns (4 index bytes, one coalesced 32-bit load per row) and keeps its 16
// activations in registers; row sums reduce through shared memory.  The BiIP
// rotation (optionally after an RMSNorm) runs in the prologue in shared memory
// with the reference's butterfly order, so the rotated activations are bit-exact.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace tqb200 {

namespace {

constexpr int kVqThreads = 256;

struct VqParams {
    const uint8_t *w;     // [codebook][indices]
    float *y;
    const float *resid;   // optional residual: y = resid + dot
    int rows, K;
    XSource x;            // X_PLAIN / X_RMSNORM / X_SWIGLU source
    const float *rot_sign, *rot_scale;  // BiIP (sign == nullptr: no rotation)
    int rot_bs;
    int nt, S;            // threads per row (K/16) and row slots
};

// In-place BiIP of v[0..K) in shared memory by the whole CTA.
__device__ void biip_smem(float *v, int K, const float *sign, const float *scale, int bs) {
    for (int j = threadIdx.x; j < K; j += blockDim.x)
        v[j] = scale ? __fmul_rn(__fdiv_rn(v[j], scale[j]), sign[j]) : __fmul_rn(v[j], sign[j]);
    __syncthreads();
    if (bs <= 1) return;
    const int nblk = K / bs;
    for (int h = 1; h < bs; h <<= 1) {
        // butterfly pairs (j, j+h) with j in [i, i+h) for i = 0, 2h, 4h, ...
        const int pairs = nblk * (bs / 2);
        for (int t = threadIdx.x; t < pairs; t += blockDim.x) {
            const int b = t / (bs / 2), r = t - b * (bs / 2);
            const int j = (r / h) * 2 * h + (r % h);
            float *blk = v + (size_t)b * bs;
            const float a = blk[j], c = blk[j + h];
            blk[j] = __fadd_rn(a, c);
            blk[j + h] = __fsub_rn(a, c);
        }
        __syncthreads();
    }
    const float inv = 1.0f / sqrtf((float)bs);
    for (int j = threadIdx.x; j < nblk * bs; j += blockDim.x) v[j] = __fmul_rn(v[j], inv);
    __syncthreads();
}

__global__ void __launch_bounds__(kVqThreads) vq2_matvec_kernel(const __grid_constant__ VqParams P) {
    extern __shared__ __align__(16) uint8_t smem[];
    float4 *cb = reinterpret_cast<float4 *>(smem);            // [256][8] float4
    float *xs = reinterpret_cast<float *>(smem + 256 * 8 * 16);   // [K]
    float *red = xs + P.K;                                     // [S][nt]
    __shared__ double s_rd[32];
    const int t = threadIdx.x, K = P.K;
    // codebook -> 8 interleaved fp32 copies (weights: no dependency on the previous kernel)
    for (int i = t; i < 256 * 8; i += blockDim.x) {
        const int k = i >> 3;
        const uint16_t *h = reinterpret_cast<const uint16_t *>(P.w) + k * 4;
        cb[i] = make_float4(h2f(h[0]), h2f(h[1]), h2f(h[2]), h2f(h[3]));
    }
    griddep_wait();
    // activation prologue: source (+RMSNorm / SwiGLU), then BiIP
    float rms_scale = 0.0f;
    if (P.x.mode == X_RMSNORM) {
        double ss = 0.0;
        for (int i = t; i < K; i += blockDim.x) {
            const double v = (double)P.x.src[i];
            ss += v * v;
        }
        ss = warp_sum_d(ss);
        if ((t & 31) == 0) s_rd[t >> 5] = ss;
        __syncthreads();
        if (t < 32) {
            double v = t < (int)(blockDim.x >> 5) ? s_rd[t] : 0.0;
            v = warp_sum_d(v);
            if (t == 0) s_rd[0] = v;
        }
        __syncthreads();
        rms_scale = 1.0f / sqrtf(__fadd_rn((float)(s_rd[0] / K), P.x.eps));
    }
    for (int i = t; i < K; i += blockDim.x) {
        float v;
        if (P.x.mode == X_RMSNORM) {
            v = __fmul_rn(__fmul_rn(P.x.src[i], rms_scale), P.x.norm_w[i]);
        } else if (P.x.mode == X_SWIGLU) {
            const float g = P.x.src[i];
            v = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), P.x.up[i]);
        } else {
            v = P.x.src[i];
        }
        xs[i] = v;
    }
    __syncthreads();
    if (P.rot_sign) biip_smem(xs, K, P.rot_sign, P.rot_scale, P.rot_bs);
    griddep_launch();

    const int nt = P.nt, S = P.S;
    const int slot = t / nt, sg = t - slot * nt;
    const bool active = slot < S;
    const int c0 = sg * 16;  // 4 blocks of 4 columns
    float xv[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) xv[i] = (active && c0 + i < K) ? xs[c0 + i] : 0.0f;
    const uint32_t lane_off = (uint32_t)(t & 7) * 16u;
    const uint8_t *cbb = smem;
    const int nb = K / 4;
    const uint8_t *idx = P.w + 2048;
    const int lane = t & 31, warp = t >> 5, nwarps = blockDim.x >> 5;
    for (int r0 = blockIdx.x * S; r0 < P.rows; r0 += gridDim.x * S) {
        const int row = r0 + slot;
        if (active) {
            float acc = 0.0f;
            if (row < P.rows) {
                const uint8_t *ip = idx + (size_t)row * nb + sg * 4;
                uint32_t wd;
                if (sg * 4 + 4 <= nb && (((uintptr_t)ip) & 3u) == 0) {
                    wd = ldg_u32(ip);
                } else {
                    wd = 0;
                    for (int b = 0; b < 4 && sg * 4 + b < nb; ++b) wd |= (uint32_t)ip[b] << (8 * b);
                }
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const uint32_t k = (wd >> (8 * b)) & 0xFFu;
                    const float4 c = *reinterpret_cast<const float4 *>(cbb + (k << 7) + lane_off);
                    acc = fmaf(c.x, xv[4 * b + 0], acc);
                    acc = fmaf(c.y, xv[4 * b + 1], acc);
                    acc = fmaf(c.z, xv[4 * b + 2], acc);
                    acc = fmaf(c.w, xv[4 * b + 3], acc);
                }
            }
            red[slot * nt + sg] = acc;
        }
        __syncthreads();
        for (int rl = warp; rl < S; rl += nwarps) {
            const int rr = r0 + rl;
            if (rr >= P.rows) continue;
            float v = 0.0f;
            for (int i = lane; i < nt; i += 32) v += red[rl * nt + i];
            v = warp_sum(v);
            if (lane == 0) P.y[rr] = P.resid ? P.resid[rr] + v : v;
        }
        __syncthreads();
    }
}

// Standalone BiIP rotation (per-op entry point): one CTA, x -> y.
__global__ void biip_kernel(const float *__restrict__ x, float *__restrict__ y, int dim,
                            const float *sign, const float *scale, int bs) {
    extern __shared__ float v[];
    for (int j = threadIdx.x; j < dim; j += blockDim.x) v[j] = x[j];
    __syncthreads();
    biip_smem(v, dim, sign, scale, bs);
    for (int j = threadIdx.x; j < dim; j += blockDim.x) y[j] = v[j];
}

}  // namespace

int launch_vq2_matvec(const VqLaunch &a, cudaStream_t st) {
    TQ_CHECK_ARG(a.rows >= 0 && a.K > 0 && a.K % 4 == 0, "vq2: bad shape %d x %d", a.rows, a.K);
    TQ_CHECK_ARG(!a.rot_sign || (a.rot_bs >= 1 && (a.rot_bs & (a.rot_bs - 1)) == 0),
                 "vq2: rotation block %d", a.rot_bs);
    if (a.rows == 0) return TQB200_OK;
    VqParams P{};
    P.w = a.w;
    P.y = a.y;
    P.resid = a.resid;
    P.rows = a.rows;
    P.K = a.K;
    P.x = a.x;
    P.rot_sign = a.rot_sign;
    P.rot_scale = a.rot_scale;
    P.rot_bs = a.rot_bs;
    P.nt = (a.K + 15) / 16;
    TQ_CHECK_ARG(P.nt <= kVqThreads, "vq2: in_dim %d above %d", a.K, 16 * kVqThreads);
    P.S = std::max(1, kVqThreads / P.nt);
    const size_t smem = 256 * 8 * 16 + (size_t)a.K * 4 + (size_t)P.S * P.nt * 4;
    static bool attr = false;
    if (!attr) {
        TQ_CUDA_TRY(cudaFuncSetAttribute(vq2_matvec_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
        attr = true;
    }
    TQ_CHECK_ARG(smem <= 160 * 1024, "vq2: in_dim %d needs too much shared memory", a.K);
    int per_sm = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, vq2_matvec_kernel, kVqThreads, smem);
    const int passes = (a.rows + P.S - 1) / P.S;
    const int grid = std::max(1, std::min(passes, std::max(1, per_sm) * num_sms()));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kVqThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr_l[1];
    attr_l[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr_l[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr_l;
    cfg.numAttrs = a.pdl ? 1 : 0;
    TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, vq2_matvec_kernel, P));
    return TQB200_OK;
}

int launch_biip(const float *x, float *y, int dim, const float *scale, const float *sign, int bs,
                cudaStream_t st) {
    TQ_CHECK_ARG(dim > 0 && sign && bs >= 1 && (bs & (bs - 1)) == 0, "biip: bad arguments");
    TQ_CHECK_ARG((size_t)dim * 4 <= 160 * 1024, "biip: dim %d too large", dim);
    static bool attr = false;
    if (!attr) {
        TQ_CUDA_TRY(cudaFuncSetAttribute(biip_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         160 * 1024));
        attr = true;
    }
    biip_kernel<<<1, 512, (size_t)dim * 4, st>>>(x, y, dim, sign, scale, bs);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

}  // namespace tqb200
