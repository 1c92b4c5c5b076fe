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
//   applied per projection as QwenModel::mv_rot does (runtime/qwen_model.cpp:229-238).
//
// Design.  VQ2 at batch 1 is latency- and gather-bound, not HBM-bound: a whole
// Qwen3-0.6B-shaped layer is 3.9 MB, and a weight byte selects a 16-byte codebook
// vector.  So a launch carries up to three matrices (q/k/v, or gate/up paired with
// the SwiGLU epilogue), each CTA owns one contiguous row block of one matrix, and
// everything a CTA reads comes in by TMA bulk copies issued up front: its
// codebook, its whole index block and the constant vectors (RMSNorm weight, BiIP
// sign and scale) before griddepcontrol.wait, the activation vector after it.
// The codebook is decoded into shared memory as 8 interleaved fp32 copies (entry
// k of copy p at byte k*128 + p*16): the 8 lanes of each LDS.128 phase (lane % 8
// = p) hit 8 distinct 16-byte bank groups, so random lookups are conflict free.
// Thread (slot, seg) owns 16 columns (4 index bytes per row) and keeps its 16
// (rotated) activations in registers; row sums reduce through shared memory.  The
// BiIP rotation runs in shared memory with the reference's butterfly order, so the
// rotated activations are bit-exact.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace tqb200 {

namespace {

constexpr int kVqMaxThreads = 256;
constexpr int kCbBytes = 2048;            // 256 entries x 4 fp16
constexpr int kCbDecoded = 256 * 8 * 16;  // 8 interleaved fp32 copies

struct VqParams {
    VqJob job[3];
    int cta_begin[4];  // CTAs [cta_begin[j], cta_begin[j+1]) serve job j (pair: job 0)
    int n_jobs, pair, K, nt, S, rpc;  // rpc: rows per CTA (a multiple of S)
    int bulk;          // bases 16-byte aligned and K % 64 == 0: bulk copies
    int region;        // bytes of one matrix's staging region (codebook + index block)
    XSource x;
    int *status;
    Stamp stamp;       // in-graph timeline (off unless the engine records one)
};

// One Hadamard block of BS = 32 * E elements in registers (lane l holds elements
// l*E .. l*E+E-1): butterfly levels h = 1, 2, 4, ... in the reference's order, the pairs
// inside a lane first, then across lanes (partner l ^ (h / E)); every butterfly is the
// reference's (a + b, a - b) on the same operands, so the result is bit-exact.
template <int E>
__device__ __forceinline__ void fwht_warp(float (&e)[E], int lane) {
#pragma unroll
    for (int h = 1; h < E; h <<= 1) {
#pragma unroll
        for (int j = 0; j < E; ++j)
            if ((j & h) == 0) {
                const float a = e[j], c = e[j + h];
                e[j] = __fadd_rn(a, c);
                e[j + h] = __fsub_rn(a, c);
            }
    }
#pragma unroll
    for (int hl = 1; hl < 32; hl <<= 1) {
        const bool upper = (lane & hl) != 0;
#pragma unroll
        for (int j = 0; j < E; ++j) {
            const float o = __shfl_xor_sync(0xffffffffu, e[j], hl);
            e[j] = upper ? __fsub_rn(o, e[j]) : __fadd_rn(e[j], o);
        }
    }
}

template <int E>
__device__ void biip_blocks_warp(float *v, int nblk, const float *sign, const float *scale) {
    constexpr int BS = 32 * E;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float inv = 1.0f / sqrtf((float)BS);
    for (int b = warp; b < nblk; b += nw) {
        float e[E];
        const int base = b * BS + lane * E;
#pragma unroll
        for (int i = 0; i < E; ++i) {
            const int j = base + i;
            e[i] = scale ? __fmul_rn(__fdiv_rn(v[j], scale[j]), sign[j]) : __fmul_rn(v[j], sign[j]);
        }
        fwht_warp<E>(e, lane);
#pragma unroll
        for (int i = 0; i < E; ++i) v[base + i] = __fmul_rn(e[i], inv);
    }
}

// In-place BiIP of v[0..K) in shared memory by the whole CTA (sign/scale anywhere).
// Blocks of 32..256 elements run one per warp in registers; other sizes through shared
// memory with a barrier per butterfly level.
__device__ void biip_smem(float *v, int K, const float *sign, const float *scale, int bs) {
    if (bs >= 32 && bs <= 256) {
        const int nblk = K / bs;
        for (int j = nblk * bs + threadIdx.x; j < K; j += blockDim.x)  // tail: sign/scale only
            v[j] = scale ? __fmul_rn(__fdiv_rn(v[j], scale[j]), sign[j]) : __fmul_rn(v[j], sign[j]);
        switch (bs) {
            case 32: biip_blocks_warp<1>(v, nblk, sign, scale); break;
            case 64: biip_blocks_warp<2>(v, nblk, sign, scale); break;
            case 128: biip_blocks_warp<4>(v, nblk, sign, scale); break;
            default: biip_blocks_warp<8>(v, nblk, sign, scale); break;
        }
        __syncthreads();
        return;
    }
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

template <bool STAMP>
__global__ void __launch_bounds__(kVqMaxThreads) vq2_matvec_kernel(const __grid_constant__ VqParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int t = threadIdx.x, K = P.K, nm = 1 + P.pair;  // matrices this CTA reads
    const size_t K4 = ((size_t)K * 4 + 15) & ~(size_t)15;
    uint64_t *bar_w = reinterpret_cast<uint64_t *>(smem);  // codebooks, indices, constants
    uint64_t *bar_x = bar_w + 1;                            // activation (+ SwiGLU up)
    uint8_t *cbf = smem + 128;                              // [nm][kCbDecoded]
    uint8_t *raw = cbf + (size_t)nm * kCbDecoded;           // [nm][region]
    float *xs = reinterpret_cast<float *>(raw + (size_t)nm * P.region);  // [K]
    float *wsm = xs + K4 / 4;                               // [K] norm weight / up
    float *xr = wsm + K4 / 4;                               // [nm][K] rotated
    float *rot = xr + (size_t)nm * K4 / 4;                  // [nm][2][K] sign, scale
    float *red = rot + (size_t)nm * 2 * K4 / 4;             // [nm][S][nt]
    __shared__ int s_err;
    __shared__ double s_rd[32];
    StampRegs stamp_r;
    stamp_enter<STAMP>(P.stamp, stamp_r);

    int j = 0;
    while (j + 1 < P.n_jobs && (int)blockIdx.x >= P.cta_begin[j + 1]) ++j;
    const int r0 = ((int)blockIdx.x - P.cta_begin[j]) * P.rpc;
    const int r1 = min(P.job[j].rows, r0 + P.rpc);
    const int nb = K / 4;  // index bytes per row
    const size_t idx_bytes = (size_t)max(0, r1 - r0) * nb;
    const bool norm = P.x.mode == X_RMSNORM;

    // ---- constant inputs (weights, norm weight, rotation vectors) before the wait
    if (t == 0) {
        mbar_init(bar_w, 1);
        mbar_init(bar_x, 1);
        fence_mbar_init();
        s_err = 0;
        if (P.bulk) {
            uint32_t tx = 0;
            for (int m = 0; m < nm; ++m) {
                const VqJob &jb = P.job[P.pair ? m : j];
                tx += kCbBytes + (uint32_t)idx_bytes;
                if (jb.rot_sign) tx += (uint32_t)K * 4u * (jb.rot_scale ? 2u : 1u);
            }
            if (norm) tx += (uint32_t)K * 4u;
            mbar_arrive_expect_tx(bar_w, tx);
            for (int m = 0; m < nm; ++m) {
                const VqJob &jb = P.job[P.pair ? m : j];
                uint8_t *dst = raw + (size_t)m * P.region;
                bulk_g2s(dst, jb.w, kCbBytes, bar_w);
                if (idx_bytes) bulk_g2s(dst + kCbBytes, jb.w + kCbBytes + (size_t)r0 * nb,
                                        (uint32_t)idx_bytes, bar_w);
                if (jb.rot_sign) {
                    bulk_g2s(rot + (size_t)(2 * m) * K4 / 4, jb.rot_sign, (uint32_t)K * 4u, bar_w);
                    if (jb.rot_scale)
                        bulk_g2s(rot + (size_t)(2 * m + 1) * K4 / 4, jb.rot_scale, (uint32_t)K * 4u,
                                 bar_w);
                }
            }
            if (norm) bulk_g2s(wsm, P.x.norm_w, (uint32_t)K * 4u, bar_w);
        }
    }
    stamp_step<STAMP>(P.stamp, stamp_r);
    griddep_wait();
    stamp_waited<STAMP>(P.stamp, stamp_r);
    griddep_launch();
    if (t == 0 && P.bulk) {
        const uint32_t xb = (uint32_t)K * 4u;
        mbar_arrive_expect_tx(bar_x, P.x.mode == X_SWIGLU ? 2 * xb : xb);
        bulk_g2s(xs, P.x.src, xb, bar_x);
        if (P.x.mode == X_SWIGLU) bulk_g2s(wsm, P.x.up, xb, bar_x);
    }
    if (!P.bulk) {
        // unaligned inputs: the same staging with plain loads, 4 in flight per thread
        for (int m = 0; m < nm; ++m) {
            const VqJob &jb = P.job[P.pair ? m : j];
            uint8_t *dst = raw + (size_t)m * P.region;
            const size_t n = kCbBytes + idx_bytes;
            for (size_t i0 = t; i0 < n; i0 += 4 * blockDim.x) {
                uint8_t v[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const size_t i = i0 + (size_t)k * blockDim.x;
                    v[k] = i < n ? jb.w[i < (size_t)kCbBytes ? i : i + (size_t)r0 * nb] : 0;
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const size_t i = i0 + (size_t)k * blockDim.x;
                    if (i < n) dst[i] = v[k];
                }
            }
            if (jb.rot_sign)
                for (int i = t; i < K; i += blockDim.x) {
                    rot[(size_t)(2 * m) * K4 / 4 + i] = jb.rot_sign[i];
                    if (jb.rot_scale) rot[(size_t)(2 * m + 1) * K4 / 4 + i] = jb.rot_scale[i];
                }
        }
        for (int i = t; i < K; i += blockDim.x) {
            xs[i] = P.x.src[i];
            if (norm) wsm[i] = P.x.norm_w[i];
            if (P.x.mode == X_SWIGLU) wsm[i] = P.x.up[i];
        }
    } else if (t == 0) {
        if (!mbar_wait(bar_w, 0, kWaitCycles)) s_err = 1;
        if (!mbar_wait(bar_x, 0, kWaitCycles)) s_err = 1;
    }
    __syncthreads();
    if (s_err) {
        if (t == 0) {  // drain before exit
            mbar_wait(bar_w, 0, kWaitCycles);
            mbar_wait(bar_x, 0, kWaitCycles);
            if (P.status) atomicExch(P.status, kDevTimeoutTma);
        }
        return;
    }
    // ---- codebooks -> 8 interleaved fp32 copies (thread t decodes entry t)
    for (int m = 0; m < nm; ++m) {
        const uint8_t *cr = raw + (size_t)m * P.region;
        float4 *cb = reinterpret_cast<float4 *>(cbf + (size_t)m * kCbDecoded);
        for (int k = t; k < 256; k += blockDim.x) {
            const uint2 h = *reinterpret_cast<const uint2 *>(cr + 8 * k);
            const float4 c = make_float4(h2f((uint16_t)(h.x & 0xFFFFu)), h2f((uint16_t)(h.x >> 16)),
                                         h2f((uint16_t)(h.y & 0xFFFFu)), h2f((uint16_t)(h.y >> 16)));
#pragma unroll
            for (int p = 0; p < 8; ++p) cb[k * 8 + p] = c;
        }
    }
    // ---- activation: RMSNorm / SwiGLU in place, then each matrix's rotation
    if (norm) {
        double ss = 0.0;
        for (int i = t; i < K; i += blockDim.x) ss += (double)xs[i] * (double)xs[i];
        ss = warp_sum_d(ss);
        if ((t & 31) == 0) s_rd[t >> 5] = ss;
        __syncthreads();
        if (t < 32) {
            double v = t < (int)(blockDim.x >> 5) ? s_rd[t] : 0.0;
            v = warp_sum_d(v);
            if (t == 0) s_rd[0] = v;
        }
        __syncthreads();
        const float rms = 1.0f / sqrtf(__fadd_rn((float)(s_rd[0] / K), P.x.eps));
        for (int i = t; i < K; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], rms), wsm[i]);
    } else if (P.x.mode == X_SWIGLU) {
        for (int i = t; i < K; i += blockDim.x) {
            const float g = xs[i];
            xs[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), wsm[i]);
        }
    }
    __syncthreads();
    const float *xm0 = xs, *xm1 = xs;
    for (int m = 0; m < nm; ++m) {
        const VqJob &jb = P.job[P.pair ? m : j];
        if (!jb.rot_sign) continue;
        float *v = xr + (size_t)m * K4 / 4;
        for (int i = t; i < K; i += blockDim.x) v[i] = xs[i];
        __syncthreads();
        biip_smem(v, K, rot + (size_t)(2 * m) * K4 / 4,
                  jb.rot_scale ? rot + (size_t)(2 * m + 1) * K4 / 4 : nullptr, jb.rot_bs);
        if (m == 0) xm0 = v;
        else xm1 = v;
    }

    const int nt = P.nt, S = P.S;
    const int slot = t / nt, sg = t - slot * nt;
    const bool active = slot < S;
    const int c0 = sg * 16;  // 4 blocks of 4 columns
    float xv[2][16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const bool in = active && c0 + i < K;
        xv[0][i] = in ? xm0[c0 + i] : 0.0f;
        xv[1][i] = (in && nm > 1) ? xm1[c0 + i] : 0.0f;
    }
    const uint32_t lane_off = (uint32_t)(t & 7) * 16u;
    const int lane = t & 31, warp = t >> 5, nwarps = blockDim.x >> 5;
    const VqJob &job = P.job[j];
    for (int rb = r0; rb < r1; rb += S) {
        const int row = rb + slot;
        if (active) {
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                if (m >= nm) break;
                float acc = 0.0f;
                if (row < r1) {
                    const uint8_t *ip =
                        raw + (size_t)m * P.region + kCbBytes + (size_t)(row - r0) * nb + sg * 4;
                    uint32_t wd = 0;
                    if (sg * 4 + 4 <= nb && ((uintptr_t)ip & 3u) == 0) {
                        wd = *reinterpret_cast<const uint32_t *>(ip);
                    } else {
                        for (int b = 0; b < 4 && sg * 4 + b < nb; ++b) wd |= (uint32_t)ip[b] << (8 * b);
                    }
                    const uint8_t *cbb = cbf + (size_t)m * kCbDecoded;
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const uint32_t k = (wd >> (8 * b)) & 0xFFu;
                        const float4 c = *reinterpret_cast<const float4 *>(cbb + (k << 7) + lane_off);
                        acc = fmaf(c.x, xv[m][4 * b + 0], acc);
                        acc = fmaf(c.y, xv[m][4 * b + 1], acc);
                        acc = fmaf(c.z, xv[m][4 * b + 2], acc);
                        acc = fmaf(c.w, xv[m][4 * b + 3], acc);
                    }
                }
                red[((size_t)m * S + slot) * nt + sg] = acc;
            }
        }
        __syncthreads();
        for (int rl = warp; rl < S; rl += nwarps) {
            const int rr = rb + rl;
            if (rr >= r1) continue;
            float v = 0.0f, u = 0.0f;
            for (int i = lane; i < nt; i += 32) v += red[(size_t)rl * nt + i];
            v = warp_sum(v);
            if (P.pair) {
                for (int i = lane; i < nt; i += 32) u += red[((size_t)S + rl) * nt + i];
                u = warp_sum(u);
            }
            if (lane == 0) {
                if (P.pair) {  // swiglu_ref (kernels/silu/swiglu_ref.cpp:41-52) on (gate, up)
                    job.y[rr] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u);
                } else {
                    job.y[rr] = job.resid ? job.resid[rr] + v : v;
                }
            }
        }
        __syncthreads();
    }
    stamp_exit<STAMP>(P.stamp, stamp_r);
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

int hadamard_bs(int dim) {  // runtime/qwen_model.cpp:61-67
    for (int b = 256; b >= 2; b >>= 1)
        if (dim % b == 0) return b;
    return 1;
}

}  // namespace

int launch_vq2_matvec(const VqLaunch &a, cudaStream_t st) {
    TQ_CHECK_ARG(a.n_jobs >= 1 && a.n_jobs <= 3, "vq2: n_jobs %d", a.n_jobs);
    TQ_CHECK_ARG(a.K > 0 && a.K % 4 == 0, "vq2: in_dim %d not a multiple of 4", a.K);
    TQ_CHECK_ARG(!a.pair_swiglu || (a.n_jobs == 2 && a.job[0].rows == a.job[1].rows),
                 "vq2: paired SwiGLU needs two jobs with equal rows");
    VqParams P{};
    P.n_jobs = a.n_jobs;
    P.pair = a.pair_swiglu ? 1 : 0;
    P.K = a.K;
    P.x = a.x;
    P.status = a.status;
    P.stamp = a.stamp;
    P.nt = (a.K + 15) / 16;
    TQ_CHECK_ARG(P.nt <= kVqMaxThreads, "vq2: in_dim %d above %d", a.K, 16 * kVqMaxThreads);
    P.S = std::max(1, kVqMaxThreads / P.nt);
    const int block = (P.S * P.nt + 31) / 32 * 32;
    auto a16 = [](const void *p) { return ((uintptr_t)p & 15u) == 0; };
    bool bulk = a.K % 64 == 0 && a16(a.x.src) && (a.x.mode != X_RMSNORM || a16(a.x.norm_w)) &&
                (a.x.mode != X_SWIGLU || a16(a.x.up));
    int total = 0;
    for (int j = 0; j < a.n_jobs; ++j) {
        const VqJob &jb = a.job[j];
        TQ_CHECK_ARG(jb.rows >= 0 && (jb.rows == 0 || (jb.w && jb.y)), "vq2: job %d", j);
        TQ_CHECK_ARG(!jb.rot_sign || jb.rot_bs == 0 || (jb.rot_bs & (jb.rot_bs - 1)) == 0,
                     "vq2: rotation block %d", jb.rot_bs);
        P.job[j] = jb;
        if (jb.rot_sign && jb.rot_bs == 0) P.job[j].rot_bs = hadamard_bs(a.K);
        bulk = bulk && a16(jb.w) &&
               (!jb.rot_sign || (a16(jb.rot_sign) && (!jb.rot_scale || a16(jb.rot_scale))));
        if (!P.pair || j == 0) total += jb.rows;
    }
    if (total == 0) return TQB200_OK;
    P.bulk = bulk ? 1 : 0;
    // rows per CTA: ~2 CTAs per SM over all the launch's rows, a multiple of S
    const int target = 2 * num_sms();
    int rpc = (total + target - 1) / target;
    rpc = std::max(P.S, (rpc + P.S - 1) / P.S * P.S);
    P.rpc = rpc;
    int ctas = 0;
    for (int j = 0; j < a.n_jobs; ++j) {
        P.cta_begin[j] = ctas;
        if (!P.pair || j == 0) ctas += (a.job[j].rows + rpc - 1) / rpc;
    }
    for (int j = a.n_jobs; j <= 3; ++j) P.cta_begin[j] = ctas;
    if (P.pair) P.cta_begin[1] = P.cta_begin[2] = P.cta_begin[3] = ctas;
    const int nm = 1 + P.pair;
    P.region = (int)(((size_t)kCbBytes + (size_t)rpc * (a.K / 4) + 15) & ~(size_t)15);
    const size_t K4 = ((size_t)a.K * 4 + 15) & ~(size_t)15;
    const size_t smem = 128 + (size_t)nm * (kCbDecoded + P.region) + 2 * K4 + (size_t)nm * 3 * K4 +
                        (size_t)nm * P.S * P.nt * 4;
    static KernelSmem attr, attr_st;
    const bool stamped = P.stamp.base != nullptr;
    auto kern = stamped ? vq2_matvec_kernel<true> : vq2_matvec_kernel<false>;
    int smem_max = 0;
    TQ_CUDA_TRY(smem_limit_once(kern, stamped ? attr_st : attr, &smem_max));
    TQ_CHECK_ARG(smem <= (size_t)smem_max, "vq2: in_dim %d needs too much shared memory", a.K);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr_l[1];
    attr_l[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr_l[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr_l;
    cfg.numAttrs = a.pdl ? 1 : 0;
    TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, P));
    return TQB200_OK;
}

int launch_biip(const float *x, float *y, int dim, const float *scale, const float *sign, int bs,
                cudaStream_t st) {
    TQ_CHECK_ARG(dim > 0 && sign && bs >= 1 && (bs & (bs - 1)) == 0, "biip: bad arguments");
    static KernelSmem attr;
    int smem_max = 0;
    TQ_CUDA_TRY(smem_limit_once(biip_kernel, attr, &smem_max));
    TQ_CHECK_ARG((size_t)dim * 4 <= (size_t)smem_max, "biip: dim %d too large", dim);
    biip_kernel<<<1, 512, (size_t)dim * 4, st>>>(x, y, dim, sign, scale, bs);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

}  // namespace tqb200
