// i4_matvec.cu — batch-1 i4 (HQQ/RTN group-quantised) matvec kernels for sm_100a.
//
// Reference semantics: matvec_i4_ref (kernels/matvec/matvec_i4_ref.cpp:45-103):
//   y[o] = sum_g sum_i ((float)q - zero_g) * scale_g * x[i]
// on rows of ceil(K/G) groups laid out [scale f16][zero f16][G/2 nibble bytes]
// (runtime/tiny_format.h:66-77), low nibble = even column.
//
// Main kernel (i4_mv_tma_kernel), HBM-bound at batch 1:
//  * The interleaved layout is streamed as stored.  A CTA owns passes of R
//    consecutive rows (one contiguous byte range each); one thread issues a
//    1-D TMA bulk copy (cp.async.bulk + mbarrier complete_tx) per pass into a
//    ring of STAGES shared-memory buffers, so loads are 16-byte granular,
//    fully coalesced and need no registers while in flight.
//  * Weight prefetch is issued before griddepcontrol.wait: under programmatic
//    dependent launch the next matvec's weights stream while the previous
//    kernel still finishes; only the activation read waits for it.
//  * Thread (slot, seg) owns one SEG-column segment (SEG = 32 or 64, dividing
//    G) of rows slot, slot+S, ... of every pass and keeps its SEG activations
//    in registers for the whole kernel.  Reads from shared memory are
//    bank-conflict free (segment stride 9 or 5 words).
//  * Math (MATH_F32): a nibble becomes an exact float with one LOP3 (bits
//    OR'ed into the mantissa of 2^23, activations pre-scaled by 16^-k) and one
//    FADD; then one FFMA per weight, using
//        sum_i (q_i - z) s x_i = s * (sum_i q_i x_i - z * sum_i x_i).
//    (MATH_DP4A): activations split into three int8 digits per segment
//    (x ~ d0*s0 + d1*s0/254 + d2*s0/254^2, error <= 6e-8 * max|x|), and the
//    nibble dots run as exact integer dp4a (2 unpack ops + 6 dp4a per 8
//    weights).
//  * Optional fused prologues (RMSNorm of the source, SwiGLU of gate/up) and
//    epilogues (bias, residual add, greedy argmax over the rows).
//  * Every mbarrier wait is bounded; on timeout the kernel records an error
//    word, drains its outstanding copies (again bounded) and returns.
// Accumulation is fp32 (the reference accumulates in double); results agree
// to ~1e-6 relative, inside the 1e-4 max-relative tolerance of the tests.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace tqb200 {

namespace {

constexpr uint32_t kMagic = 0x4B000000u;  // 2^23
constexpr float kMagicF = 8388608.0f;
constexpr int kMaxStages = 8;
constexpr int MATH_F32 = 0;
constexpr int MATH_DP4A = 1;

struct MvParams {
    I4Job job[3];
    int pass_begin[4];
    int n_jobs;
    int K, G, nt, S, RP, R;
    int stages;
    uint32_t stage_bytes;
    int pair;  // jobs 0 and 1 (gate, up) share passes; y0 = silu(W0 x) * (W1 x)
    XSource x;
    ArgmaxOut am;
    int *status;
};

__device__ __forceinline__ float nib_f(uint32_t w, uint32_t mask) {
    return __uint_as_float((w & mask) | kMagic) - kMagicF;
}

// One 32-bit word of 8 nibbles against 8 activations pre-scaled by 16^-pos.
__device__ __forceinline__ void dot8(uint32_t w, const float *xs, float &a0, float &a1) {
    const uint32_t w2 = w >> 12;
    a0 = fmaf(nib_f(w, 0x0000000Fu), xs[0], a0);
    a1 = fmaf(nib_f(w, 0x000000F0u), xs[1], a1);
    a0 = fmaf(nib_f(w, 0x00000F00u), xs[2], a0);
    a1 = fmaf(nib_f(w, 0x0000F000u), xs[3], a1);
    a0 = fmaf(nib_f(w, 0x000F0000u), xs[4], a0);
    a1 = fmaf(nib_f(w2, 0x00000F00u), xs[5], a1);
    a0 = fmaf(nib_f(w2, 0x0000F000u), xs[6], a0);
    a1 = fmaf(nib_f(w2, 0x000F0000u), xs[7], a1);
}

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ int round_half_away(float v) {
    return (int)(v >= 0.0f ? v + 0.5f : v - 0.5f);
}

__device__ __forceinline__ void better(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

__device__ void block_argmax(float &bv, int &bi, float *sv, int *si) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        better(bv, bi, ov, oi);
    }
    __syncthreads();
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

// Rows [row0, row1) of one matrix -> a 16-byte aligned shared-memory region of `cap`
// bytes: the 16-byte aligned interior goes by one bulk copy (returned byte count),
// the ragged tail of the matrix (< 16 bytes) by plain loads.  *head = offset of row0.
__device__ uint32_t stage_rows(const MvParams &P, const I4Job &job, int row0, int row1,
                               uint8_t *dst, size_t cap, uint32_t *head, const uint8_t **src16) {
    const size_t RB = (size_t)((P.K + P.G - 1) / P.G) * (4 + P.G / 2);
    const uintptr_t a = (uintptr_t)(job.w + (size_t)row0 * RB);
    uintptr_t b = (uintptr_t)(job.w + (size_t)row1 * RB);
    const uintptr_t mat_end16 = (uintptr_t)(job.w + (size_t)job.rows * RB) & ~(uintptr_t)15;
    const uintptr_t a16 = a & ~(uintptr_t)15;
    uintptr_t b16 = (b + 15) & ~(uintptr_t)15;
    if (b16 > mat_end16) b16 = mat_end16;
    if (b16 < a16) b16 = a16;
    uint32_t bytes = (uint32_t)(b16 - a16);
    if ((size_t)(b - a16) > cap) {  // self-check: never write past the stage buffer
        if (P.status) atomicExch(P.status, kDevBadStage);
        bytes = 0;
        b = a16;
    }
    for (uintptr_t q = b16; q < b; ++q) dst[q - a16] = *(const uint8_t *)q;
    *head = (uint32_t)(a - a16);
    *src16 = (const uint8_t *)a16;
    return bytes;
}

// Thread 0: stream the rows of pass p into stage buffer s.  In paired mode the stage
// holds the same rows of job 0 and job 1 (gate and up) in its two halves.
__device__ void issue_pass(const MvParams &P, int p, int s, uint64_t *bars, uint8_t *stage_base,
                           uint32_t *s_head) {
    int j = 0;
    while (j + 1 < P.n_jobs && p >= P.pass_begin[j + 1]) ++j;
    const I4Job &job = P.job[j];
    const int row0 = (p - P.pass_begin[j]) * P.R;
    const int row1 = min(job.rows, row0 + P.R);
    uint8_t *dst = stage_base + (size_t)s * P.stage_bytes;
    const size_t cap = P.pair ? P.stage_bytes / 2 : P.stage_bytes;
    const uint8_t *src0, *src1 = nullptr;
    const uint32_t b0 = stage_rows(P, job, row0, row1, dst, cap, &s_head[s], &src0);
    uint32_t b1 = 0;
    if (P.pair)
        b1 = stage_rows(P, P.job[1], row0, row1, dst + cap, cap, &s_head[kMaxStages + s], &src1);
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&bars[s], b0 + b1);
    if (b0) bulk_g2s(dst, src0, b0, &bars[s]);
    if (b1) bulk_g2s(dst + cap, src1, b1, &bars[s]);
}

template <int SEG, int MATH>
__global__ void __launch_bounds__(512) i4_mv_tma_kernel(const __grid_constant__ MvParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NW = SEG / 8;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    uint8_t *stage_base = smem + 128;
    float *red = reinterpret_cast<float *>(stage_base + (size_t)P.stages * P.stage_bytes);
    __shared__ uint32_t s_head[2 * kMaxStages];
    __shared__ int s_err;
    __shared__ double s_rd[32];
    __shared__ float s_bv[32];
    __shared__ int s_bi[32];
    __shared__ bool s_last;

    const int t = threadIdx.x;
    const int total = P.pass_begin[P.n_jobs];
    if (t == 0) {
        for (int s = 0; s < P.stages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        s_err = 0;
    }
    __syncthreads();
    if (t == 0) {
        for (int s = 0; s < P.stages; ++s) {
            const int p = blockIdx.x + s * gridDim.x;
            if (p < total) issue_pass(P, p, s, bars, stage_base, s_head);
        }
    }
    // weights are in flight; now wait for the producer of x and let our dependents start
    griddep_wait();
    griddep_launch();

    const int nt = P.nt, S = P.S, K = P.K, G = P.G;
    const int slot = t / nt;
    const int sg = t - slot * nt;
    const bool active = slot < S;
    const int GB = 4 + G / 2;
    const size_t RB = (size_t)((K + G - 1) / G) * GB;
    const int spg = G / SEG;
    const int g = sg / spg;
    const int col0 = sg * SEG;
    const uint32_t hdr_off = (uint32_t)g * GB;
    const uint32_t seg_off = hdr_off + 4u + (uint32_t)(sg - g * spg) * (SEG / 2);

    // ---- activation prologue: the whole vector into shared memory with coalesced
    // loads (RMSNorm / SwiGLU applied there), then each thread takes its segment
    // [nt * SEG] floats, zero past K
    float *xsm = red + (((size_t)(1 + P.pair) * P.R * nt + 3) & ~(size_t)3);
    {
        const int KP = nt * SEG;  // every segment a thread can own (>= K)
        double ss = 0.0;
        for (int i = t; i < KP; i += blockDim.x) {
            float v = 0.0f;
            if (i < K) {
                if (P.x.mode == X_SWIGLU) {
                    const float gv = P.x.src[i];
                    v = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), P.x.up[i]);
                } else {
                    v = P.x.src[i];
                }
            }
            if (P.x.mode == X_RMSNORM) ss += (double)v * (double)v;
            xsm[i] = v;
        }
        if (P.x.mode == X_RMSNORM) {
            ss = warp_sum_d(ss);
            if ((t & 31) == 0) s_rd[t >> 5] = ss;
            __syncthreads();
            if (t < 32) {
                double v = t < (int)(blockDim.x >> 5) ? s_rd[t] : 0.0;
                v = warp_sum_d(v);
                if (t == 0) s_rd[0] = v;
            }
            __syncthreads();
            const float mean_sq = (float)(s_rd[0] / K);
            const float rms_scale = 1.0f / sqrtf(__fadd_rn(mean_sq, P.x.eps));
            for (int i = t; i < K; i += blockDim.x)
                xsm[i] = __fmul_rn(__fmul_rn(xsm[i], rms_scale), P.x.norm_w[i]);
        }
        __syncthreads();
    }
    // ---- per-segment tables, built once per CTA by all warps together (one warp per
    // segment, SEG/32 elements per lane): the segment sum X and, for dp4a, the three
    // int8 digit planes packed to match the nibble order of a 32-bit word
    // (lo word = even columns, hi word = odd columns) plus the digit scales.
    float *seg_x = xsm + (size_t)nt * SEG;                                  // [nt]
    float *seg_sc = seg_x + nt;                                             // [nt][3]
    uint32_t *seg_dig = reinterpret_cast<uint32_t *>(seg_sc + 3 * nt + 3);  // [nt][6*NW]
    seg_dig = reinterpret_cast<uint32_t *>(((uintptr_t)seg_dig + 15) & ~(uintptr_t)15);
    {
        const int lane_ = t & 31, warp_ = t >> 5, nw_ = blockDim.x >> 5;
        constexpr int EPL = SEG / 32;  // elements per lane
        for (int sgi = warp_; sgi < nt; sgi += nw_) {
            float v[EPL];
            float sum = 0.0f, amax = 0.0f;
#pragma unroll
            for (int e = 0; e < EPL; ++e) {
                v[e] = xsm[sgi * SEG + lane_ * EPL + e];
                sum += v[e];
                amax = fmaxf(amax, fabsf(v[e]));
            }
            sum = warp_sum(sum);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            if constexpr (MATH == MATH_DP4A) {
                const float s0 = amax > 0.0f ? amax / 127.0f : 1.0f;
                const float s1 = s0 / 254.0f, s2 = s1 / 254.0f;
                const float i0 = 1.0f / s0, i1 = 1.0f / s1, i2 = 1.0f / s2;
                uint8_t *db = reinterpret_cast<uint8_t *>(seg_dig + (size_t)sgi * 6 * NW);
#pragma unroll
                for (int e = 0; e < EPL; ++e) {
                    const int c = lane_ * EPL + e;               // column within the segment
                    const int chunk = c >> 3, k = c & 7;
                    const int word = 6 * chunk + (k & 1), byte = k >> 1;
                    const int q0 = max(-127, min(127, round_half_away(v[e] * i0)));
                    const float r1 = fmaf(-(float)q0, s0, v[e]);
                    const int q1 = max(-127, min(127, round_half_away(r1 * i1)));
                    const float r2 = fmaf(-(float)q1, s1, r1);
                    const int q2 = max(-127, min(127, round_half_away(r2 * i2)));
                    db[(word + 0) * 4 + byte] = (uint8_t)q0;
                    db[(word + 2) * 4 + byte] = (uint8_t)q1;
                    db[(word + 4) * 4 + byte] = (uint8_t)q2;
                }
                if (lane_ == 0) {
                    seg_sc[3 * sgi + 0] = s0;
                    seg_sc[3 * sgi + 1] = s1;
                    seg_sc[3 * sgi + 2] = s2;
                }
            }
            if (lane_ == 0) seg_x[sgi] = sum;
        }
        __syncthreads();
    }
    const float X = seg_x[sg];
    float xs[MATH == MATH_F32 ? SEG : 1];
    uint32_t xd[MATH == MATH_DP4A ? 6 * NW : 1];
    float dsc0 = 0.0f, dsc1 = 0.0f, dsc2 = 0.0f;
    if constexpr (MATH == MATH_F32) {
#pragma unroll
        for (int i = 0; i < NW; ++i)
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int pos = k < 5 ? k : k - 3;
                xs[8 * i + k] = xsm[col0 + 8 * i + k] * __uint_as_float((uint32_t)(127 - 4 * pos) << 23);
            }
    } else {
        const uint4 *src4 = reinterpret_cast<const uint4 *>(seg_dig + (size_t)sg * 6 * NW);
#pragma unroll
        for (int i = 0; i < 6 * NW / 4; ++i) {
            const uint4 w4 = src4[i];
            xd[4 * i + 0] = w4.x, xd[4 * i + 1] = w4.y, xd[4 * i + 2] = w4.z, xd[4 * i + 3] = w4.w;
        }
        dsc0 = seg_sc[3 * sg + 0];
        dsc1 = seg_sc[3 * sg + 1];
        dsc2 = seg_sc[3 * sg + 2];
    }

    const int lane = t & 31, warp = t >> 5, nwarps = blockDim.x >> 5;
    float bv = -INFINITY;
    int bi = INT_MAX;
    int i_pass = 0;
    for (;; ++i_pass) {
        const int p = blockIdx.x + i_pass * gridDim.x;
        if (p >= total) break;
        const int s = i_pass % P.stages;
        const uint32_t parity = (uint32_t)(i_pass / P.stages) & 1u;
        int j = 0;
        while (j + 1 < P.n_jobs && p >= P.pass_begin[j + 1]) ++j;
        const I4Job &job = P.job[j];
        const int row0 = (p - P.pass_begin[j]) * P.R;
        if (!mbar_wait(&bars[s], parity, kWaitCycles)) s_err = 1;
        const size_t half_bytes = P.stage_bytes / 2;
        if (active) {
            for (int r = 0; r < P.RP * (1 + P.pair); ++r) {
                const int jb = r >= P.RP;  // paired mode: second half = job 1
                const int rl = slot + (r - jb * P.RP) * S;
                const uint8_t *sb = stage_base + (size_t)s * P.stage_bytes +
                                    (jb ? half_bytes + s_head[kMaxStages + s] : s_head[s]);
                float part = 0.0f;
                if (row0 + rl < job.rows) {
                    const uint8_t *rp = sb + (size_t)rl * RB;
                    const uint32_t hv = lds_u32(rp + hdr_off);
                    const float sc = h2f((uint16_t)(hv & 0xFFFFu));
                    const float zr = h2f((uint16_t)(hv >> 16));
                    if constexpr (MATH == MATH_F32) {
                        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
                        for (int i = 0; i < NW; ++i) dot8(lds_u32(rp + seg_off + 4 * i), xs + 8 * i, a0, a1);
                        part = sc * fmaf(-zr, X, a0 + a1);
                    } else {
                        int D0 = 0, D1 = 0, D2 = 0;
#pragma unroll
                        for (int i = 0; i < NW; ++i) {
                            const uint32_t wd = lds_u32(rp + seg_off + 4 * i);
                            const uint32_t lo = wd & 0x0F0F0F0Fu, hi = (wd >> 4) & 0x0F0F0F0Fu;
                            D0 = dp4a_us(lo, xd[6 * i + 0], D0);
                            D0 = dp4a_us(hi, xd[6 * i + 1], D0);
                            D1 = dp4a_us(lo, xd[6 * i + 2], D1);
                            D1 = dp4a_us(hi, xd[6 * i + 3], D1);
                            D2 = dp4a_us(lo, xd[6 * i + 4], D2);
                            D2 = dp4a_us(hi, xd[6 * i + 5], D2);
                        }
                        const float dot = fmaf((float)D0, dsc0, fmaf((float)D1, dsc1, (float)D2 * dsc2));
                        part = sc * fmaf(-zr, X, dot);
                    }
                }
                red[(jb * P.R + rl) * nt + sg] = part;
            }
        }
        __syncthreads();
        if (s_err) break;
        for (int rl = warp; rl < P.R; rl += nwarps) {
            const int row = row0 + rl;
            if (row >= job.rows) continue;
            // segment partials summed in double, rounded once (the reference's row dot
            // is a double sum rounded to float)
            double vd = 0.0;
            for (int i = lane; i < nt; i += 32) vd += (double)red[rl * nt + i];
            float v = (float)warp_sum_d(vd);
            float u = 0.0f;
            if (P.pair) {
                double ud = 0.0;
                for (int i = lane; i < nt; i += 32) ud += (double)red[(P.R + rl) * nt + i];
                u = (float)warp_sum_d(ud);
            }
            if (lane == 0) {
                if (P.pair) {
                    // swiglu_ref (kernels/silu/swiglu_ref.cpp:41-52) on (gate, up)
                    v = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u);
                } else {
                    if (job.bias) v += job.bias[row];
                    if (job.resid) v = job.resid[row] + v;
                }
                job.y[row] = v;
                if (P.am.token && j == 0) better(bv, bi, v, row + P.am.row_offset);
            }
        }
        __syncthreads();
        if (t == 0) {
            const int pn = blockIdx.x + (i_pass + P.stages) * gridDim.x;
            if (pn < total) issue_pass(P, pn, s, bars, stage_base, s_head);
        }
    }
    if (s_err) {
        // drain every copy this CTA still has in flight before the CTA exits
        if (t == 0) {
            for (int k = 0; k < P.stages; ++k) {
                const int ii = i_pass + k;
                if (blockIdx.x + ii * gridDim.x >= total) break;
                mbar_wait(&bars[ii % P.stages], (uint32_t)(ii / P.stages) & 1u, kWaitCycles);
            }
            if (P.status) atomicExch(P.status, kDevTimeoutTma);
        }
        return;
    }
    if (P.am.token) {
        block_argmax(bv, bi, s_bv, s_bi);
        if (t == 0) {
            P.am.part_v[blockIdx.x] = bv;
            P.am.part_i[blockIdx.x] = bi;
            __threadfence();
            s_last = atomicAdd(P.am.ticket, 1u) == gridDim.x - 1;
        }
        __syncthreads();
        if (s_last) {
            __threadfence();
            bv = -INFINITY;
            bi = INT_MAX;
            for (int b = t; b < (int)gridDim.x; b += blockDim.x)
                better(bv, bi, __ldcg(P.am.part_v + b), __ldcg(P.am.part_i + b));
            block_argmax(bv, bi, s_bv, s_bi);
            if (t == 0) {
                *P.am.token = bi == INT_MAX ? P.am.row_offset : bi;
                if (P.am.value) *P.am.value = bv;
                *P.am.ticket = 0u;
            }
        }
    }
}

// Fallback for odd group sizes or unaligned bases: one warp per row, byte loads.
__global__ void i4_matvec_generic_kernel(MvParams P) {
    const int K = P.K, G = P.G;
    const int ng = (K + G - 1) / G;
    const int GB = 4 + G / 2;
    const size_t RB = (size_t)ng * GB;
    const int lane = threadIdx.x & 31;
    const int wpb = blockDim.x >> 5;
    const int total = P.pass_begin[P.n_jobs];  // one pass == one row here
    for (int p = blockIdx.x * wpb + (threadIdx.x >> 5); p < total; p += gridDim.x * wpb) {
        int j = 0;
        while (j + 1 < P.n_jobs && p >= P.pass_begin[j + 1]) ++j;
        const I4Job &job = P.job[j];
        const int row = p - P.pass_begin[j];
        const uint8_t *rp = job.w + (size_t)row * RB;
        float acc = 0.0f;
        for (int gi = lane; gi < ng; gi += 32) {
            const uint8_t *gp = rp + (size_t)gi * GB;
            const float s = h2f((uint16_t)(gp[0] | (gp[1] << 8)));
            const float z = h2f((uint16_t)(gp[2] | (gp[3] << 8)));
            const int c0 = gi * G;
            const int n = min(G, K - c0);
            float a = 0.0f, xsum = 0.0f;
            for (int i = 0; i < n; ++i) {
                const uint8_t b = gp[4 + (i >> 1)];
                const float q = (float)((i & 1) ? (b >> 4) : (b & 15));
                const float xv = P.x.src[c0 + i];
                a = fmaf(q, xv, a);
                xsum += xv;
            }
            acc += s * fmaf(-z, xsum, a);
        }
        acc = warp_sum(acc);
        if (lane == 0) {
            if (job.bias) acc += job.bias[row];
            if (job.resid) acc = job.resid[row] + acc;
            job.y[row] = acc;
        }
    }
}

// ------------------------------------------------------------------ W4A8 symmetric
// round-half-away-from-zero of clamp(x*inv, +-127), as quantize_x_i8_v3
// (kernels/matvec/matvec_i4_sdot5.cpp:60-75)
__device__ __forceinline__ int quant_x_i8(float v, float inv) {
    float t = v * inv;
    t = t > 127.0f ? 127.0f : (t < -127.0f ? -127.0f : t);
    return (int)(t >= 0.0f ? t + 0.5f : t - 0.5f);
}

template <int SEG>
__global__ void __launch_bounds__(512) i4_matvec_sym_kernel(const uint8_t *__restrict__ w,
                                                            const float *__restrict__ x,
                                                            float *__restrict__ y, int rows,
                                                            int K, int G, int nt, int S) {
    extern __shared__ float red[];
    __shared__ float s_amax[32];
    constexpr int NW = SEG / 8;
    const int t = threadIdx.x;
    const int lane = t & 31, warp = t >> 5, nwarps = blockDim.x >> 5;
    float am = 0.0f;
    for (int i = t; i < K; i += blockDim.x) am = fmaxf(am, fabsf(__ldg(x + i)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    if (lane == 0) s_amax[warp] = am;
    __syncthreads();
    if (t < 32) {
        float v = t < nwarps ? s_amax[t] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (t == 0) s_amax[0] = v;
    }
    __syncthreads();
    const float amax = s_amax[0];
    const float scale_x = amax > 0.0f ? amax / 127.0f : 1.0f;
    const float inv = 1.0f / scale_x;

    const int slot = t / nt;
    const int sg = t - slot * nt;
    const int ng = (K + G - 1) / G;
    const int GB = 4 + G / 2;
    const size_t RB = (size_t)ng * GB;
    const int spg = G / SEG;
    const int g = sg / spg;
    const int col0 = sg * SEG;
    const uint32_t hdr_off = (uint32_t)g * GB;
    const uint32_t seg_off = hdr_off + 4u + (uint32_t)(sg - g * spg) * (SEG / 2);
    const bool active = slot < S;

    uint32_t xlo[NW], xhi[NW];
    int xqsum = 0;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int ce = col0 + 8 * i + 2 * b, co = ce + 1;
            const int qe = (active && ce < K) ? quant_x_i8(__ldg(x + ce), inv) : 0;
            const int qo = (active && co < K) ? quant_x_i8(__ldg(x + co), inv) : 0;
            xqsum += qe + qo;
            lo |= ((uint32_t)qe & 0xFFu) << (8 * b);
            hi |= ((uint32_t)qo & 0xFFu) << (8 * b);
        }
        xlo[i] = lo;
        xhi[i] = hi;
    }

    for (int p = blockIdx.x; p * S < rows; p += gridDim.x) {
        const int row = p * S + slot;
        if (active && row < rows) {
            const uint8_t *rp = w + (size_t)row * RB;
            const uint32_t hv = ldg_u32(rp + hdr_off);
            int dot = 0;
#pragma unroll
            for (int i = 0; i < NW; ++i) {
                const uint32_t wd = ldg_u32(rp + seg_off + 4 * i);
                dot = dp4a_us(wd & 0x0F0F0F0Fu, xlo[i], dot);
                dot = dp4a_us((wd >> 4) & 0x0F0F0F0Fu, xhi[i], dot);
            }
            dot -= 8 * xqsum;
            const float A = h2f((uint16_t)(hv & 0xFFFFu)) * scale_x;
            red[slot * nt + sg] = A * (float)dot;
        }
        __syncthreads();
        for (int rho = warp; rho < S; rho += nwarps) {
            const int r2 = p * S + rho;
            if (r2 >= rows) continue;
            float v = 0.0f;
            for (int i = lane; i < nt; i += 32) v += red[rho * nt + i];
            v = warp_sum(v);
            if (lane == 0) y[r2] = v;
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------ dequant
__global__ void i4_dequant_kernel(const uint8_t *__restrict__ w, int rows, int dim, int G,
                                  float *__restrict__ out) {
    const int ng = (dim + G - 1) / G;
    const int GB = 4 + G / 2;
    const long total = (long)rows * ng;
    for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < total;
         idx += (long)gridDim.x * blockDim.x) {
        const int row = (int)(idx / ng), g = (int)(idx % ng);
        const uint8_t *gp = w + ((size_t)row * ng + g) * GB;
        const float s = h2f((uint16_t)(gp[0] | (gp[1] << 8)));
        const float z = h2f((uint16_t)(gp[2] | (gp[3] << 8)));
        const int c0 = g * G;
        const int n = min(G, dim - c0);
        float *o = out + (size_t)row * dim + c0;
        for (int i = 0; i < n; ++i) {
            const uint8_t b = gp[4 + (i >> 1)];
            const float q = (float)((i & 1) ? (b >> 4) : (b & 15));
            o[i] = __fmul_rn(__fsub_rn(q, z), s);
        }
    }
}

int g_num_sms = 0;
int g_math = -1;  // MATH_F32 / MATH_DP4A, from TQB200_I4_MATH (default dp4a)

int math_mode() {
    if (g_math < 0) {
        const char *e = getenv("TQB200_I4_MATH");
        g_math = (e && e[0] == 'f') ? MATH_F32 : MATH_DP4A;
    }
    return g_math;
}

struct Shape {
    int seg = 0, nt = 0, S = 0, RP = 0, R = 0, block = 0, stages = 0;
    uint32_t stage_bytes = 0;
    size_t smem = 0;
};

Shape plan(int K, int G, bool pair) {
    Shape L;
    L.seg = (G % 64 == 0) ? 64 : 32;
    const int ng = (K + G - 1) / G;
    L.nt = ng * (G / L.seg);
    if (L.nt > 512) {
        L.seg = 0;
        return L;
    }
    const size_t RB = (size_t)ng * (4 + G / 2);
    L.S = std::max(1, 256 / L.nt);
    L.block = ((L.nt * L.S + 31) / 32) * 32;
    const size_t target = 16 * 1024;
    L.RP = (int)std::max<size_t>(1, std::min<size_t>(8, (target + L.S * RB - 1) / (L.S * RB)));
    L.R = L.S * L.RP;
    const size_t region = ((size_t)L.R * RB + 32 + 127) / 128 * 128;
    L.stage_bytes = (uint32_t)(pair ? 2 * region : region);
    // one or two persistent CTAs per SM: ~96 KB of weights in flight per SM
    L.stages = (int)std::max<size_t>(2, std::min<size_t>(kMaxStages, (48 * 1024) / L.stage_bytes));
    const size_t kp = (size_t)L.nt * L.seg;
    const size_t red = (((size_t)(pair ? 2 : 1) * L.R * L.nt + 3) & ~(size_t)3);
    const size_t tables = (size_t)L.nt * 4 + 3 + 16 + (size_t)L.nt * 6 * (L.seg / 8);  // words
    L.smem = 128 + (size_t)L.stages * L.stage_bytes + (red + kp + tables) * 4;
    return L;
}

template <typename Kern>
int grid_for(Kern k, int block, size_t smem, int work) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, block, smem) != cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        per_sm = 1;
    }
    return std::max(1, std::min(work, per_sm * num_sms()));
}

template <int SEG, int MATH>
int launch_tma(const MvParams &P, const Shape &L, int passes, bool pdl, cudaStream_t st) {
    auto k = i4_mv_tma_kernel<SEG, MATH>;
    static bool attr_set = false;
    if (!attr_set) {
        TQ_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        attr_set = true;
    }
    // persistent: at most two CTAs per SM, so the x prologue is paid once per CTA
    const int grid = std::min(grid_for(k, L.block, L.smem, passes), 2 * num_sms());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(L.block);
    cfg.dynamicSmemBytes = L.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    TQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, k, P));
    return TQB200_OK;
}

}  // namespace

int num_sms() {
    if (g_num_sms == 0) {
        int dev = 0, n = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_num_sms = n > 0 ? n : 148;
    }
    return g_num_sms;
}

int i4_argmax_slots(int rows, int in_dim, int group_size) {
    (void)rows;
    (void)in_dim;
    (void)group_size;
    return 8 * num_sms();  // >= any grid the launcher picks (<= per_sm * SMs, per_sm <= 8)
}

int launch_i4_matvec_ex(const I4Job *jobs, int n_jobs, int in_dim, int group_size,
                        const I4LaunchOpts &o, cudaStream_t stream) {
    TQ_CHECK_ARG(n_jobs >= 1 && n_jobs <= 3, "n_jobs %d", n_jobs);
    TQ_CHECK_ARG(in_dim > 0 && group_size > 0 && group_size % 2 == 0,
                 "bad in_dim %d / group_size %d", in_dim, group_size);
    MvParams P{};
    P.n_jobs = n_jobs;
    P.K = in_dim;
    P.G = group_size;
    P.x = o.x;
    P.am = o.argmax;
    P.status = o.status;
    const bool pair = o.pair_swiglu;
    TQ_CHECK_ARG(!pair || (n_jobs == 2 && jobs[0].rows == jobs[1].rows && !o.argmax.token),
                 "paired SwiGLU needs two jobs with equal rows");
    const Shape L = plan(in_dim, group_size, pair);
    bool aligned = true;  // the TMA path needs 16-byte aligned matrix bases
    for (int j = 0; j < n_jobs; ++j) aligned = aligned && ((uintptr_t)jobs[j].w % 16u == 0);
    const bool fast = (group_size % 32 == 0) && L.seg != 0 && aligned;
    if (!fast) {
        TQ_CHECK_ARG(o.x.mode == X_PLAIN && !o.argmax.token && !pair,
                     "fused prologue/epilogue needs group_size %% 32 == 0 and aligned weights");
    }
    const int R = fast ? L.R : 1;
    int acc = 0;
    for (int j = 0; j < n_jobs; ++j) {
        TQ_CHECK_ARG(jobs[j].rows >= 0, "rows %d", jobs[j].rows);
        P.job[j] = jobs[j];
        P.pass_begin[j] = acc;
        if (!pair || j == 0) acc += (jobs[j].rows + R - 1) / R;
    }
    P.pass_begin[n_jobs] = acc;
    P.pair = pair ? 1 : 0;
    if (acc == 0) return TQB200_OK;
    if (fast) {
        P.nt = L.nt;
        P.S = L.S;
        P.RP = L.RP;
        P.R = L.R;
        P.stages = L.stages;
        P.stage_bytes = L.stage_bytes;
        const bool dp4a = math_mode() == MATH_DP4A;
        if (L.seg == 64)
            return dp4a ? launch_tma<64, MATH_DP4A>(P, L, acc, o.pdl, stream)
                        : launch_tma<64, MATH_F32>(P, L, acc, o.pdl, stream);
        return dp4a ? launch_tma<32, MATH_DP4A>(P, L, acc, o.pdl, stream)
                    : launch_tma<32, MATH_F32>(P, L, acc, o.pdl, stream);
    }
    const int grid = std::max(1, std::min((acc + 7) / 8, num_sms() * 8));
    i4_matvec_generic_kernel<<<grid, 256, 0, stream>>>(P);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_i4_matvec(const I4Job *jobs, int n_jobs, const float *x, int in_dim, int group_size,
                     cudaStream_t stream) {
    I4LaunchOpts o;
    o.x.mode = X_PLAIN;
    o.x.src = x;
    return launch_i4_matvec_ex(jobs, n_jobs, in_dim, group_size, o, stream);
}

int launch_i4_matvec_sym(const uint8_t *w, const float *x, float *y, int rows, int in_dim,
                         int group_size, cudaStream_t stream) {
    TQ_CHECK_ARG(in_dim > 0 && group_size > 0 && group_size % 32 == 0,
                 "symmetric W4A8 path needs group_size %% 32 == 0 (got %d)", group_size);
    TQ_CHECK_ARG((uintptr_t)w % 4u == 0, "symmetric W4A8 path needs 4-byte aligned weights");
    if (rows == 0) return TQB200_OK;
    const int seg = (group_size % 64 == 0) ? 64 : 32;
    const int nt = ((in_dim + group_size - 1) / group_size) * (group_size / seg);
    TQ_CHECK_ARG(nt <= 512, "in_dim %d too large", in_dim);
    const int S = std::max(1, 384 / nt);
    const int block = ((nt * S + 31) / 32) * 32;
    const size_t smem = (size_t)S * nt * sizeof(float);
    const int passes = (rows + S - 1) / S;
    if (seg == 64) {
        auto k = i4_matvec_sym_kernel<64>;
        k<<<grid_for(k, block, smem, passes), block, smem, stream>>>(w, x, y, rows, in_dim,
                                                                     group_size, nt, S);
    } else {
        auto k = i4_matvec_sym_kernel<32>;
        k<<<grid_for(k, block, smem, passes), block, smem, stream>>>(w, x, y, rows, in_dim,
                                                                     group_size, nt, S);
    }
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_i4_dequant(const uint8_t *w, int rows, int dim, int group_size, float *out,
                      cudaStream_t stream) {
    TQ_CHECK_ARG(rows >= 0 && dim > 0 && group_size > 0 && group_size % 2 == 0,
                 "bad dequant shape");
    if (rows == 0) return TQB200_OK;
    const long total = (long)rows * ((dim + group_size - 1) / group_size);
    const int block = 256;
    const int grid = (int)std::min<long>((total + block - 1) / block, (long)num_sms() * 16);
    i4_dequant_kernel<<<grid, block, 0, stream>>>(w, rows, dim, group_size, out);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

}  // namespace tqb200
