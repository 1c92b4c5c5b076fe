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
//  * Warp 0 is the producer (one lane issues the copies and refills a stage once
//    every consumer warp has arrived on its "empty" mbarrier); consumer thread
//    (slot, seg) owns one SEG-column segment (SEG = 32 or 64, dividing G) of
//    rows slot, slot+S, ... of every pass.  512 threads, one CTA per SM.
//  * Math: activations split into three int8 digits with one scale for the
//    whole vector (x ~ (d0 + d1/254 + d2/254^2) * max|x|/127, error
//    <= 6.1e-8 * max|x|; a fourth digit, error / 254, when most of the values
//    lie below max/64: outlier channels), built once per CTA from
//    activations held in registers, and the nibble dots run as exact integer
//    dp4a (two masks, no shift: high nibbles enter as 16x bytes; 6 dp4a per 8
//    weights, 8 with the fourth digit, independent accumulators), using
//        sum_i (q_i - z) s x_i = s * (sum_i q_i x_i - z * sum_i x_i).
//    A pass needs one named barrier among the consumers (partials are
//    double-buffered); a row's segment partials are summed by one lane, and the
//    bias / residual of its rows are fetched before the weights are waited on.
//  * Optional fused prologues (RMSNorm of the source, SwiGLU of gate/up) and
//    epilogues (bias, residual add, greedy argmax over the rows).
//  * Every mbarrier wait is bounded; on timeout the kernel records an error
//    word, drains its outstanding copies (again bounded) and returns.
// Accumulation is fp32 (the reference accumulates in double); results agree
// to ~1e-6 relative, inside the 1e-4 max-relative tolerance of the tests.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace tqb200 {

namespace {

constexpr int kMaxStages = 8;

struct MvParams {
    I4Job job[3];
    int pass_begin[4];
    int n_jobs;
    int K, G, nt, S, RP, R;
    int stages;
    uint32_t stage_bytes;
    int pair;  // jobs 0 and 1 (gate, up) share passes; y0 = silu(W0 x) * (W1 x)
    int x_bulk;  // activation vectors 16-byte aligned with K % 4 == 0: one bulk copy each
    XSource x;
    ArgmaxOut am;
    int *status;
    // MoE experts.  Expert mode (eidx != nullptr): the rows of job j form nslots blocks
    // of erows rows, block b being expert eidx[b] at job.w + eidx[b] * estride (passes
    // never straddle blocks: R divides erows); eidx[b] == -1 marks another rank's expert
    // (expert parallelism): its block is neither staged nor written.  Slot mode (nslots > 0 with xslots):
    // CTA c serves block c % nslots only, with x = x.src + (c % nslots) * K.
    const int *eidx;
    long long estride;
    int erows, nslots, n_experts;
    int xslots;
    Stamp stamp;  // in-graph timeline (off unless the engine records one)
    const XWait *xw;  // tensor parallelism (device descriptors, XCHG instance only): x's
    const XPut *xp;   // exchange before reading x; written rows also to every peer
};

// Pass index of a CTA's i-th pass (>= total when it has none).
__device__ __forceinline__ int pass_of(const MvParams &P, int i) {
    if (!P.xslots) return blockIdx.x + i * gridDim.x;
    const int nsub = gridDim.x / P.nslots;
    const int slot = blockIdx.x % P.nslots, sub = blockIdx.x / P.nslots;
    const int pps = P.erows / P.R;
    const int pl = sub + i * nsub;
    return (pl < pps && sub < nsub) ? slot * pps + pl : INT_MAX;
}

// Reciprocal to about one ulp (the digit planes below need no exact quotient).
__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
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
    const uint8_t *base = job.w;
    int rows_end = job.rows;
    bool skip = false;
    if (P.eidx) {  // the block's expert: rows relative to its own matrix
        const int blk = row0 / P.erows;
        int e = P.eidx[blk];
        if (e == -1) {  // another rank's expert (expert parallelism): nothing to stage
            skip = true;
            e = 0;
        } else if (e < 0 || e >= P.n_experts) {  // self-check: never read outside the experts
            if (P.status) atomicExch(P.status, kDevBadExpert);
            e = 0;
        }
        base = job.w + (size_t)e * (size_t)P.estride;
        row0 -= blk * P.erows;
        row1 -= blk * P.erows;
        rows_end = P.erows;
    }
    const uintptr_t a = (uintptr_t)(base + (size_t)row0 * RB);
    uintptr_t b = (uintptr_t)(base + (size_t)row1 * RB);
    const uintptr_t mat_end16 = (uintptr_t)(base + (size_t)rows_end * RB) & ~(uintptr_t)15;
    const uintptr_t a16 = a & ~(uintptr_t)15;
    uintptr_t b16 = (b + 15) & ~(uintptr_t)15;
    if (b16 > mat_end16) b16 = mat_end16;
    if (b16 < a16) b16 = a16;
    uint32_t bytes = (uint32_t)(b16 - a16);
    if (skip) {
        bytes = 0;
        b = a16;
    }
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
    // pieces of <= 16 KB: one bulk copy is fetched at a limited rate per SM, several in
    // flight reach the full rate
    constexpr uint32_t kPiece = 16384;
    for (uint32_t o = 0; o < b0; o += kPiece) bulk_g2s(dst + o, src0 + o, min(kPiece, b0 - o), &bars[s]);
    for (uint32_t o = 0; o < b1; o += kPiece)
        bulk_g2s(dst + cap + o, src1 + o, min(kPiece, b1 - o), &bars[s]);
}

constexpr int kBarBytes = 256;  // 2*kMaxStages + 2 mbarriers, rounded up

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier 1 over the consumer warps, returning the OR of `pred` across them
// (uniform: every consumer thread gets the same answer).
__device__ __forceinline__ bool consumer_sync_or(int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.or.pred p, 1, %2, q;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(nthreads)
        : "memory");
    return r != 0;
}

// Sum of n segment partials (four interleaved fp32 accumulators; n <= 480 partials
// of a row whose terms are already dp4a-exact per segment, so the sum's rounding error
// stays near 1e-6 relative, far inside the 1e-4 bound).
__device__ __forceinline__ float row_sum(const float *p, int n) {
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    int i = 0;
    for (; i + 4 <= n; i += 4) {
        a0 += p[i];
        a1 += p[i + 1];
        a2 += p[i + 2];
        a3 += p[i + 3];
    }
    for (; i < n; ++i) a0 += p[i];
    return (a0 + a1) + (a2 + a3);
}

// dp4a digit planes of one segment: 6 words per 8 columns, then 4 words of padding
// (a row stride of 6*NW+4 words keeps the 16-byte loads of 8 consecutive segments on
// distinct bank groups)
template <int NW> struct DigitLayout { static constexpr int stride = 6 * NW + 4; };

constexpr int kI4Threads = 512;  // producer warp + 15 consumer warps, one CTA per SM
constexpr int kI4MaxItems = 3;   // 8-column activation chunks per thread (K <= 12288)

template <int SEG, bool STAMP, bool XCHG>
__global__ void __launch_bounds__(kI4Threads, 1) i4_mv_tma_kernel(const __grid_constant__ MvParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NW = SEG / 8;
    constexpr int DS = DigitLayout<NW>::stride;
    const int t = threadIdx.x;
    const int lane = t & 31, warp = t >> 5;
    const int total = P.pass_begin[P.n_jobs];
    const int nt = P.nt, S = P.S, K = P.K, G = P.G, np = 1 + P.pair;
    const int KP = nt * SEG;  // every column a segment can own (>= K), a multiple of 32
    const int ncw = (int)(blockDim.x >> 5) - 1;  // consumer warps (warp 0 is the producer)
    const bool norm = P.x.mode == X_RMSNORM, swiglu = P.x.mode == X_SWIGLU;
    // shared memory: barriers | weight stages | red x2 | digit planes [nt][DS] |
    // 8-column chunk sums | RMSNorm weight (norm mode only)
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);  // [kMaxStages] weights landed
    uint64_t *empty = full + kMaxStages;                   // [kMaxStages] stage consumed
    uint64_t *wbar = full + 2 * kMaxStages;                // norm-weight copy
    uint8_t *stage_base = smem + kBarBytes;
    float *red = reinterpret_cast<float *>(stage_base + (size_t)P.stages * P.stage_bytes);
    const int ntp = nt + 1;  // partial-row stride (odd: conflict-free per-lane row sums)
    const size_t red_n = (size_t)np * P.R * ntp;  // one buffer
    uint32_t *dig = reinterpret_cast<uint32_t *>(red + ((2 * red_n + 3) & ~(size_t)3));
    float *csum = reinterpret_cast<float *>(dig + (size_t)DS * nt);
    float *wsm = csum + (((size_t)KP / 8 + 3) & ~(size_t)3);
    __shared__ uint32_t s_head[2 * kMaxStages];
    __shared__ int s_err, s_issued;  // s_issued: passes whose copies were issued
    __shared__ double s_rd[32];
    __shared__ float s_am[32];
    __shared__ float s_bv[32];
    __shared__ int s_bi[32];
    __shared__ bool s_last;
    const bool bulk_x = P.x_bulk != 0;
    StampRegs stamp_r;
    stamp_enter<STAMP>(P.stamp, stamp_r);

    if (t == 0) {
        for (int s = 0; s < P.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ncw);
        }
        mbar_init(wbar, 1);
        fence_mbar_init();
        s_err = 0;
        s_issued = 0;
        if (!P.eidx) {  // constant weights: before the dependency wait
            for (int s = 0; s < P.stages; ++s) {
                const int p = pass_of(P, s);
                if (p < total) {
                    issue_pass(P, p, s, full, stage_base, s_head);
                    s_issued = s + 1;
                }
            }
        }
        if (bulk_x && norm) {  // constant weights: before the dependency wait
            mbar_arrive_expect_tx(wbar, (uint32_t)K * 4u);
            bulk_g2s(wsm, P.x.norm_w, (uint32_t)K * 4u, wbar);
        }
    }
    __syncthreads();  // barrier initialisation visible to every thread
    // weights are in flight; now wait for the producer of x and let our dependents start
    stamp_step<STAMP>(P.stamp, stamp_r);
    griddep_wait();
    stamp_waited<STAMP>(P.stamp, stamp_r);
    griddep_launch();
    if (P.eidx && t == 0) {  // expert weights: which ones is known only now
        for (int s = 0; s < P.stages; ++s) {
            const int p = pass_of(P, s);
            if (p < total) {
                issue_pass(P, p, s, full, stage_base, s_head);
                s_issued = s + 1;
            }
        }
    }
    // x gathered from the peers (tensor parallelism): their rows have landed
    if constexpr (XCHG)
        if (P.xw) xwait(*P.xw, P.status);
    // this CTA's activation vector (slot mode: its block's own)
    const float *xsrc = P.x.src + (P.xslots ? (size_t)(blockIdx.x % P.nslots) * K : 0);

    // ---- activation, 8-column chunks c = t, t + blockDim, ... held in registers: one
    // round of 16-byte loads (unaligned sources: scalar loads), SwiGLU applied, the sum
    // of squares (RMSNorm, in double as rmsnorm_ref) and max |value| for the digit scale
    const int nchunks = KP / 8;
    float xv[kI4MaxItems][8];
#pragma unroll
    for (int it = 0; it < kI4MaxItems; ++it) {
        const int c = t + it * (int)blockDim.x;
#pragma unroll
        for (int k = 0; k < 8; ++k) xv[it][k] = 0.0f;
        if (c >= nchunks) continue;
        if (bulk_x && 8 * c + 8 <= K) {
            const float4 *s4 = reinterpret_cast<const float4 *>(xsrc) + 2 * c;
            const float4 a = s4[0], b = s4[1];
            xv[it][0] = a.x, xv[it][1] = a.y, xv[it][2] = a.z, xv[it][3] = a.w;
            xv[it][4] = b.x, xv[it][5] = b.y, xv[it][6] = b.z, xv[it][7] = b.w;
            if (swiglu) {
                const float4 *u4 = reinterpret_cast<const float4 *>(P.x.up) + 2 * c;
                const float4 ua = u4[0], ub = u4[1];
                const float u[8] = {ua.x, ua.y, ua.z, ua.w, ub.x, ub.y, ub.z, ub.w};
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float g = xv[it][k];
                    xv[it][k] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u[k]);
                }
            }
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int i = 8 * c + k;
                if (i < K) {
                    float v = xsrc[i];
                    if (swiglu) v = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), P.x.up[i]);
                    xv[it][k] = v;
                }
            }
        }
    }
    if (norm) {
        if (bulk_x) {
            if (t == 0 && !mbar_wait(wbar, 0, kWaitCycles)) s_err = 1;
        } else {
            for (int i = t; i < K; i += blockDim.x) wsm[i] = P.x.norm_w[i];
        }
        __syncthreads();  // norm weights in shared memory
    }
    // pass A: max |value| (under RMSNorm, of x * w: the RMSNorm scale is common to all
    // columns) and the RMSNorm sum of squares in double as rmsnorm_ref; block-reduced
    // (one barrier)
    float am_mine = 0.0f;  // this thread's own max
    {
        double ss = 0.0;
        float am = 0.0f;
#pragma unroll
        for (int it = 0; it < kI4MaxItems; ++it) {
            const int c = t + it * (int)blockDim.x;
            if (c >= nchunks) continue;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float v = xv[it][k];
                float a = v;
                if (norm) {
                    ss += (double)v * (double)v;
                    a = v * (8 * c + k < K ? wsm[8 * c + k] : 0.0f);
                }
                am = fmaxf(am, fabsf(a));
            }
        }
        am_mine = am;
        if (norm) ss = warp_sum_d(ss);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        if (lane == 0) {
            s_rd[warp] = ss;
            s_am[warp] = am;
        }
    }
    __syncthreads();
    float rms_scale = 1.0f, amax = 0.0f;
    {  // the warps' partials, reduced across a warp's lanes (every warp, no extra barrier)
        const int nwp = (int)(blockDim.x >> 5);
        double tot = lane < nwp ? s_rd[lane] : 0.0;
        amax = lane < nwp ? s_am[lane] : 0.0f;
        if (norm) tot = warp_sum_d(tot);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (norm) {
            const float mean_sq = (float)(tot / K);
            rms_scale = 1.0f / sqrtf(__fadd_rn(mean_sq, P.x.eps));
        }
    }
    // three digits leave an error of up to 6.1e-8 of max |x| in every element; when the
    // max stands far out of the bulk of the vector (outlier channels), that is coarse for
    // the bulk, and a fourth digit (error / 254) is kept: when fewer than half of the
    // threads holding activations see a value above max/64 among their own (one counting
    // barrier; the choice is uniform over the CTA)
    const int holders = min((int)blockDim.x, nchunks);
    const bool four = 2 * __syncthreads_count(t < holders && am_mine * 64.0f > amax) < holders;
    if (norm) amax = amax * rms_scale * 1.0000005f;  // bound on |(x*r)*w| after rounding
    // pass B, per chunk: RMSNorm applied, the chunk sum, and the dp4a digit planes of
    // the vector with ONE scale for all of it:
    //   x ~ (d0 + d1/254 + d2/254^2 [+ d3/254^3]) * s0,  s0 = max|x| / 127;
    // word order per chunk (lo, hi) x (d0, d1, d2), lo = even columns, hi = odd ones,
    // matching the nibble order of a weight word (the fourth digit's lo, hi words in a
    // plane of their own).  Rounding to the nearest integer uses the 1.5*2^23 trick (one
    // FFMA; the digit's byte is the low byte of the sum's bits), so no float/int
    // conversions; |digit| <= 127 by construction (any s0 >= max|x| / 127 to within a
    // few ulp keeps every digit within +-127).  Approximate reciprocals suffice: a digit
    // is round(r * i) of the residual r the digits before it left, so an i off by an ulp
    // moves |digit| by ~1e-5 (never past 127.5) and the next digit absorbs the rest.
    const float dsc0 = amax > 0.0f ? amax * (1.0f / 127.0f) : 1.0f;
    const float dsc1 = dsc0 * (1.0f / 254.0f), dsc2 = dsc1 * (1.0f / 254.0f);
    const float dsc3 = four ? dsc2 * (1.0f / 254.0f) : 0.0f;
    uint2 d3w[kI4MaxItems];  // fourth digit (lo, hi words) of this thread's chunks
    {
        constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
        const float i0 = rcp_approx(dsc0), i1 = i0 * 254.0f, i2 = i1 * 254.0f, i3 = i2 * 254.0f;
#pragma unroll
        for (int it = 0; it < kI4MaxItems; ++it) {
            const int c = t + it * (int)blockDim.x;
            if (c >= nchunks) continue;
            float v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                v[k] = xv[it][k];
                if (norm)
                    v[k] = 8 * c + k < K ? __fmul_rn(__fmul_rn(v[k], rms_scale), wsm[8 * c + k]) : 0.0f;
            }
            csum[c] = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
            uint32_t d0[8], d1[8], d2[8];  // digit k of each column, in the low byte
            float r2s[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float t0 = fmaf(v[k], i0, kRound);
                const float r1 = fmaf(-(t0 - kRound), dsc0, v[k]);
                const float t1 = fmaf(r1, i1, kRound);
                const float r2 = fmaf(-(t1 - kRound), dsc1, r1);
                const float t2 = fmaf(r2, i2, kRound);
                d0[k] = __float_as_uint(t0);
                d1[k] = __float_as_uint(t1);
                d2[k] = __float_as_uint(t2);
                r2s[k] = r2;
            }
            // low bytes of columns (0,2,4,6) -> lo word, (1,3,5,7) -> hi word
            auto pack = [](const uint32_t *d, int o) {
                const uint32_t a = __byte_perm(d[o], d[o + 2], 0x0040);
                const uint32_t b = __byte_perm(d[o + 4], d[o + 6], 0x0040);
                return __byte_perm(a, b, 0x5410);
            };
            const uint32_t wd[6] = {pack(d0, 0), pack(d0, 1), pack(d1, 0),
                                    pack(d1, 1), pack(d2, 0), pack(d2, 1)};
            const int sgi = c / NW, ci = c - sgi * NW;
            uint2 *dst = reinterpret_cast<uint2 *>(dig + (size_t)sgi * DS + 6 * ci);
            dst[0] = make_uint2(wd[0], wd[1]);
            dst[1] = make_uint2(wd[2], wd[3]);
            dst[2] = make_uint2(wd[4], wd[5]);
            if (four) {
                uint32_t d3[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float r3 = fmaf(-(__uint_as_float(d2[k]) - kRound), dsc2, r2s[k]);
                    d3[k] = __float_as_uint(fmaf(r3, i3, kRound));
                }
                d3w[it] = make_uint2(pack(d3, 0), pack(d3, 1));
            }
        }
    }
    __syncthreads();

    // consumer thread (slot, sg) of warps 1.. holds its segment's digit words in
    // registers for the whole kernel
    const int tc = t - 32;
    const int slot = tc / nt;
    const int sg = tc - slot * nt;
    const bool active = warp > 0 && slot < S;
    float X = 0.0f;  // segment sum (zero-point term)
    uint32_t xd[6 * NW];
    if (active) {
#pragma unroll
        for (int ci = 0; ci < NW; ++ci) X += csum[sg * NW + ci];
        const uint4 *src = reinterpret_cast<const uint4 *>(dig + (size_t)sg * DS);
#pragma unroll
        for (int w = 0; w < 6 * NW / 4; ++w) {
            const uint4 v4 = src[w];
            xd[4 * w + 0] = v4.x, xd[4 * w + 1] = v4.y, xd[4 * w + 2] = v4.z, xd[4 * w + 3] = v4.w;
        }
    }
    // outlier channels: with the first three digits in registers the digit rows are free,
    // and the fourth digit plane goes there (2 words per chunk, segment sg at 2 NW sg),
    // so it costs no shared memory beyond the three-digit layout
    uint2 *dig3 = reinterpret_cast<uint2 *>(dig);
    if (four) {
        __syncthreads();
#pragma unroll
        for (int it = 0; it < kI4MaxItems; ++it) {
            const int c = t + it * (int)blockDim.x;
            if (c < nchunks) dig3[c] = d3w[it];
        }
        __syncthreads();
    }

    float bv = -INFINITY;
    int bi = INT_MAX;
    bool c_err = false;  // consumer-side error (uniform across consumers)
    if (warp == 0) {
        // ---- producer: refill stage s with pass i once every consumer warp is done
        // with pass i - stages there
        if (lane == 0) {
            for (int i = P.stages;; ++i) {
                const int p = pass_of(P, i);
                if (p >= total) break;
                const int s = i % P.stages;
                if (!mbar_wait(&empty[s], (uint32_t)(i / P.stages - 1) & 1u, kWaitCycles)) {
                    s_err = 1;
                    break;
                }
                issue_pass(P, p, s, full, stage_base, s_head);
                s_issued = i + 1;
            }
        }
    } else {
        // ---- consumers: thread (slot, seg) over the rows of every pass
        const int cw = warp - 1;
        const int GB = 4 + G / 2;
        const size_t RB = (size_t)((K + G - 1) / G) * GB;
        const int spg = G / SEG;
        const int g = sg / spg;
        const uint32_t hdr_off = (uint32_t)g * GB;
        const uint32_t seg_off = hdr_off + 4u + (uint32_t)(sg - g * spg) * (SEG / 2);
        const int ncons = ncw * 32;
        // this thread's rows of a full pass: slot, slot + S, ... below R (the same in every
        // pass); row pointers and partial slots advance by fixed strides
        const int my_rows = active ? (P.R - slot + S - 1) / S : 0;
        const size_t rstride = (size_t)S * RB;
        const int pstride = S * ntp;
        // one row's segment partial from its bytes in the stage
        auto seg_part = [&](const uint8_t *rp, auto four_c) -> float {
            constexpr bool kFour = decltype(four_c)::value;
            const uint32_t hv = lds_u32(rp + hdr_off);
            const float sc = h2f((uint16_t)(hv & 0xFFFFu));
            const float zr = h2f((uint16_t)(hv >> 16));
            // low nibbles as bytes, high nibbles as 16x bytes (one mask each, no shift): six
            // independent accumulators, the high ones scaled back by 16
            int L0 = 0, L1 = 0, L2 = 0, H0 = 0, H1 = 0, H2 = 0;
            float dot3 = 0.0f;
            if constexpr (!kFour) {
#pragma unroll
                for (int i = 0; i < NW; ++i) {
                    const uint32_t wd = lds_u32(rp + seg_off + 4 * i);
                    const uint32_t lo = wd & 0x0F0F0F0Fu, hi = wd & 0xF0F0F0F0u;
                    L0 = dp4a_us(lo, xd[6 * i + 0], L0);
                    H0 = dp4a_us(hi, xd[6 * i + 1], H0);
                    L1 = dp4a_us(lo, xd[6 * i + 2], L1);
                    H1 = dp4a_us(hi, xd[6 * i + 3], H1);
                    L2 = dp4a_us(lo, xd[6 * i + 4], L2);
                    H2 = dp4a_us(hi, xd[6 * i + 5], H2);
                }
            } else {  // outlier channels: the fourth digit plane from shared memory
                int L3 = 0, H3 = 0;
                const uint2 *x3 = dig3 + (size_t)sg * NW;
#pragma unroll
                for (int i = 0; i < NW; ++i) {
                    const uint32_t wd = lds_u32(rp + seg_off + 4 * i);
                    const uint32_t lo = wd & 0x0F0F0F0Fu, hi = wd & 0xF0F0F0F0u;
                    const uint2 d3 = x3[i];
                    L0 = dp4a_us(lo, xd[6 * i + 0], L0);
                    H0 = dp4a_us(hi, xd[6 * i + 1], H0);
                    L1 = dp4a_us(lo, xd[6 * i + 2], L1);
                    H1 = dp4a_us(hi, xd[6 * i + 3], H1);
                    L2 = dp4a_us(lo, xd[6 * i + 4], L2);
                    H2 = dp4a_us(hi, xd[6 * i + 5], H2);
                    L3 = dp4a_us(lo, d3.x, L3);
                    H3 = dp4a_us(hi, d3.y, H3);
                }
                dot3 = (float)(L3 + (H3 >> 4)) * dsc3;
            }
            const int D0 = L0 + (H0 >> 4), D1 = L1 + (H1 >> 4), D2 = L2 + (H2 >> 4);
            const float dot = fmaf((float)D0, dsc0, fmaf((float)D1, dsc1, fmaf((float)D2, dsc2, dot3)));
            return sc * fmaf(-zr, X, dot);
        };
        // the pass loop, compiled twice: with and without the fourth digit plane (the
        // choice is uniform over the CTA, so each thread runs one straight-line version).
        // Per pass: stage s and its phase, and the consumer warp that reduces the pass's
        // first chunk of 32 rows (chunk c goes to warp (first + c) mod ncw, so the
        // reductions of consecutive passes spread over the warps), all advanced
        // incrementally; the pass's job index only grows.
        auto passes = [&](auto four_c) {
            int s = 0, first = 0, j = 0;
            uint32_t parity = 0;
            for (int i_pass = 0;; ++i_pass) {
                const int p = pass_of(P, i_pass);
                if (p >= total) break;
                while (j + 1 < P.n_jobs && p >= P.pass_begin[j + 1]) ++j;
                const I4Job &job = P.job[j];
                const int row0 = (p - P.pass_begin[j]) * P.R;
                const int rows_here = min(P.R, job.rows - row0);  // a job's last pass may be short
                float *rb = red + (size_t)(i_pass & 1) * red_n;  // double-buffered partials
                // bias / residual of the rows this warp reduces (below), fetched before the
                // weight wait
                float pre_b0 = 0.0f, pre_b1 = 0.0f, pre_r0 = 0.0f, pre_r1 = 0.0f;
                if (!P.pair && (job.bias || job.resid)) {
                    for (int c = 0, k = 0, w = first; c * 32 < rows_here && k < 2; ++c) {
                        if (w == cw) {
                            const int row = row0 + c * 32 + lane;
                            if (c * 32 + lane < rows_here) {
                                const float b = job.bias ? job.bias[row] : 0.0f;
                                const float r = job.resid ? job.resid[row] : 0.0f;
                                if (k == 0) pre_b0 = b, pre_r0 = r;
                                else pre_b1 = b, pre_r1 = r;
                            }
                            ++k;
                        }
                        if (++w == ncw) w = 0;
                    }
                }
                const bool ok = mbar_wait(&full[s], parity, kWaitCycles);
                if (active && ok) {
                    // rows slot, slot+S, ... of each job; two at a time for independent chains
                    const int n = rows_here == P.R ? my_rows
                                                   : (rows_here > slot ? (rows_here - slot + S - 1) / S : 0);
                    const uint8_t *stage = stage_base + (size_t)s * P.stage_bytes;
                    for (int jb = 0; jb < np; ++jb) {
                        const uint8_t *rp = stage + (jb ? P.stage_bytes / 2 + s_head[kMaxStages + s]
                                                        : s_head[s]) +
                                            (size_t)slot * RB;
                        float *pp = rb + (size_t)(jb * P.R + slot) * ntp + sg;
                        int r = 0;
                        for (; r + 2 <= n; r += 2) {
                            const float p0 = seg_part(rp, four_c);
                            const float p1 = seg_part(rp + rstride, four_c);
                            pp[0] = p0;
                            pp[pstride] = p1;
                            rp += 2 * rstride;
                            pp += 2 * pstride;
                        }
                        if (r < n) pp[0] = seg_part(rp, four_c);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with stage s
                // partials of this pass complete; an error anywhere stops every consumer
                if (consumer_sync_or(ncons, !ok)) {
                    c_err = true;
                    break;
                }
                // rows of this pass, 32 per warp (a lane per row): the row's segment partials
                // summed by one lane
                for (int c = 0, k = 0, w = first; c * 32 < rows_here; ++c) {
                    const bool mine = w == cw;
                    if (++w == ncw) w = 0;
                    if (!mine) continue;
                    const int kk = k++;
                    const int rl = c * 32 + lane, row = row0 + rl;
                    if (rl >= rows_here) continue;
                    float v = row_sum(rb + (size_t)rl * ntp, nt);
                    if (P.pair) {
                        const float u = row_sum(rb + (size_t)(P.R + rl) * ntp, nt);
                        // swiglu_ref (kernels/silu/swiglu_ref.cpp:41-52) on (gate, up)
                        v = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u);
                    } else {
                        const float b_ = kk == 0 ? pre_b0 : kk == 1 ? pre_b1 : (job.bias ? job.bias[row] : 0.0f);
                        const float r_ = kk == 0 ? pre_r0 : kk == 1 ? pre_r1 : (job.resid ? job.resid[row] : 0.0f);
                        if (job.bias) v += b_;
                        if (job.resid) v = r_ + v;
                    }
                    if (P.eidx && P.eidx[row / P.erows] == -1) continue;  // another rank's expert
                    if constexpr (XCHG) {
                        if (P.xp) xput_val(*P.xp, job.y + row, v);
                        else job.y[row] = v;
                    } else {
                        job.y[row] = v;
                    }
                    if (P.am.token && j == 0) better(bv, bi, v, row + P.am.row_offset);
                }
                if (++s == P.stages) s = 0, parity ^= 1u;
                if (++first == ncw) first = 0;
            }
        };
        if (four)
            passes(std::true_type{});
        else
            passes(std::false_type{});
    }
    if (c_err && t == 32) s_err = 1;
    __syncthreads();  // producer and consumers done
    if (s_err) {
        // drain the copies this CTA may still have in flight (the most recent pass of
        // every stage), report, exit
        if (t == 0) {
            const int issued = s_issued;
            for (int i = max(0, issued - P.stages); i < issued; ++i)
                mbar_wait(&full[i % P.stages], (uint32_t)(i / P.stages) & 1u, kWaitCycles);
            if (bulk_x && norm) mbar_wait(wbar, 0, kWaitCycles);
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
                const int tok = bi == INT_MAX ? P.am.row_offset : bi;
                if constexpr (XCHG) {
                    if (P.xp) {
                        xput_val(*P.xp, P.am.token, tok);
                        if (P.am.value) xput_val(*P.xp, P.am.value, bv);
                    } else {
                        *P.am.token = tok;
                        if (P.am.value) *P.am.value = bv;
                    }
                } else {
                    *P.am.token = tok;
                    if (P.am.value) *P.am.value = bv;
                }
                *P.am.ticket = 0u;
            }
        }
    }
    if constexpr (XCHG)
        if (P.xp) xput_arrive(*P.xp);
    stamp_exit<STAMP>(P.stamp, stamp_r);
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
struct Shape {
    int seg = 0, nt = 0, S = 0, RP = 0, R = 0, block = 0, stages = 0;
    uint32_t stage_bytes = 0;
    size_t smem = 0;
};

// Launch shape.  One CTA per SM (512 threads: the producer warp and S row slots of
// nt segment threads; the block takes the whole register file).  A pass is R
// consecutive rows, one bulk copy (two in paired mode; copies split in 16 KB pieces),
// R = rows / SMs (one pass) or half of it (two passes), through a ring of up to
// ~200 KB, all in flight.
Shape plan(int K, int G, bool pair, bool norm, int rows_total, int r_div = 0) {
    Shape L;
    L.seg = (G % 64 == 0) ? 64 : 32;
    const int ng = (K + G - 1) / G;
    L.nt = ng * (G / L.seg);
    const int consumers = kI4Threads - 32;
    const size_t kp = (size_t)L.nt * L.seg;
    if (L.nt > consumers || kp / 8 > (size_t)kI4Threads * kI4MaxItems) {
        L.seg = 0;  // the generic kernel
        return L;
    }
    const size_t RB = (size_t)ng * (4 + G / 2);
    const int np = pair ? 2 : 1;
    L.S = std::max(1, consumers / L.nt);
    L.block = kI4Threads;
    const int per_cta = std::max(1, (rows_total + num_sms() - 1) / num_sms());
    // A pass costs a consumer barrier and a reduction, so a CTA's share of up to 100 KB
    // is one pass; larger shares go in at least three passes of at most 80 KB (the first
    // lands sooner and the later ones stream while it is computed; measured against two
    // passes of 96 KB, four of 48 KB and 64 KB single passes on the Qwen3-4B decode step).
    if ((size_t)per_cta * RB * np <= 100 * 1024) {
        L.R = per_cta;
    } else {
        const size_t cap = 80 * 1024 / (RB * np);
        L.R = (int)std::max<size_t>(1, std::min<size_t>((per_cta + 2) / 3, cap));
        // a multiple of the slots S: every consumer thread then has the same number of
        // rows in a pass and no warp idles at the pass barrier (rounded up while a pass
        // stays within the 80 KB, else down)
        if (L.R > L.S) {
            const int up = (L.R + L.S - 1) / L.S * L.S;
            L.R = (size_t)up <= cap ? up : L.R / L.S * L.S;
        }
    }
    if (r_div > 0) {  // passes must not straddle r_div-row blocks
        L.R = std::min(L.R, r_div);
        while (r_div % L.R) --L.R;
    }
    L.RP = (L.R + L.S - 1) / L.S;
    const size_t region = ((size_t)L.R * RB + 32 + 127) / 128 * 128;
    L.stage_bytes = (uint32_t)(np * region);
    const size_t red = ((2 * (size_t)np * L.R * (L.nt + 1) + 3) & ~(size_t)3);
    const size_t dig = (size_t)L.nt * (6 * (L.seg / 8) + 4);
    const size_t csum = (kp / 8 + 3) & ~(size_t)3;
    const size_t wsm = norm ? (((size_t)K + 3) & ~(size_t)3) : 0;
    const size_t fixed = kBarBytes + (red + dig + csum + wsm) * 4;
    const size_t cap = 200 * 1024;
    const size_t ring = cap > fixed ? cap - fixed : 0;
    L.stages = (int)std::min<size_t>(kMaxStages, ring / L.stage_bytes);
    const int passes_per_cta =
        (int)(((size_t)(rows_total + L.R - 1) / L.R + num_sms() - 1) / num_sms());
    L.stages = std::min(L.stages, passes_per_cta);
    L.smem = fixed + (size_t)std::max(1, L.stages) * L.stage_bytes;
    if (L.stages < 1) L.seg = 0;  // no TMA shape: the generic kernel
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

template <int SEG, bool STAMP, bool XCHG>
int launch_tma(const MvParams &P, const Shape &L, int passes, bool pdl, cudaStream_t st,
               int grid_fixed = 0) {
    auto k = i4_mv_tma_kernel<SEG, STAMP, XCHG>;
    static KernelSmem attr_set;
    int smem_max = 0;
    TQ_CUDA_TRY(smem_limit_once(k, attr_set, &smem_max));
    TQ_CHECK_ARG(L.smem <= (size_t)smem_max, "i4 matvec: %zu B of shared memory above the %d B limit",
                 L.smem, smem_max);
    // one CTA per SM for this kernel (the activation prologue is paid once per SM); the
    // SM's second slot is for the next kernel
    const int grid = grid_fixed > 0 ? grid_fixed : std::min(grid_for(k, L.block, L.smem, passes), num_sms());
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
    int rows_total = 0;
    for (int j = 0; j < n_jobs; ++j)
        if (!pair || j == 0) rows_total += std::max(0, jobs[j].rows);
    if (o.eidx) {
        TQ_CHECK_ARG(o.erows > 0 && o.nslots > 0 && o.n_experts > 0 && !o.argmax.token,
                     "expert matvec: bad erows %d / nslots %d / n_experts %d", o.erows, o.nslots,
                     o.n_experts);
        for (int j = 0; j < n_jobs; ++j)
            TQ_CHECK_ARG(jobs[j].rows == o.nslots * o.erows && (uintptr_t)jobs[j].w % 16u == 0 &&
                             o.estride % 16 == 0,
                         "expert matvec: job %d is not nslots x erows aligned rows", j);
        TQ_CHECK_ARG(!o.xslots || (n_jobs == 1 && !pair && o.x.mode == X_PLAIN),
                     "per-slot activations need one plain job");
    }
    P.eidx = o.eidx;
    P.estride = o.estride;
    P.erows = o.erows;
    P.nslots = o.nslots;
    P.n_experts = o.n_experts;
    P.xslots = o.xslots ? 1 : 0;
    P.stamp = o.stamp;
    P.xw = o.xwait;
    P.xp = o.put;
    const Shape L = plan(in_dim, group_size, pair, o.x.mode == X_RMSNORM, rows_total,
                         o.eidx ? o.erows : 0);
    bool aligned = true;  // the TMA path needs 16-byte aligned matrix bases
    for (int j = 0; j < n_jobs; ++j) aligned = aligned && ((uintptr_t)jobs[j].w % 16u == 0);
    const bool fast = (group_size % 32 == 0) && L.seg != 0 && aligned;
    if (!fast) {
        TQ_CHECK_ARG(o.x.mode == X_PLAIN && !o.argmax.token && !pair && !o.eidx && !o.put &&
                         !o.xwait,
                     "fused prologue/epilogue, expert mode and peer exchange need group_size "
                     "%% 32 == 0 and aligned weights");
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
    auto a16 = [](const void *p) { return ((uintptr_t)p & 15u) == 0; };
    P.x_bulk = (in_dim % 4 == 0) && a16(o.x.src) && (o.x.mode != X_RMSNORM || a16(o.x.norm_w)) &&
               (o.x.mode != X_SWIGLU || a16(o.x.up));
    TQ_CHECK_ARG(!o.xslots || P.x_bulk, "per-slot activations need 16-byte aligned rows of x");
    TQ_CHECK_ARG(acc > 0 || !o.put, "peer exchange: a launch with no rows never arrives");
    if (acc == 0) return TQB200_OK;
    if (fast) {
        P.nt = L.nt;
        P.S = L.S;
        P.RP = L.RP;
        P.R = L.R;
        P.stages = L.stages;
        P.stage_bytes = L.stage_bytes;
        // slot mode: a multiple of nslots CTAs, every block served by the same count
        const int grid = o.xslots ? o.nslots * std::max(1, num_sms() / o.nslots) : 0;
        const int mode = (P.stamp.base != nullptr ? 1 : 0) | (P.xw || P.xp ? 2 : 0);
#define TQ_I4_LAUNCH(SEGV)                                                              \
    switch (mode) {                                                                    \
        case 0: return launch_tma<SEGV, false, false>(P, L, acc, o.pdl, stream, grid); \
        case 1: return launch_tma<SEGV, true, false>(P, L, acc, o.pdl, stream, grid);  \
        case 2: return launch_tma<SEGV, false, true>(P, L, acc, o.pdl, stream, grid);  \
        default: return launch_tma<SEGV, true, true>(P, L, acc, o.pdl, stream, grid); \
    }
        if (L.seg == 64) TQ_I4_LAUNCH(64)
        TQ_I4_LAUNCH(32)
#undef TQ_I4_LAUNCH
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
