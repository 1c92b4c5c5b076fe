// i4_matvec.cu — batch-1 i4 (HQQ/RTN group-quantised) matvec kernels for sm_100a.
//
// Reference semantics: matvec_i4_ref (kernels/matvec/matvec_i4_ref.cpp:45-103):
//   y[o] = sum_g sum_i ((float)q - zero_g) * scale_g * x[i]
// on rows of ceil(K/G) groups laid out [scale f16][zero f16][G/2 nibble bytes]
// (runtime/tiny_format.h:66-77), low nibble = even column.
//
// Design (B200, HBM-bound at batch 1): the kernel streams the interleaved
// layout as stored, with no repack.  A CTA owns a block of R consecutive rows
// per pass; thread (slot, seg) owns one SEG-column segment (SEG = 32 or 64, a
// divisor of G) of rows slot, slot+S, ... of the block, so the whole CTA
// reads one contiguous byte range per pass (coalesced 4-byte loads, L1
// absorbs the 36-byte group stride).  Each thread keeps its SEG activations
// in registers for the whole kernel, pre-scaled per nibble position so that
// a nibble becomes an exact float with a single LOP3 (bits OR'ed into the
// mantissa of 2^23) and one FADD; the dot is then one FFMA per weight:
//   sum_i (q_i - z) s x_i = s * (sum_i q_i x_i - z * sum_i x_i)
// Row sums reduce through shared memory (deterministic order).
// Accumulation is fp32 (the reference accumulates in double); results agree
// to ~1e-6 relative, inside the 1e-4 max-relative tolerance the tests use.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace tqb200 {

namespace {

constexpr uint32_t kMagic = 0x4B000000u;   // 2^23
constexpr float kMagicF = 8388608.0f;

struct I4JobsParam {
    I4Job job[3];
    int pass_begin[4];
    int n_jobs;
};

__device__ __forceinline__ float nib_f(uint32_t w, uint32_t mask) {
    return __uint_as_float((w & mask) | kMagic) - kMagicF;
}

// Accumulates one 32-bit word of 8 nibbles against 8 pre-scaled activations.
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

template <int SEG, int RP>
__global__ void __launch_bounds__(512) i4_matvec_kernel(I4JobsParam P, const float *__restrict__ x,
                                                         int K, int G, int nt, int S) {
    extern __shared__ float red[];  // [R][nt]
    constexpr int NW = SEG / 8;     // nibble words per segment
    const int t = threadIdx.x;
    const int slot = t / nt;
    const int sg = t - slot * nt;
    const int R = S * RP;
    const int ng = (K + G - 1) / G;
    const int GB = 4 + G / 2;
    const size_t RB = (size_t)ng * GB;
    const int spg = G / SEG;
    const int g = sg / spg;
    const int sub = sg - g * spg;
    const int col0 = sg * SEG;
    const uint32_t hdr_off = (uint32_t)g * GB;
    const uint32_t seg_off = hdr_off + 4u + (uint32_t)sub * (SEG / 2);
    const bool active = slot < S;

    // activations of this segment, pre-scaled by 16^-k for nibble position k
    float xs[SEG];
    float X = 0.0f;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int col = col0 + 8 * i + k;
            const float v = (active && col < K) ? __ldg(x + col) : 0.0f;
            X += v;
            const int pos = k < 5 ? k : k - 3;
            xs[8 * i + k] = v * __uint_as_float((uint32_t)(127 - 4 * pos) << 23);
        }
    }

    const int nwarps = blockDim.x >> 5;
    const int lane = t & 31, warp = t >> 5;
    const int total = P.pass_begin[P.n_jobs];
    for (int p = blockIdx.x; p < total; p += gridDim.x) {
        int j = 0;
        while (j + 1 < P.n_jobs && p >= P.pass_begin[j + 1]) ++j;
        const I4Job &job = P.job[j];
        const int row_base = (p - P.pass_begin[j]) * R;

        uint32_t wv[RP][NW];
        uint32_t hv[RP];
#pragma unroll
        for (int r = 0; r < RP; ++r) {
            const int row = row_base + slot + r * S;
            if (active && row < job.rows) {
                const uint8_t *rp = job.w + (size_t)row * RB;
                hv[r] = ldg_u32(rp + hdr_off);
#pragma unroll
                for (int i = 0; i < NW; ++i) wv[r][i] = ldg_u32(rp + seg_off + 4 * i);
            } else {
                hv[r] = 0u;
#pragma unroll
                for (int i = 0; i < NW; ++i) wv[r][i] = 0u;
            }
        }
#pragma unroll
        for (int r = 0; r < RP; ++r) {
            float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
            for (int i = 0; i < NW; ++i) dot8(wv[r][i], xs + 8 * i, a0, a1);
            const float s = h2f((uint16_t)(hv[r] & 0xFFFFu));
            const float z = h2f((uint16_t)(hv[r] >> 16));
            const float part = s * fmaf(-z, X, a0 + a1);
            if (active) red[(slot + r * S) * nt + sg] = part;
        }
        __syncthreads();
        for (int rho = warp; rho < R; rho += nwarps) {
            const int row = row_base + rho;
            if (row >= job.rows) continue;
            float v = 0.0f;
            for (int i = lane; i < nt; i += 32) v += red[rho * nt + i];
            v = warp_sum(v);
            if (lane == 0) {
                if (job.bias) v += job.bias[row];
                if (job.resid) v = job.resid[row] + v;
                job.y[row] = v;
            }
        }
        __syncthreads();
    }
}

// Generic path for group sizes that are not a multiple of 32 (e.g. 48): one
// warp per row, lanes over groups, byte loads.
__global__ void i4_matvec_generic_kernel(I4JobsParam P, const float *__restrict__ x, int K,
                                         int G) {
    const int ng = (K + G - 1) / G;
    const int GB = 4 + G / 2;
    const size_t RB = (size_t)ng * GB;
    const int lane = threadIdx.x & 31;
    const int warps_per_block = blockDim.x >> 5;
    const int total = P.pass_begin[P.n_jobs];  // one "pass" == one row here
    for (int p = blockIdx.x * warps_per_block + (threadIdx.x >> 5); p < total;
         p += gridDim.x * warps_per_block) {
        int j = 0;
        while (j + 1 < P.n_jobs && p >= P.pass_begin[j + 1]) ++j;
        const I4Job &job = P.job[j];
        const int row = p - P.pass_begin[j];
        const uint8_t *rp = job.w + (size_t)row * RB;
        float acc = 0.0f;
        for (int g = lane; g < ng; g += 32) {
            const uint8_t *gp = rp + (size_t)g * GB;
            const float s = h2f((uint16_t)(gp[0] | (gp[1] << 8)));
            const float z = h2f((uint16_t)(gp[2] | (gp[3] << 8)));
            const int c0 = g * G;
            const int n = min(G, K - c0);
            float a = 0.0f, xsum = 0.0f;
            for (int i = 0; i < n; ++i) {
                const uint8_t b = gp[4 + (i >> 1)];
                const float q = (float)((i & 1) ? (b >> 4) : (b & 15));
                const float xv = x[c0 + i];
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
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

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
    // amax over all of x (every CTA recomputes it: K floats from L2)
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
    const int sub = sg - g * spg;
    const int col0 = sg * SEG;
    const uint32_t hdr_off = (uint32_t)g * GB;
    const uint32_t seg_off = hdr_off + 4u + (uint32_t)sub * (SEG / 2);
    const bool active = slot < S;

    // xq packed to match (lo nibbles = even cols, hi nibbles = odd cols) per word
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
        float part = 0.0f;
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
            part = A * (float)dot;
            red[slot * nt + sg] = part;
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

__global__ void i4_embed_row_kernel(const uint8_t *__restrict__ w, const int *__restrict__ token,
                                    int dim, int G, float *__restrict__ out) {
    const int ng = (dim + G - 1) / G;
    const int GB = 4 + G / 2;
    const uint8_t *row = w + (size_t)(*token) * ng * GB;
    for (int c = threadIdx.x + blockIdx.x * blockDim.x; c < dim; c += blockDim.x * gridDim.x) {
        const int g = c / G, i = c - g * G;
        const uint8_t *gp = row + (size_t)g * GB;
        const float s = h2f((uint16_t)(gp[0] | (gp[1] << 8)));
        const float z = h2f((uint16_t)(gp[2] | (gp[3] << 8)));
        const uint8_t b = gp[4 + (i >> 1)];
        const float q = (float)((i & 1) ? (b >> 4) : (b & 15));
        out[c] = __fmul_rn(__fsub_rn(q, z), s);
    }
}

int g_num_sms = 0;

struct LaunchShape {
    int seg, nt, S, block;
};

LaunchShape pick_shape(int K, int G, int rp) {
    LaunchShape L{};
    L.seg = (G % 64 == 0) ? 64 : 32;
    const int ng = (K + G - 1) / G;
    L.nt = ng * (G / L.seg);
    if (L.nt > 512) {
        L.seg = 0;
        return L;
    }
    const int target = 384;
    L.S = std::max(1, std::min(512 / L.nt, (target + L.nt - 1) / L.nt));
    L.block = ((L.nt * L.S + 31) / 32) * 32;
    (void)rp;
    return L;
}

template <typename Kern>
int occupancy_grid(Kern k, int block, size_t smem, int work) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, block, smem) != cudaSuccess ||
        per_sm < 1)
        per_sm = 1;
    return std::max(1, std::min(work, per_sm * num_sms()));
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

int launch_i4_matvec(const I4Job *jobs, int n_jobs, const float *x, int in_dim, int group_size,
                     cudaStream_t stream) {
    TQ_CHECK_ARG(n_jobs >= 1 && n_jobs <= 3, "n_jobs %d", n_jobs);
    TQ_CHECK_ARG(in_dim > 0 && group_size > 0 && group_size % 2 == 0,
                 "bad in_dim %d / group_size %d", in_dim, group_size);
    I4JobsParam P{};
    P.n_jobs = n_jobs;
    constexpr int RP = 2;
    const LaunchShape L = pick_shape(in_dim, group_size, RP);
    bool aligned = true;  // the fast path reads 4-byte words
    for (int j = 0; j < n_jobs; ++j) aligned = aligned && ((uintptr_t)jobs[j].w % 4u == 0);
    const bool fast = (group_size % 32 == 0) && L.seg != 0 && aligned;
    const int R = fast ? L.S * RP : 1;
    int acc = 0;
    for (int j = 0; j < n_jobs; ++j) {
        TQ_CHECK_ARG(jobs[j].rows >= 0, "rows %d", jobs[j].rows);
        P.job[j] = jobs[j];
        P.pass_begin[j] = acc;
        acc += (jobs[j].rows + R - 1) / R;
    }
    P.pass_begin[n_jobs] = acc;
    if (acc == 0) return TQB200_OK;
    if (fast) {
        const size_t smem = (size_t)L.S * RP * L.nt * sizeof(float);
        if (L.seg == 64) {
            auto k = i4_matvec_kernel<64, RP>;
            const int grid = occupancy_grid(k, L.block, smem, acc);
            k<<<grid, L.block, smem, stream>>>(P, x, in_dim, group_size, L.nt, L.S);
        } else {
            auto k = i4_matvec_kernel<32, RP>;
            const int grid = occupancy_grid(k, L.block, smem, acc);
            k<<<grid, L.block, smem, stream>>>(P, x, in_dim, group_size, L.nt, L.S);
        }
    } else {
        const int block = 256;
        const int grid = std::max(1, std::min((acc + 7) / 8, num_sms() * 8));
        i4_matvec_generic_kernel<<<grid, block, 0, stream>>>(P, x, in_dim, group_size);
    }
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_i4_matvec_sym(const uint8_t *w, const float *x, float *y, int rows, int in_dim,
                         int group_size, cudaStream_t stream) {
    TQ_CHECK_ARG(in_dim > 0 && group_size > 0 && group_size % 32 == 0,
                 "symmetric W4A8 path needs group_size %% 32 == 0 (got %d)", group_size);
    if (rows == 0) return TQB200_OK;
    const LaunchShape L = pick_shape(in_dim, group_size, 1);
    TQ_CHECK_ARG(L.seg != 0, "in_dim %d too large", in_dim);
    const size_t smem = (size_t)L.S * L.nt * sizeof(float);
    const int passes = (rows + L.S - 1) / L.S;
    if (L.seg == 64) {
        auto k = i4_matvec_sym_kernel<64>;
        const int grid = occupancy_grid(k, L.block, smem, passes);
        k<<<grid, L.block, smem, stream>>>(w, x, y, rows, in_dim, group_size, L.nt, L.S);
    } else {
        auto k = i4_matvec_sym_kernel<32>;
        const int grid = occupancy_grid(k, L.block, smem, passes);
        k<<<grid, L.block, smem, stream>>>(w, x, y, rows, in_dim, group_size, L.nt, L.S);
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

int launch_i4_embed_row(const uint8_t *w, const int *token, int dim, int group_size, float *out,
                        cudaStream_t stream) {
    const int block = 256;
    const int grid = std::max(1, std::min((dim + block - 1) / block, 32));
    i4_embed_row_kernel<<<grid, block, 0, stream>>>(w, token, dim, group_size, out);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

}  // namespace tqb200
