// matmul_i4_tc.cu — batched i4 (HQQ/RTN group-quantised) matmul on the sm_100a tensor
// cores (tcgen05.mma, accumulator in TMEM).
//
// Reference semantics: matmul_i4_ref (kernels/matvec/matmul_i4_ref.cpp:53-114):
//   Y[:, n] = matvec_i4(W, X[:, n]) for every column n, X [K, N] and Y [M, N] column-major
// (one token per column), each weight dequantised as ((float)q - zero) * scale in fp32
// and the products accumulated in double.
//
// Design (one CTA = a tile of 128 weight rows x NT token columns, all of K):
//  * The tensor cores cannot apply a per-(row, group) scale inside the K reduction, so
//    the weights are dequantised into the MMA operand: w = ((float)q - z) * s exactly as
//    the reference (fp32), then split w = hi + lo into two bf16 values.  X is split the
//    same way by a small pre-pass, and Y = Whi Xhi + Whi Xlo + Wlo Xhi with fp32
//    accumulation in TMEM (three kind::f16 MMAs per K step; the dropped Wlo Xlo term and
//    the two rounding residues are ~2^-17 of each product, far inside the 1e-4 bound).
//  * Dequantisation by table: for each (row, group) the 16 possible weights are built
//    once (hi|lo packed in one 32-bit word) in shared memory, and each nibble becomes
//    one shared-memory lookup plus one byte permute for the hi and lo operand words.
//  * Roles: warps 0-7 dequantise (thread = row r, K half h of a 64-wide stage) and
//    afterwards drain TMEM in the epilogue; warp 8 allocates TMEM and one of its lanes
//    issues the MMAs.  The X operand planes of a stage arrive by 1-D bulk copies (TMA)
//    issued by thread 0; stages are handed over by mbarriers (full: 8 producer warps +
//    the copy bytes; empty: tcgen05.commit after the stage's MMAs).
//  * Operand layout in shared memory: the canonical K-major, no-swizzle UMMA layout of
//    8-row x 16-byte core matrices, core matrices of one 8-row group adjacent along K
//    (leading byte offset 128) and 8-row groups 1024 bytes apart (stride byte offset).
//  * Every mbarrier wait is bounded; on a timeout the kernel records an error word,
//    stops issuing work, drains what it issued and frees its TMEM before returning.
#include <algorithm>
#include <atomic>

#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"

namespace tqb200 {

namespace {

constexpr int kMmRows = 128;       // UMMA M
constexpr int kMmKs = 64;          // K per pipeline stage
constexpr int kMmProducers = 256;  // warps 0-7
constexpr int kMmThreads = kMmProducers + 32;
constexpr int kMmMaxStages = 4;
constexpr uint32_t kABytes = kMmRows * kMmKs * 2;  // one bf16 plane of a stage (16 KB)
constexpr uint32_t kLutBytes = 16 * kMmProducers * 4;  // one buffer (16 KB)

struct MmParams {
    MmJob job0;            // used when jobs == nullptr
    const MmJob *jobs;     // device array (grouped launch) or nullptr
    int n_jobs;
    int K, G, ks;          // ks = ceil(K / 64) stages
    int nt;                // tile width in columns (multiple of 16, <= 256)
    const uint16_t *bhi, *blo;  // X planes (bf16 bits), see mm_pack_x_kernel
    int stages;
    uint32_t stage_bytes;  // 2 * kABytes + 2 * nt * 128
    uint32_t tmem_cols;
    int *status;
};

// ---------------------------------------------------------------- tcgen05 wrappers
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    // start address, leading / stride byte offsets (all >> 4), version 1 (sm_100),
    // base offset 0, no swizzle
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) |
           ((uint64_t)(sbo >> 4) << 32) | (1ull << 46);
}

// kind::f16 instruction descriptor: bf16 A and B (K-major), fp32 accumulator, M = 128.
__device__ __forceinline__ uint32_t umma_idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(kMmRows >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_plain(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// Named barrier 1 over the producer warps; returns the OR of `pred` across them.
__device__ __forceinline__ bool producers_sync_or(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.or.pred p, 1, %2, q;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "n"(kMmProducers)
        : "memory");
    return r != 0;
}

// bf16 hi | lo split of an fp32 value, hi in the low half of the word.
__device__ __forceinline__ uint32_t split_bf16(float v) {
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const float r = __fsub_rn(v, __bfloat162float(hi));
    const __nv_bfloat16 lo = __float2bfloat16_rn(r);
    return (uint32_t)__bfloat16_as_ushort(hi) | ((uint32_t)__bfloat16_as_ushort(lo) << 16);
}

__device__ __forceinline__ const MmJob &job_of(const MmParams &P, int j) {
    return P.jobs ? P.jobs[j] : P.job0;
}

// ---------------------------------------------------------------- X pre-pass
// X (column n at x + col(n) * ldx, K floats) -> two bf16 planes (hi, lo) laid out
// [stage][n/8][kc][n%8][8]: stage = k/64, kc = (k%64)/8, i.e. every (stage, 8-column
// block) is one kilobyte holding eight 8x16-byte core matrices of the K-major UMMA
// layout.  Columns >= N and k >= K are zero.  One thread per 8-k chunk of a column.
__global__ void mm_pack_x_kernel(const float *__restrict__ x, const int *__restrict__ cols, int ldx,
                                 int K, int N, int npad, int ks, uint16_t *__restrict__ bhi,
                                 uint16_t *__restrict__ blo) {
    const long long total = (long long)npad * ks * 8;
    for (long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x; c < total;
         c += (long long)gridDim.x * blockDim.x) {
        // c = ((stage * npad/8 + nb) * 8 + kc) * 8 + n%8: consecutive threads write
        // consecutive 16-byte rows of a core matrix
        const int n8 = (int)(c & 7);
        const long long r = c >> 3;
        const int kc = (int)(r & 7);
        const long long sb = r >> 3;
        const int nb = (int)(sb % (npad / 8));
        const int st = (int)(sb / (npad / 8));
        const int n = nb * 8 + n8;
        const int k0 = st * kMmKs + kc * 8;
        uint32_t w[8];
        if (n < N) {
            const float *src = x + (size_t)(cols ? cols[n] : n) * ldx;
#pragma unroll
            for (int e = 0; e < 8; ++e) w[e] = k0 + e < K ? split_bf16(src[k0 + e]) : 0u;
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) w[e] = 0u;
        }
        uint4 h, l;
        h.x = __byte_perm(w[0], w[1], 0x5410), h.y = __byte_perm(w[2], w[3], 0x5410);
        h.z = __byte_perm(w[4], w[5], 0x5410), h.w = __byte_perm(w[6], w[7], 0x5410);
        l.x = __byte_perm(w[0], w[1], 0x7632), l.y = __byte_perm(w[2], w[3], 0x7632);
        l.z = __byte_perm(w[4], w[5], 0x7632), l.w = __byte_perm(w[6], w[7], 0x7632);
        reinterpret_cast<uint4 *>(bhi)[c] = h;
        reinterpret_cast<uint4 *>(blo)[c] = l;
    }
}

// ---------------------------------------------------------------- the GEMM
__global__ void __launch_bounds__(kMmThreads, 1) mm_i4_tc_kernel(const __grid_constant__ MmParams P) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);  // [kMmMaxStages]
    uint64_t *empty = full + kMmMaxStages;                 // [kMmMaxStages]
    uint64_t *done = empty + kMmMaxStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    uint32_t *lut = reinterpret_cast<uint32_t *>(smem + 1024);  // [2][16][256]
    uint8_t *stage_base = smem + 1024 + 2 * kLutBytes;
    __shared__ int s_err;

    // ---- which tile: job j, rows m0.., columns n0..n0+nw
    int j = 0;
    const int tile = blockIdx.x;
    while (j + 1 < P.n_jobs && tile >= job_of(P, j + 1).tile_begin) ++j;
    const MmJob &job = job_of(P, j);
    const int local = tile - job.tile_begin;
    const int mt = (job.M + kMmRows - 1) / kMmRows;
    const int npad = (job.N + 15) & ~15;
    const int m0 = (local % mt) * kMmRows;
    const int n0 = (local / mt) * P.nt;
    const int nw = min(P.nt, npad - n0);  // this tile's MMA N (multiple of 16)
    const uint32_t b_bytes = (uint32_t)nw * 128u;  // one X plane of a stage
    const uint32_t stage_bytes = P.stage_bytes;
    const int G = P.G, K = P.K, ks = P.ks;
    const int GB = 4 + G / 2;
    const size_t RB = (size_t)((K + G - 1) / G) * GB;

    if (t == 0) {
        for (int s = 0; s < P.stages; ++s) {
            mbar_init(&full[s], kMmProducers / 32);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        s_err = 0;
    }
    if (warp == 8) {  // TMEM accumulator: 128 lanes x tmem_cols fp32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(P.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < 8) {
        // ---------------- producers: thread = (row r, half h) of every stage
        const int r = t & (kMmRows - 1), h = t >> 7;
        const int row = m0 + r;
        const bool row_ok = row < job.M;
        const uint8_t *wrow = job.w + (size_t)(row_ok ? row : 0) * RB;
        const bool shared_lut = G >= kMmKs;  // both halves of a stage share the group
        const int slot = shared_lut ? r : t;
        int issued = 0;
        bool abort = false;
        // weight words of stage i (group header + 4 nibble words): fetched two stages
        // ahead into registers so the global-load latency overlaps the work in between
        auto fetch = [&](int i, uint32_t &hdr, uint32_t(&nb)[4]) {
            hdr = 0u;
            nb[0] = nb[1] = nb[2] = nb[3] = 0u;
            const int k = i * kMmKs + 32 * h;
            // the table's group exists (with a shared table the partner half may need it
            // even when this half lies past K); same group for both halves when shared
            if (i >= ks || !row_ok || (shared_lut ? i * kMmKs : k) >= K) return;
            const uint8_t *gp = wrow + (size_t)(k / G) * GB;
            hdr = ldg_u32(gp);
            if (k < K) {
                const uint8_t *np_ = gp + 4 + (k % G) / 2;
#pragma unroll
                for (int q = 0; q < 4; ++q) nb[q] = ldg_u32(np_ + 4 * q);
            }
        };
        uint32_t hdr0, nib0[4], hdr1, nib1[4];
        fetch(0, hdr0, nib0);
        fetch(1, hdr1, nib1);
        for (int i = 0; i < ks; ++i) {
            const int s = i % P.stages;
            const int k = i * kMmKs + 32 * h;  // first column of this thread's half
            uint32_t hdr2, nib2[4];
            fetch(i + 2, hdr2, nib2);
            bool ok = true;
            if (i >= P.stages)
                ok = mbar_wait(&empty[s], (uint32_t)((i / P.stages) - 1) & 1u, kWaitCycles);
            // table of the 16 dequantised values of this (row, group) in buffer i & 1
            uint32_t *lb = lut + (size_t)(i & 1) * (16 * kMmProducers);
            const bool have = row_ok && k < K;  // this half holds weights
            const bool full_half = k + 32 <= K;
            const bool build = row_ok && (shared_lut ? i * kMmKs : k) < K;
            uint32_t nib[4] = {nib0[0], nib0[1], nib0[2], nib0[3]};
            if (build) {
                const float sc = h2f((uint16_t)(hdr0 & 0xFFFFu));
                const float z = h2f((uint16_t)(hdr0 >> 16));
                const int q0 = shared_lut ? 8 * h : 0, q1 = shared_lut ? q0 + 8 : 16;
                for (int q = q0; q < q1; ++q)
                    lb[q * kMmProducers + slot] = split_bf16(__fmul_rn(__fsub_rn((float)q, z), sc));
            }
            hdr0 = hdr1;
            hdr1 = hdr2;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                nib0[q] = nib1[q];
                nib1[q] = nib2[q];
            }
            abort = producers_sync_or(!ok);  // also: the tables are complete
            if (abort) break;
            uint8_t *st = stage_base + (size_t)s * stage_bytes;
            if (t == 0) {  // X planes of this stage: two bulk copies
                mbar_expect_tx(&full[s], 2u * b_bytes);
                const size_t blk = ((size_t)i * (npad / 8) + n0 / 8) * 512;  // bf16 elements
                bulk_g2s(st + 2 * kABytes, P.bhi + job.b_off + blk, b_bytes, &full[s]);
                bulk_g2s(st + 2 * kABytes + b_bytes, P.blo + job.b_off + blk, b_bytes, &full[s]);
                issued = i + 1;
            }
            // dequantise 32 weights: nibble -> table word -> (hi, lo) bf16 pairs
            const uint32_t off = (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 16u;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint4 hv = make_uint4(0u, 0u, 0u, 0u), lv = hv;
                if (have) {
                    uint32_t e[8];
                    const uint32_t *lt = lb + slot;
#pragma unroll
                    for (int n = 0; n < 8; ++n) {
                        const int kk = k + 8 * q + n;
                        e[n] = (full_half || kk < K) ? lt[((nib[q] >> (4 * n)) & 15u) * kMmProducers] : 0u;
                    }
                    hv.x = __byte_perm(e[0], e[1], 0x5410), hv.y = __byte_perm(e[2], e[3], 0x5410);
                    hv.z = __byte_perm(e[4], e[5], 0x5410), hv.w = __byte_perm(e[6], e[7], 0x5410);
                    lv.x = __byte_perm(e[0], e[1], 0x7632), lv.y = __byte_perm(e[2], e[3], 0x7632);
                    lv.z = __byte_perm(e[4], e[5], 0x7632), lv.w = __byte_perm(e[6], e[7], 0x7632);
                }
                const uint32_t o = off + (uint32_t)(4 * h + q) * 128u;
                *reinterpret_cast<uint4 *>(st + o) = hv;
                *reinterpret_cast<uint4 *>(st + kABytes + o) = lv;
            }
            fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive_plain(&full[s]);
        }
        if (abort && t == 0) s_err = 1;
        // drain: the copies of the last issued stages have landed before smem is released
        if (t == 0) {
            for (int i = max(0, issued - P.stages); i < issued; ++i)
                if (!mbar_wait(&full[i % P.stages], (uint32_t)(i / P.stages) & 1u, kWaitCycles))
                    s_err = 1;
        }
        // ---------------- epilogue: TMEM -> Y (column-major), lanes 32*(warp%4).., columns
        // split between warps w and w+4
        // warp-uniform: tcgen05.ld below is a whole-warp instruction
        const bool fin = __all_sync(0xffffffffu, mbar_wait(done, 0u, kWaitCycles));
        tc_fence_after();
        if (fin) {
            const int lq = warp & 3;
            const int half = nw / 2;  // multiple of 8
            const int c0 = (warp >> 2) * half;
            const int orow = m0 + 32 * lq + lane;
            for (int c = c0; c < c0 + half; c += 8) {
                uint32_t v[8];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                    "tcgen05.wait::ld.sync.aligned;\n"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                      "=r"(v[6]), "=r"(v[7])
                    : "r"(tmem + ((uint32_t)(32 * lq) << 16) + (uint32_t)c)
                    : "memory");
                if (orow < job.M) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int n = n0 + c + e;
                        if (n < job.N) job.y[(size_t)n * job.ldy + orow] = __uint_as_float(v[e]);
                    }
                }
            }
        } else if (t == 0) {
            s_err = 1;
        }
    } else if (lane == 0) {
        // ---------------- MMA issuer
        bool ok = true;
        const uint32_t idesc = umma_idesc_bf16(nw);
        for (int i = 0; i < ks && ok; ++i) {
            const int s = i % P.stages;
            if (!mbar_wait(&full[s], (uint32_t)(i / P.stages) & 1u, kWaitCycles)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t a_hi = smem_u32(stage_base + (size_t)s * stage_bytes);
            const uint32_t a_lo = a_hi + kABytes;
            const uint32_t b_hi = a_hi + 2 * kABytes;
            const uint32_t b_lo = b_hi + b_bytes;
#pragma unroll
            for (int kk = 0; kk < kMmKs / 16; ++kk) {
                const uint32_t o = (uint32_t)kk * 256u;  // two 16-byte core-matrix columns
                const uint64_t ah = umma_desc(a_hi + o, 128, 1024), al = umma_desc(a_lo + o, 128, 1024);
                const uint64_t bh = umma_desc(b_hi + o, 128, 1024), bl = umma_desc(b_lo + o, 128, 1024);
                umma_bf16(tmem, ah, bh, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                umma_bf16(tmem, ah, bl, idesc, 1u);
                umma_bf16(tmem, al, bh, idesc, 1u);
            }
            umma_commit(&empty[s]);  // stage s free once these MMAs have read it
        }
        if (!ok) s_err = 1;
        umma_commit(done);  // every MMA issued above has completed
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(P.tmem_cols)
                     : "memory");
    }
    if (t == 0 && s_err && P.status) atomicExch(P.status, kDevTimeoutTma);
}

std::atomic<unsigned long long> g_mm_smem_set{0};

}  // namespace

size_t mm_x_planes_bytes(int K, int N) {
    const size_t ks = (size_t)(K + kMmKs - 1) / kMmKs;
    const size_t npad = (size_t)(N + 15) & ~(size_t)15;
    return 2 * ks * kMmKs * npad * 2;  // hi + lo bf16
}

// Widest column tile (fewest re-dequantisations of a weight tile) that still gives every
// SM a CTA; the narrowest that covers the columns when nothing fills the SMs.
int mm_tile_width(int M, int N) {
    const int npad = (N + 15) & ~15;
    const int mt = (M + kMmRows - 1) / kMmRows;
    const int sms = num_sms();
    for (int nt = 256; nt >= 16; nt >>= 1) {
        if (nt > npad && nt > 16) continue;
        if (mt * ((npad + nt - 1) / nt) >= sms) return nt;
    }
    return std::min(npad, 128);
}

int launch_matmul_i4_grouped(const MmJob *host_jobs, const MmJob *dev_jobs, int n_jobs, int K,
                             int G, int nt, const uint16_t *bhi, const uint16_t *blo, int total_tiles,
                             int *status, cudaStream_t st) {
    TQ_CHECK_ARG(n_jobs >= 1, "matmul_i4: no jobs");
    TQ_CHECK_ARG(G % 32 == 0 && G >= 32, "matmul_i4 (tensor cores): group_size %d not a multiple of 32", G);
    TQ_CHECK_ARG(nt % 16 == 0 && nt >= 16 && nt <= 256, "matmul_i4: bad tile width %d", nt);
    TQ_CHECK_ARG(((uintptr_t)bhi & 15) == 0 && ((uintptr_t)blo & 15) == 0, "matmul_i4: X planes not 16-byte aligned");
    if (total_tiles == 0) return TQB200_OK;
    MmParams P{};
    if (dev_jobs == nullptr) P.job0 = host_jobs[0];
    P.jobs = dev_jobs;
    P.n_jobs = dev_jobs ? n_jobs : 1;
    P.K = K;
    P.G = G;
    P.ks = (K + kMmKs - 1) / kMmKs;
    P.nt = nt;
    P.bhi = bhi;
    P.blo = blo;
    P.stage_bytes = 2 * kABytes + 2u * (uint32_t)nt * 128u;
    uint32_t cols = 32;
    while ((int)cols < nt) cols <<= 1;
    P.tmem_cols = cols;
    P.status = status;
    int limit = 0;
    TQ_CUDA_TRY(smem_limit_once(mm_i4_tc_kernel, g_mm_smem_set, &limit));
    const int fixed = 1024 + 2 * (int)kLutBytes;
    int stages = std::min(kMmMaxStages, (limit - fixed) / (int)P.stage_bytes);
    stages = std::min(stages, P.ks);
    TQ_CHECK_ARG(stages >= 1, "matmul_i4: tile of %d columns does not fit shared memory", nt);
    P.stages = stages;
    const size_t smem = (size_t)fixed + (size_t)stages * P.stage_bytes;
    mm_i4_tc_kernel<<<total_tiles, kMmThreads, smem, st>>>(P);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_mm_pack_x(const float *x, const int *cols, int ldx, int K, int N, uint16_t *bhi,
                     uint16_t *blo, cudaStream_t st) {
    const int npad = (N + 15) & ~15;
    const int ks = (K + kMmKs - 1) / kMmKs;
    const long long total = (long long)npad * ks * 8;
    if (total == 0) return TQB200_OK;
    const int threads = 256;
    const long long blocks = std::min<long long>((total + threads - 1) / threads, 148LL * 16);
    mm_pack_x_kernel<<<(int)blocks, threads, 0, st>>>(x, cols, ldx, K, N, npad, ks, bhi, blo);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

// Y = W X for one matrix: X planes from the caller's scratch (mm_x_planes_bytes(K, N)).
int launch_matmul_i4(const uint8_t *w, const float *x, float *y, int M, int K, int N, int G,
                     void *scratch, int *status, cudaStream_t st) {
    TQ_CHECK_ARG(M >= 0 && K > 0 && N >= 0, "matmul_i4: bad shape %d x %d x %d", M, K, N);
    if (M == 0 || N == 0) return TQB200_OK;
    TQ_CHECK_ARG(((uintptr_t)w & 3) == 0, "matmul_i4: weights not 4-byte aligned");
    const int npad = (N + 15) & ~15;
    const size_t plane = mm_x_planes_bytes(K, N) / 2;
    uint16_t *bhi = static_cast<uint16_t *>(scratch);
    uint16_t *blo = reinterpret_cast<uint16_t *>(static_cast<uint8_t *>(scratch) + plane);
    int r = launch_mm_pack_x(x, nullptr, K, K, N, bhi, blo, st);
    if (r != TQB200_OK) return r;
    const int nt = mm_tile_width(M, N);
    MmJob j{};
    j.w = w;
    j.y = y;
    j.M = M;
    j.N = N;
    j.ldy = M;
    j.tile_begin = 0;
    j.b_off = 0;
    const int tiles = ((M + kMmRows - 1) / kMmRows) * ((npad + nt - 1) / nt);
    return launch_matmul_i4_grouped(&j, nullptr, 1, K, G, nt, bhi, blo, tiles, status, st);
}

}  // namespace tqb200
