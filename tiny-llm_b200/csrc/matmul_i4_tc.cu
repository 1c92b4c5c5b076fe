// matmul_i4_tc.cu — batched i4 (HQQ/RTN group-quantised) matmul on the sm_100a tensor
// cores (tcgen05.mma, accumulators in TMEM).
//
// Reference semantics: matmul_i4_ref (kernels/matvec/matmul_i4_ref.cpp:53-114):
//   Y[:, n] = matvec_i4(W, X[:, n]) for every column n, X [K, N] and Y [M, N] column-major
// (one token per column), each weight dequantised as ((float)q - zero) * scale in fp32
// and the products accumulated in double.
//
// Design (one CTA = a tile of 128 weight rows x NT token columns, all of K):
//  * Group partials on the tensor cores.  With s, z the group's scale and zero,
//        y = sum_g s_g * P_g,   P_g = sum_{k in g} q_k x_k - z_g X_g,   X_g = sum_{k in g} x_k.
//    The codes q (0..15) are exact in bf16, so the A operand is the raw nibbles widened
//    with one LOP3 (0x4300 | q is bf16 128 + q) and one packed bf16 subtract of 128: no
//    dequantisation arithmetic and no rounding.  X is split into bf16 hi + lo (the lo
//    residue ~2^-17 of x), stored as rows [0, nw) and [nw, 2nw) of the B operand, so one
//    MMA of N = 2nw per K step yields the hi and lo partial sums side by side in TMEM.
//    The zero term rides in the same MMAs as one extra K step of 16 slots per group:
//    A = -(z1, z1, z1, z2, z2, z2) (z = z1 + z2 exactly, z is binary16) against
//    B = (X1, X2, X3, X1, X2, X3) in the hi rows (X_g = X1 + X2 + X3, three bf16 parts of
//    the fp32 group sum; zeros in the lo rows), so each group's P_g lands in TMEM whole.
//  * Epilogue per group: 8 warps read P_g's two halves from TMEM (double-buffered
//    accumulators, so the MMAs of group g+1 overlap the read of group g) and fold
//    y += s_g * (P_hi + P_lo) in fp32 registers.
//  * Roles: warps 0-7 build the A operand (thread = weight row of the 256-row tile) from
//    the weight blocks (256 rows x 4 groups) that warp 17 stages a few blocks ahead,
//    together with the stage's X planes, which a pre-pass kernel lays out in the MMA's
//    shared-memory order.  A weight block comes by one 3-D tensor copy (TMA) straight out
//    of the interleaved rows (runtime/tiny_format.h:66-77) the decode matvec reads, so the
//    model's i4 bytes are held once; where a row's byte length is not a multiple of 16
//    (K / G not a multiple of 4) no tensor map exists for it, and the block comes by 1-D
//    bulk copies from a tile-contiguous repacked copy instead.  Warps 8-15 are the epilogue; warp 16 allocates TMEM and one
//    lane issues the MMAs; warp 18 does the MMA warp's barrier waits.  Stages (one quantisation group each) are handed over with
//    mbarriers: full (8 producer warps + the X-plane copy bytes), empty (tcgen05.commit),
//    tmem_full per row half (commit) and tmem_empty per row half (its 4 epilogue warps);
//    rawbar/rawfree for the weight blocks.
//  * Operand layout in shared memory: the canonical K-major, no-swizzle UMMA layout of
//    8-row x 16-byte core matrices, the core matrices of one 8-row group adjacent along
//    K (leading byte offset 128), 8-row groups (G+16)*16 bytes apart (stride offset).
//    Within every 16-byte core-matrix row the 8 K positions hold columns
//    (0, 4, 1, 5, 2, 6, 3, 7) of that 8-column chunk, the order the nibble widening
//    produces; X is stored in the same order, so the dot products are unchanged.
//  * Every wait is bounded; on a timeout the kernel records an error word, stops issuing,
//    waits (bounded) for what it issued and frees its TMEM before returning.
// Accuracy: products carry the x residue (~2^-17 relative), the zero term ~2^-24, and
// accumulation is fp32 (the reference's is double): ~1e-5 relative, inside 1e-4.
#include <cuda.h>
#include <cuda_bf16.h>
#include <string.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace tqb200 {

namespace {

constexpr int kMmRows = 128;       // UMMA M
constexpr int kProdWarps = 8;      // warps 0-7: A operand, one weight row per thread
constexpr int kEpiWarps = 8;       // warps 8-15: TMEM -> registers -> Y
constexpr int kMmaWarp = kProdWarps + kEpiWarps;  // warp 16: TMEM allocation, MMA issue
constexpr int kLoadWarp = kMmaWarp + 1;           // warp 17: bulk copies (TMA)
constexpr int kGateWarp = kLoadWarp + 1;           // warp 18: waits on behalf of the MMA warp
constexpr int kMmThreads = (kGateWarp + 1) * 32;
// Named barriers between the gate warp and the MMA warp (0 is __syncthreads): stage
// ready, then row half 0 / 1 drained.  A shared-memory wait issued by the MMA thread right
// after its MMAs stalls until they have read their operands, so the MMA warp only meets
// the gate warp at hardware barriers.
constexpr int kBarStage = 1, kBarHalf0 = 2;
constexpr int kMmMaxStages = 4;
constexpr int kTileRows = 2 * kMmRows;  // weight rows per CTA: two accumulators share X
static_assert(kTileRows == kMmTileRows, "tile rows");
constexpr int kMmMaxCols = 64;     // tile width limit (epilogue registers)
// group scales handed from producers to the epilogue: a slot is rewritten only after the
// epilogue has read it (the producer's stage wait orders it behind MMA i-S, which waited
// for the epilogue's drain of group i-S-2)
constexpr int kSclRing = kMmMaxStages + 3;
constexpr int kMaxRaw = 8;         // weight blocks staged ahead, at most
constexpr int kGpb = kMmGroupsPerBlock;  // quantisation groups per weight block
constexpr int kTmemCols = 512;     // the CTA's TMEM allocation (one CTA per SM: registers)

struct MmParams {
    MmJob job0;            // used when jobs == nullptr
    const MmJob *jobs;     // device array (grouped launch) or nullptr
    int n_jobs;
    const int *tile_job;   // device-planned launch: job of every tile (else binary search)
    const int *n_tiles;    // device-planned launch: tiles in use
    int K, ng;             // ng = ceil(K / G) groups = pipeline stages of a tile
    int nt;                // tile width in columns (multiple of 16, <= kMmMaxCols)
    const uint16_t *bhi, *blo;  // X planes (bf16 bits), see mm_pack_x_kernel
    int stages;
    uint32_t stage_bytes;
    int raw_depth;         // groups of raw weight bytes staged ahead (2..4)
    uint32_t tmem_cols;
    int a_col;             // first TMEM column of the A stages (after the accumulators)
    int *status;
    // single-job launch: the weight tensor map itself (used when tm0_set; a map in the
    // kernel's parameters needs no proxy fence)
    int tm0_set;
    alignas(64) uint8_t tm0[128];
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

// D (TMEM) (+)= A (TMEM, lane = row, 8 columns = 16 bf16 of K) x B (shared memory).
__device__ __forceinline__ void umma_bf16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t b,
                                             uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 8 consecutive TMEM columns of this warp's 32 lanes <- 8 words per thread.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t *v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
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

// One box of a 3-D tensor map in global memory -> shared memory, completion on `bar`.
// The map was written by the host before the launch; the acquire fence orders this
// thread's use of it through the tensor-map proxy.
__device__ __forceinline__ void tmap_acquire(const void *tmap) {
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(tmap) : "memory");
}
__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap, int x, int y, int z,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_plain(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier `id` over the gate and MMA warps (64 threads); returns the OR of `pred`.
__device__ __forceinline__ bool gate_sync_or(int id, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.or.pred p, %2, 64, q;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id)
        : "memory");
    return r != 0;
}

// 8 TMEM columns of this warp's 32 lanes starting at `taddr`.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float *v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint16_t bf16_bits(float v) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}
__device__ __forceinline__ float bf16_val(uint16_t b) {
    return __bfloat162float(__ushort_as_bfloat16(b));
}

__device__ __forceinline__ const MmJob &job_of(const MmParams &P, int j) {
    return P.jobs ? P.jobs[j] : P.job0;
}

// ---------------------------------------------------------------- X pre-pass
// X (column n at x + col(n) * ldx, K floats) -> two bf16 planes (hi, lo) laid out
// [group g][n/8][kc][n%8][8 positions], kc < (G+16)/8: every (group, 8-column block) is
// (G+16)*16 bytes of K-major core matrices.  Chunks kc < G/8 hold columns
// g*G + 8*kc + (0,4,1,5,2,6,3,7); chunk G/8 of the hi plane holds the zero-term operand
// (X1, X2, X3, X1, X2, X3, 0, 0) of the group sum X_g = sum x (fp32, k < K); everything
// else (columns >= N, k >= K, the lo plane's extra chunks) is zero.
// With u set, the column's values are SwiGLU(x, u) = x / (1 + exp(-x)) * u (the
// reference's silu and product roundings) instead of x.
// One warp per (group, 8-column block): lane l takes column l/4 and the G/4 consecutive
// K values (l%4)*G/4 .. (coalesced), which are whole 8-position chunks, so each lane
// builds its 16-byte chunk words in registers and the 8 lanes of a chunk store 128
// contiguous bytes.  A CTA's 8 warps take 8 consecutive groups of one column block.
constexpr int kPackWarps = 8;

__device__ __forceinline__ float pack_value(float g, const float *u, size_t i) {
    if (!u) return g;
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u[i]);
}

// Grouped form: the 8-column blocks of all jobs are numbered together (job j's first
// block is col0/8), map[b] is the job of block b and *count the blocks in use.
template <int G>
__global__ void __launch_bounds__(kPackWarps * 32) mm_pack_x_kernel(const MmPackJob job0,
                                                                    const MmPackJob *__restrict__ jobs,
                                                                    const int *__restrict__ map,
                                                                    const int *__restrict__ count,
                                                                    int K, int ng, int nb_grid,
                                                                    uint16_t *__restrict__ bhi,
                                                                    uint16_t *__restrict__ blo) {
    constexpr int CK = (G + 16) / 8;
    constexpr int PER = G / 4;   // values per lane: PER / 8 whole chunks
    constexpr int NCH = PER / 8;
    const int gq = blockIdx.x / nb_grid, gb = blockIdx.x % nb_grid;
    MmPackJob jb;
    int nb;
    if (map) {
        if (gb >= *count) return;  // uniform
        jb = jobs[map[gb]];
        nb = gb - jb.col0 / 8;
    } else {
        jb = job0;
        nb = gb;
    }
    const int npad = (jb.N + 15) & ~15;
    if (nb >= npad / 8) return;  // uniform
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = gq * kPackWarps + warp;
    if (g >= ng) return;  // warp-uniform; no CTA barrier below
    const int c = lane >> 2, part = lane & 3;
    const int n = nb * 8 + c;
    const size_t row = n < jb.N ? (size_t)(jb.cols ? jb.cols[n] : n) * jb.ldx : 0;
    const float *src = n < jb.N ? jb.x + row : nullptr;
    const int k0 = g * G + part * PER;
    float v[PER];
    if (src && k0 + PER <= K && (((uintptr_t)(src + k0)) & 15) == 0 &&
        (!jb.u || (((uintptr_t)(jb.u + row + k0)) & 15) == 0)) {
#pragma unroll
        for (int i = 0; i < PER; i += 4) {
            const float4 f = *reinterpret_cast<const float4 *>(src + k0 + i);
            v[i] = f.x, v[i + 1] = f.y, v[i + 2] = f.z, v[i + 3] = f.w;
        }
        if (jb.u) {
#pragma unroll
            for (int i = 0; i < PER; ++i) v[i] = pack_value(v[i], jb.u, row + k0 + i);
        }
    } else {
#pragma unroll
        for (int i = 0; i < PER; ++i)
            v[i] = (src && k0 + i < K) ? pack_value(src[k0 + i], jb.u, row + k0 + i) : 0.0f;
    }
    float xs = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; ++i) xs = __fadd_rn(xs, v[i]);
    xs = __fadd_rn(xs, __shfl_xor_sync(0xffffffffu, xs, 1));
    xs = __fadd_rn(xs, __shfl_xor_sync(0xffffffffu, xs, 2));
    const size_t base = (size_t)jb.b_off + ((size_t)g * (npad / 8) + nb) * CK * 64 + (size_t)c * 8;
    uint4 *dh = reinterpret_cast<uint4 *>(bhi + base);  // chunk kc at dh[kc * 8]
    uint4 *dl = reinterpret_cast<uint4 *>(blo + base);
#pragma unroll
    for (int q = 0; q < NCH; ++q) {  // position 2p+e of a chunk holds its column p + 4e
        uint32_t h[4], l[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const float a = v[8 * q + p], b = v[8 * q + p + 4];
            const uint16_t h0 = bf16_bits(a), h1 = bf16_bits(b);
            const uint16_t l0 = bf16_bits(__fsub_rn(a, bf16_val(h0)));
            const uint16_t l1 = bf16_bits(__fsub_rn(b, bf16_val(h1)));
            h[p] = (uint32_t)h0 | ((uint32_t)h1 << 16);
            l[p] = (uint32_t)l0 | ((uint32_t)l1 << 16);
        }
        const int kc = part * NCH + q;
        dh[kc * 8] = make_uint4(h[0], h[1], h[2], h[3]);
        dl[kc * 8] = make_uint4(l[0], l[1], l[2], l[3]);
    }
    if (part == 0) {  // the zero-term chunk and the padding chunk of this column
        const uint16_t x1 = bf16_bits(xs);
        const float r1 = __fsub_rn(xs, bf16_val(x1));
        const uint16_t x2 = bf16_bits(r1);
        const uint16_t x3 = bf16_bits(__fsub_rn(r1, bf16_val(x2)));
        dh[(G / 8) * 8] = make_uint4((uint32_t)x1 | ((uint32_t)x2 << 16),
                                     (uint32_t)x3 | ((uint32_t)x1 << 16),
                                     (uint32_t)x2 | ((uint32_t)x3 << 16), 0u);
        dh[(G / 8 + 1) * 8] = make_uint4(0u, 0u, 0u, 0u);
        dl[(G / 8) * 8] = make_uint4(0u, 0u, 0u, 0u);
        dl[(G / 8 + 1) * 8] = make_uint4(0u, 0u, 0u, 0u);
    }
}

// ---------------------------------------------------------------- weight repack
// Interleaved i4 rows (runtime/tiny_format.h:66-77) -> tile-contiguous blocks: for every
// 256-row tile and group g, the 256 rows' group bytes ([scale][zero][G/2 nibble bytes])
// back to back, rows past M zero.  Bytes are copied unchanged (a pure permutation of
// 4-byte words), so the block of (tile, g) holds exactly what the row layout held.
__global__ void mm_repack_w_kernel(const uint32_t *__restrict__ w, int M, int ng, int wr,
                                   uint32_t *__restrict__ out, long long total) {
    for (long long o = blockIdx.x * (long long)blockDim.x + threadIdx.x; o < total;
         o += (long long)gridDim.x * blockDim.x) {
        const int wd = (int)(o % wr);
        const long long rest = o / wr;
        const int r = (int)(rest % kTileRows);
        const long long tg = rest / kTileRows;
        const int g = (int)(tg % ng);
        const long long tile = tg / ng;
        const long long row = tile * kTileRows + r;
        out[o] = row < M ? w[(size_t)row * ng * wr + (size_t)g * wr + wd] : 0u;
    }
}

// ---------------------------------------------------------------- the GEMM
template <int G>
__global__ void __launch_bounds__(kMmThreads, 1) mm_i4_tc_kernel(const __grid_constant__ MmParams P) {
    constexpr int CK = (G + 16) / 8;          // 16-byte chunks per row of a stage
    constexpr uint32_t SBO = CK * 128;        // bytes between 8-row groups (B operand)
    constexpr int KS = G / 16 + 1;            // MMA K steps per group (the last: zero term)
    constexpr int GB = 4 + G / 2;             // bytes per group of a weight row
    constexpr int WR = GB / 4;                // words per row of a group (odd)
    constexpr uint32_t kRawBytes = kTileRows * GB;  // one group of the tile's rows
    constexpr uint32_t kBlkBytes = kGpb * kRawBytes;  // one staged weight block
    extern __shared__ __align__(1024) uint8_t smem[];
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);  // [kMmMaxStages] A built
    uint64_t *empty = full + kMmMaxStages;                 // [kMmMaxStages] stage consumed
    uint64_t *tfull = empty + kMmMaxStages;                // [2] accumulator of row half h ready
    uint64_t *tempty = tfull + 2;                          // [2] accumulator of row half h drained
    uint64_t *done = tempty + 2;
    uint64_t *rawbar = done + 1;                           // [kMaxRaw] weight block landed
    uint64_t *rawfree = rawbar + kMaxRaw;                  // [kMaxRaw] weight block read
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(rawfree + kMaxRaw);
    float *scl = reinterpret_cast<float *>(smem + 1024);   // [kSclRing][256] group scales
    uint8_t *stage_base = smem + 1024 + kSclRing * kTileRows * 4;
    __shared__ int s_err;

    // ---- which tile: job j, rows m0.., columns n0..n0+nw
    int j = 0;
    const int tile = blockIdx.x;
    if (P.tile_job) {
        if (tile >= *P.n_tiles) return;  // uniform: before any barrier or TMEM use
        j = P.tile_job[tile];
    } else {  // last job whose first tile is at or before this one
        int hi = P.n_jobs - 1;
        while (j < hi) {
            const int mid = (j + hi + 1) >> 1;
            if (tile >= job_of(P, mid).tile_begin) j = mid;
            else hi = mid - 1;
        }
    }
    const MmJob &job = job_of(P, j);
    const int local = tile - job.tile_begin;
    const int mt = (job.M + kTileRows - 1) / kTileRows;
    const int npad = (job.N + 15) & ~15;
    const int m0 = (local % mt) * kTileRows;
    const int n0 = (local / mt) * P.nt;
    const int nw = min(P.nt, npad - n0);           // this tile's MMA N (multiple of 16)
    const uint32_t b_bytes = (uint32_t)nw * CK * 16u;  // one X plane of a stage
    const uint32_t stage_bytes = P.stage_bytes;
    const int ng = P.ng, S = P.stages, RD = P.raw_depth;
    uint8_t *raw = stage_base + (size_t)S * stage_bytes;  // [RD] weight blocks
    // a block holds groups 4b .. 4b+3 of the tile's 256 rows: from the tensor map as
    // [row][4 groups] (row t's group c at word t * 4 WR + c * WR), repacked as
    // [group][row] (at word c * 256 WR + t * WR)
    const void *tmap = P.tm0_set ? static_cast<const void *>(P.tm0) : job.tmap;
    const bool tmw = tmap != nullptr;
    const int nblk = (ng + kGpb - 1) / kGpb;
    const int w_rs = tmw ? kGpb * WR : WR, w_gs = tmw ? WR : kTileRows * WR;

    if (t == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], kProdWarps + 1);  // 8 producer warps + the X-plane copies
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kEpiWarps / 2);
        }
        mbar_init(done, 1);
        for (int r = 0; r < RD; ++r) {
            mbar_init(&rawbar[r], 1);
            mbar_init(&rawfree[r], kProdWarps);
        }
        fence_mbar_init();
        s_err = 0;
    }
    if (warp == kMmaWarp) {  // TMEM: 2 buffers x 2 row halves x nt fp32 columns x 128 lanes
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

    if (warp < kProdWarps) {
        // ---------------- A operand: thread = weight row t of the tile, codes widened to
        // bf16 from the tile-contiguous weight block of the group (mm_repack_w_kernel) and
        // stored to the stage's TMEM columns of its row half (lane = row; warp w may reach
        // lanes 32 * (w % 4) ..); K step kk = 8 columns, K positions 2c, 2c+1 in column c
        const uint32_t a_lane = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        const int half = t >> 7;
        const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.0f, 128.0f);
        for (int i = 0; i < ng; ++i) {
            const int s = i % S, b = i / kGpb, r = b % RD, c = i - b * kGpb;
            bool ok = true;
            if (i >= S) ok = mbar_wait_sleep(&empty[s], (uint32_t)((i / S) - 1) & 1u, kWaitCycles);
            if (ok) ok = mbar_wait_sleep(&rawbar[r], (uint32_t)(b / RD) & 1u, kWaitCycles);
            if (!__all_sync(0xffffffffu, ok)) {  // warp-uniform stop; the MMA side times out
                if (lane == 0) s_err = 1;
                break;
            }
            tc_fence_after();  // the MMAs that read this stage's TMEM columns are complete
            const uint32_t *d =
                reinterpret_cast<const uint32_t *>(raw + (size_t)r * kBlkBytes) + t * w_rs + c * w_gs;
            uint32_t wv[WR];
#pragma unroll
            for (int q = 0; q < WR; ++q) wv[q] = d[q];  // [0] header, then nibble words
            __syncwarp();
            if (lane == 0 && (c == kGpb - 1 || i == ng - 1)) mbar_arrive_plain(&rawfree[r]);  // slot r read
            const uint32_t ta = a_lane + (uint32_t)(P.a_col + (s * 2 + half) * KS * 8);
#pragma unroll
            for (int kk = 0; kk < G / 16; ++kk) {  // 16 codes -> 8 words: (q0,q4) (q1,q5) ...
                uint32_t o[8];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t w = wv[1 + 2 * kk + h];
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const uint32_t wide = ((w >> (4 * p)) & 0x000F000Fu) | 0x43004300u;  // 128 + q
                        const __nv_bfloat162 v = __hsub2(*reinterpret_cast<const __nv_bfloat162 *>(&wide), k128);
                        o[4 * h + p] = *reinterpret_cast<const uint32_t *>(&v);
                    }
                }
                tmem_st8(ta + (uint32_t)(kk * 8), o);
            }
            {  // zero term: -(z1, z1, z1, z2, z2, z2, 0, ...), z = z1 + z2 exactly
                const float z = h2f((uint16_t)(wv[0] >> 16));
                const uint16_t z1 = bf16_bits(-z);
                const uint16_t z2 = bf16_bits(__fsub_rn(-z, bf16_val(z1)));
                const uint32_t o[8] = {(uint32_t)z1 | ((uint32_t)z1 << 16),
                                       (uint32_t)z1 | ((uint32_t)z2 << 16),
                                       (uint32_t)z2 | ((uint32_t)z2 << 16), 0u, 0u, 0u, 0u, 0u};
                tmem_st8(ta + (uint32_t)((G / 16) * 8), o);
            }
            scl[(i % kSclRing) * kTileRows + t] = h2f((uint16_t)(wv[0] & 0xFFFFu));  // for the epilogue
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_plain(&full[s]);
        }
    } else if (warp < kMmaWarp) {
        // ---------------- epilogue: y += s_g * P_g per group, in registers; warp e owns
        // row half e/4, TMEM lane quarter warp%4, all nw columns
        const int e = warp - kProdWarps;
        const int half = e >> 2;
        const int quarter = warp & 3;  // TMEM lanes this warp may access
        const int rl = 128 * half + 32 * quarter + lane;  // row within the tile
        const int row = m0 + rl;
        // accumulator of row half h = TMEM columns [2h * nt, + 2nw): P of the hi plane in
        // the first nw columns, of the lo plane in the next nw
        const uint32_t lane_addr = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(half * 2 * P.nt);
        float y[kMmMaxCols];
#pragma unroll
        for (int c = 0; c < kMmMaxCols; ++c) y[c] = 0.0f;
        for (int i = 0; i < ng; ++i) {
            if (!__all_sync(0xffffffffu, mbar_wait_sleep(&tfull[half], (uint32_t)i & 1u, kWaitCycles))) {
                if (lane == 0) s_err = 1;
                break;
            }
            tc_fence_after();
            const float sc = scl[(i % kSclRing) * kTileRows + rl];
#pragma unroll
            for (int h = 0; h < kMmMaxCols / 8; ++h) {  // 8 columns (hi and lo) at a time
                if (h * 8 < nw) {
                    float v[8], u[8];
                    tmem_ld8(lane_addr + (uint32_t)(h * 8), v);
                    tmem_ld8(lane_addr + (uint32_t)(nw + h * 8), u);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 8; ++c) y[h * 8 + c] = fmaf(sc, v[c] + u[c], y[h * 8 + c]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_plain(&tempty[half]);
        }
        if (row < job.M) {
#pragma unroll
            for (int c = 0; c < kMmMaxCols; ++c) {
                const int n = n0 + c;
                if (c < nw && n < job.N) {
                    const size_t o = (size_t)n * job.ldy + row;
                    float v = y[c];
                    if (job.bias) v = v + job.bias[row];
                    job.y[o] = job.resid ? job.resid[o] + v : v;
                }
            }
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer (lane 0): per group and row half, G/16 K steps of
        // codes (TMEM) x [X hi | X lo] (shared memory; one MMA of N = 2nw, the lo plane's
        // rows following the hi plane's), then the zero term.  Each half has one
        // accumulator: the epilogue drains half 0 of group i while the MMAs of half 1 run,
        // and the reverse.  The gate warp has done the waiting when each barrier opens.
        const uint32_t idesc = umma_idesc_bf16(2 * nw);
        bool bad = false;
        for (int i = 0; i < ng; ++i) {
            const int s = i % S;
            bad = gate_sync_or(kBarStage, bad);  // A and X planes of group i in place
            const uint32_t bh = smem_u32(stage_base + (size_t)s * stage_bytes);
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                bad = gate_sync_or(kBarHalf0 + hf, bad);  // half hf of group i-1 drained
                if (!bad && lane == 0) {
                    tc_fence_after();
                    const uint32_t ta = tmem + (uint32_t)(P.a_col + (s * 2 + hf) * KS * 8);
                    const uint32_t dd = tmem + (uint32_t)(hf * 2 * P.nt);
#pragma unroll
                    for (int kk = 0; kk < G / 16; ++kk) {
                        const uint32_t o = (uint32_t)kk * 256u;  // two 16-byte core-matrix columns
                        umma_bf16_ta(dd, ta + (uint32_t)(kk * 8), umma_desc(bh + o, 128, SBO), idesc,
                                     kk > 0 ? 1u : 0u);
                    }
                    const uint32_t oz = (uint32_t)(G / 16) * 256u;  // zero term
                    umma_bf16_ta(dd, ta + (uint32_t)((G / 16) * 8), umma_desc(bh + oz, 128, SBO), idesc, 1u);
                    umma_commit(&tfull[hf]);  // half hf holds P_i
                }
                __syncwarp();
            }
            if (!bad && lane == 0) umma_commit(&empty[s]);  // stage s free once read
            __syncwarp();
        }
        if (lane == 0) {
            if (bad) s_err = 1;
            umma_commit(done);  // every MMA issued above has completed
            if (!mbar_wait_sleep(done, 0u, kWaitCycles)) s_err = 1;
        }
    } else if (warp == kGateWarp) {
        // ---------------- gate: the MMA warp's waits, met at the named barriers in the
        // same order; after a timeout it keeps meeting them without waiting
        bool bad = false;
        for (int i = 0; i < ng; ++i) {
            const int s = i % S;
            if (!bad && lane == 0) bad = !mbar_wait_sleep(&full[s], (uint32_t)(i / S) & 1u, kWaitCycles);
            bad = gate_sync_or(kBarStage, __shfl_sync(0xffffffffu, bad, 0));
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                if (!bad && i >= 1 && lane == 0)
                    bad = !mbar_wait_sleep(&tempty[hf], (uint32_t)(i - 1) & 1u, kWaitCycles);
                bad = gate_sync_or(kBarHalf0 + hf, __shfl_sync(0xffffffffu, bad, 0));
            }
        }
        if (bad && lane == 0) s_err = 1;
    } else if (lane == 0) {
        // ---------------- loader: weight blocks RD - 1 groups ahead, X planes per stage
        // weight block b: groups 4b .. 4b+3 of this row tile.  Tensor map: the box at
        // word 4b * WR of rows m0 .. m0+255 of matrix tz (x a multiple of 16 bytes; rows past
        // M read as zeros).  Repacked: the tile's groups are back to back, one bulk copy.
        const uint8_t *wblk = job.w + (size_t)(local % mt) * ng * kRawBytes;
        if (tmw && !P.tm0_set) tmap_acquire(tmap);  // written to global memory by the host
        auto issue_raw = [&](int b) {
            uint64_t *bar = &rawbar[b % RD];
            uint8_t *dst = raw + (size_t)(b % RD) * kBlkBytes;
            if (tmw) {
                mbar_arrive_expect_tx(bar, kBlkBytes);
                tma_load_3d(dst, tmap, b * kGpb * WR, m0, job.tz, bar);
            } else {
                const uint32_t bytes = (uint32_t)min(kGpb, ng - b * kGpb) * kRawBytes;
                const uint8_t *src = wblk + (size_t)b * kBlkBytes;
                mbar_arrive_expect_tx(bar, bytes);
                for (uint32_t o = 0; o < bytes; o += 16384u)
                    bulk_g2s(dst + o, src + o, min(16384u, bytes - o), bar);
            }
        };
        int raw_issued = 0, b_issued = 0;
        bool ok = true;
        for (int b = 0; b < RD - 1 && b < nblk; ++b) issue_raw(b), raw_issued = b + 1;
        for (int g = 0; g < ng && ok; ++g) {
            const int b = g / kGpb, br = b + RD - 1;  // block br into the slot block b - 1 used
            if (g == b * kGpb && br < nblk) {
                if (b >= 1) ok = mbar_wait_sleep(&rawfree[(b - 1) % RD], (uint32_t)((b - 1) / RD) & 1u, kWaitCycles);
                if (!ok) break;
                issue_raw(br);
                raw_issued = br + 1;
            }
            const int s = g % S;  // X planes of group g into stage s
            if (g >= S) ok = mbar_wait_sleep(&empty[s], (uint32_t)((g / S) - 1) & 1u, kWaitCycles);
            if (!ok) break;
            uint8_t *st = stage_base + (size_t)s * stage_bytes;
            const size_t blk = ((size_t)g * (npad / 8) + n0 / 8) * (CK * 64);  // bf16 elements
            mbar_arrive_expect_tx(&full[s], 2u * b_bytes);
            bulk_g2s(st, P.bhi + job.b_off + blk, b_bytes, &full[s]);
            bulk_g2s(st + b_bytes, P.blo + job.b_off + blk, b_bytes, &full[s]);
            b_issued = g + 1;
        }
        if (!ok) s_err = 1;
        // copies still in flight land before shared memory is released
        for (int b = max(0, raw_issued - RD); b < raw_issued; ++b)
            if (!mbar_wait_sleep(&rawbar[b % RD], (uint32_t)(b / RD) & 1u, kWaitCycles)) s_err = 1;
        for (int g = max(0, b_issued - S); g < b_issued; ++g)
            if (!mbar_wait_sleep(&full[g % S], (uint32_t)(g / S) & 1u, kWaitCycles)) s_err = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(P.tmem_cols)
                     : "memory");
    }
    if (t == 0 && s_err && P.status) atomicExch(P.status, kDevTimeoutTma);
}

KernelSmem g_mm_smem_set[3];

template <int G>
uint32_t mm_stage_bytes(int nt) {  // the X hi and lo planes of one group (B operand)
    return (uint32_t)(2 * nt) * ((G + 16) / 8) * 16u;
}

template <int G>
int launch_grouped_g(MmParams &P, int total_tiles, cudaStream_t st, int gi) {
    P.stage_bytes = mm_stage_bytes<G>(P.nt);
    int limit = 0;
    TQ_CUDA_TRY(smem_limit_once(mm_i4_tc_kernel<G>, g_mm_smem_set[gi], &limit));
    const int fixed = 1024 + kSclRing * kTileRows * 4;
    const int raw_group = kGpb * kTileRows * (4 + G / 2);  // bytes of one staged weight block
    // TMEM: 4 nt accumulator columns (two row halves of [hi | lo]), then per stage two row
    // halves of (G/16 + 1) K steps of 8 columns of A
    const int a_stage_cols = 2 * (G / 16 + 1) * 8;
    const int tmem_stages = (kTmemCols - 4 * P.nt) / a_stage_cols;
    TQ_CHECK_ARG(tmem_stages >= 1, "matmul_i4: tile of %d columns leaves no TMEM for A", P.nt);
    P.tmem_cols = kTmemCols;
    P.a_col = 4 * P.nt;
    // deepest pipeline that fits: operand stages first (2 wanted), then the weight ring
    int stages = 0, rd = 0;
    for (int s = std::min({kMmMaxStages, P.ng, tmem_stages}); s >= 1 && !stages; --s)
        for (int r = kMaxRaw; r >= 2; --r)
            if (fixed + s * (int)P.stage_bytes + r * raw_group <= limit && (s >= 2 || r == 2)) {
                stages = s;
                rd = r;
                break;
            }
    TQ_CHECK_ARG(stages >= 1, "matmul_i4: tile of %d columns does not fit shared memory", P.nt);
    P.stages = stages;
    P.raw_depth = rd;
    const size_t smem = fixed + (size_t)stages * P.stage_bytes + (size_t)rd * raw_group;
    mm_i4_tc_kernel<G><<<total_tiles, kMmThreads, smem, st>>>(P);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

}  // namespace

bool mm_group_supported(int G) { return G == 32 || G == 64 || G == 128; }

size_t mm_x_planes_bytes(int K, int N, int G) {
    if (!mm_group_supported(G)) return 0;
    const size_t ng = (size_t)(K + G - 1) / G;
    const size_t npad = (size_t)(N + 15) & ~(size_t)15;
    return 2 * ng * (size_t)(G + 16) * npad * 2;  // hi + lo bf16
}

size_t mm_repacked_bytes(int M, int K, int G) {
    if (!mm_group_supported(G)) return 0;
    const size_t ng = (size_t)(K + G - 1) / G;
    const size_t mt = (size_t)(M + kTileRows - 1) / kTileRows;
    return mt * ng * kTileRows * (size_t)(4 + G / 2);
}

bool mm_encode_weight_map(const uint8_t *w, int M, int K, int G, int E, size_t stride,
                          void *map128) {
    if (!mm_group_supported(G) || M <= 0 || K <= 0 || E <= 0) return false;
    const int ng = (K + G - 1) / G, wr = (4 + G / 2) / 4;
    const size_t row = (size_t)ng * wr * 4;  // bytes of one interleaved row
    if (ng % kGpb != 0 || row % 16 != 0 || (((uintptr_t)w) & 15) != 0) return false;
    // matrices apart by `stride` (one matrix: its own length, rounded up to 16 bytes)
    const size_t zs = E > 1 ? stride : ((row * (size_t)M + 15) & ~(size_t)15);
    if (zs % 16 != 0 || zs < row * (size_t)M) return false;
    // 32-bit words: x over a row's ng * WR words, y over rows, z over matrices; the box is
    // kGpb groups (a multiple of 16 bytes for every supported G) of 256 rows
    const cuuint64_t dims[3] = {(cuuint64_t)ng * wr, (cuuint64_t)M, (cuuint64_t)E};
    const cuuint64_t strides[2] = {(cuuint64_t)row, (cuuint64_t)zs};
    const cuuint32_t box[3] = {(cuuint32_t)(kGpb * wr), (cuuint32_t)kTileRows, 1u};
    const cuuint32_t elem[3] = {1u, 1u, 1u};
    // the driver's encoder, looked up at run time (the library links no driver API, so it
    // loads on hosts without a GPU driver)
    using Encode = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static Encode encode = [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                             &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            fn = nullptr;
        }
        return reinterpret_cast<Encode>(fn);
    }();
    if (!encode) return false;
    CUtensorMap m;
    const CUresult r = encode(
        &m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t *>(w), dims, strides, box, elem,
        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    static_assert(sizeof(CUtensorMap) == 128, "CUtensorMap size");
    memcpy(map128, &m, sizeof(m));
    return true;
}

int launch_mm_repack_w(const uint8_t *w, int M, int K, int G, uint8_t *out, cudaStream_t st) {
    TQ_CHECK_ARG(mm_group_supported(G), "matmul_i4: group_size %d not 32, 64 or 128", G);
    TQ_CHECK_ARG((((uintptr_t)w) & 3) == 0 && (((uintptr_t)out) & 15) == 0,
                 "matmul_i4: weights not 4-byte / repack buffer not 16-byte aligned");
    const int ng = (K + G - 1) / G, wr = (4 + G / 2) / 4;
    const long long total = (long long)(mm_repacked_bytes(M, K, G) / 4);
    if (total == 0) return TQB200_OK;
    const int threads = 256;
    const int blocks = (int)std::min<long long>((total + threads - 1) / threads, 148LL * 16);
    mm_repack_w_kernel<<<blocks, threads, 0, st>>>(reinterpret_cast<const uint32_t *>(w), M, ng,
                                                   wr, reinterpret_cast<uint32_t *>(out), total);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

size_t mm_scratch_bytes(int M, int K, int N, int G) {
    if (!mm_group_supported(G)) return 0;
    const size_t a = (mm_repacked_bytes(M, K, G) + 255) & ~(size_t)255;
    return a + mm_x_planes_bytes(K, N, G);
}

// Column tile width by a cost model: a CTA's time per group is about (36 + nt) units (each
// MMA instruction has a fixed cost of about 36 columns' worth; measured), and the launch
// takes as many such CTA times as it has waves over the SMs.  Ties go to the wider tile.
int mm_tile_width(int M, int N) {
    const int npad = (N + 15) & ~15;
    const int mt = (M + kTileRows - 1) / kTileRows;
    const int widest = std::min(npad, kMmMaxCols);
    const int sms = num_sms();
    int best = widest;
    long long best_cost = -1;
    for (int nt = widest; nt >= 16; nt -= 16) {
        const long long tiles = (long long)mt * ((npad + nt - 1) / nt);
        const long long cost = ((tiles + sms - 1) / sms) * (36 + nt);
        if (best_cost < 0 || cost < best_cost) {
            best = nt;
            best_cost = cost;
        }
    }
    return best;
}

int launch_matmul_i4_grouped(const MmJob *host_jobs, const MmJob *dev_jobs, int n_jobs, int K,
                             int G, int nt, const uint16_t *bhi, const uint16_t *blo, int total_tiles,
                             int *status, cudaStream_t st, const void *map128) {
    TQ_CHECK_ARG(n_jobs >= 1, "matmul_i4: no jobs");
    TQ_CHECK_ARG(mm_group_supported(G), "matmul_i4 (tensor cores): group_size %d not 32, 64 or 128", G);
    TQ_CHECK_ARG(nt % 16 == 0 && nt >= 16 && nt <= kMmMaxCols, "matmul_i4: bad tile width %d", nt);
    TQ_CHECK_ARG(((uintptr_t)bhi & 15) == 0 && ((uintptr_t)blo & 15) == 0, "matmul_i4: X planes not 16-byte aligned");
    if (total_tiles == 0) return TQB200_OK;
    MmParams P{};
    if (dev_jobs == nullptr) P.job0 = host_jobs[0];
    if (map128) {
        TQ_CHECK_ARG(dev_jobs == nullptr, "matmul_i4: a parameter tensor map serves one job");
        memcpy(P.tm0, map128, sizeof(P.tm0));
        P.tm0_set = 1;
    }
    P.jobs = dev_jobs;
    P.n_jobs = dev_jobs ? n_jobs : 1;
    P.K = K;
    P.ng = (K + G - 1) / G;
    P.nt = nt;
    P.bhi = bhi;
    P.blo = blo;
    P.status = status;
    if (G == 32) return launch_grouped_g<32>(P, total_tiles, st, 0);
    if (G == 64) return launch_grouped_g<64>(P, total_tiles, st, 1);
    return launch_grouped_g<128>(P, total_tiles, st, 2);
}

int launch_matmul_i4_planned(const MmJob *dev_jobs, const int *dev_tile_job, const int *dev_n_tiles,
                             int max_tiles, int K, int G, int nt, const uint16_t *bhi,
                             const uint16_t *blo, int *status, cudaStream_t st) {
    TQ_CHECK_ARG(dev_jobs && dev_tile_job && dev_n_tiles, "matmul_i4: planned launch needs its plan");
    TQ_CHECK_ARG(mm_group_supported(G), "matmul_i4 (tensor cores): group_size %d not 32, 64 or 128", G);
    TQ_CHECK_ARG(nt % 16 == 0 && nt >= 16 && nt <= kMmMaxCols, "matmul_i4: bad tile width %d", nt);
    TQ_CHECK_ARG(((uintptr_t)bhi & 15) == 0 && ((uintptr_t)blo & 15) == 0, "matmul_i4: X planes not 16-byte aligned");
    if (max_tiles <= 0) return TQB200_OK;
    MmParams P{};
    P.jobs = dev_jobs;
    P.n_jobs = 0;
    P.tile_job = dev_tile_job;
    P.n_tiles = dev_n_tiles;
    P.K = K;
    P.ng = (K + G - 1) / G;
    P.nt = nt;
    P.bhi = bhi;
    P.blo = blo;
    P.status = status;
    if (G == 32) return launch_grouped_g<32>(P, max_tiles, st, 0);
    if (G == 64) return launch_grouped_g<64>(P, max_tiles, st, 1);
    return launch_grouped_g<128>(P, max_tiles, st, 2);
}

int launch_pack(const MmPackJob &job0, const MmPackJob *jobs, const int *map, const int *count,
                int K, int G, int nb_grid, uint16_t *bhi, uint16_t *blo, cudaStream_t st) {
    TQ_CHECK_ARG(mm_group_supported(G), "matmul_i4: group_size %d not 32, 64 or 128", G);
    if (nb_grid <= 0) return TQB200_OK;
    const int ng = (K + G - 1) / G;
    const long long bx = (long long)((ng + kPackWarps - 1) / kPackWarps) * nb_grid;
    TQ_CHECK_ARG(bx < (1LL << 31), "matmul_i4: X pack grid %lld", bx);
    const int threads = kPackWarps * 32;
    if (G == 32)
        mm_pack_x_kernel<32><<<(unsigned)bx, threads, 0, st>>>(job0, jobs, map, count, K, ng, nb_grid, bhi, blo);
    else if (G == 64)
        mm_pack_x_kernel<64><<<(unsigned)bx, threads, 0, st>>>(job0, jobs, map, count, K, ng, nb_grid, bhi, blo);
    else
        mm_pack_x_kernel<128><<<(unsigned)bx, threads, 0, st>>>(job0, jobs, map, count, K, ng, nb_grid, bhi, blo);
    TQ_CUDA_TRY(cudaGetLastError());
    return TQB200_OK;
}

int launch_mm_pack_x(const float *x, const int *cols, int ldx, int K, int N, int G, uint16_t *bhi,
                     uint16_t *blo, cudaStream_t st, const float *u) {
    MmPackJob j{};
    j.x = x;
    j.u = u;
    j.cols = cols;
    j.ldx = ldx;
    j.N = N;
    j.b_off = 0;
    j.col0 = 0;
    return launch_pack(j, nullptr, nullptr, nullptr, K, G, ((N + 15) & ~15) / 8, bhi, blo, st);
}

int mm_job_tiles(int M, int N, int nt) {
    const int npad = (N + 15) & ~15;
    return ((M + kTileRows - 1) / kTileRows) * ((npad + nt - 1) / nt);
}

long long mm_plane_elems(int K, int N, int G) {
    const long long ng = (K + G - 1) / G;
    const long long npad = (N + 15) & ~15;
    return ng * (G + 16) * npad;
}

int launch_mm_pack_x_mapped(const MmPackJob *dev_jobs, const int *dev_map, const int *dev_count,
                            int max_blocks, int K, int G, uint16_t *bhi, uint16_t *blo, cudaStream_t st) {
    TQ_CHECK_ARG(dev_jobs && dev_map && dev_count, "matmul_i4: mapped X pack needs its map");
    return launch_pack(MmPackJob{}, dev_jobs, dev_map, dev_count, K, G, max_blocks, bhi, blo, st);
}

// Y = W X for one matrix.  scratch (mm_scratch_bytes(M, K, N, G)) receives the
// tile-contiguous weights and the X planes.
int launch_matmul_i4(const uint8_t *w, const float *x, float *y, int M, int K, int N, int G,
                     void *scratch, int *status, cudaStream_t st) {
    TQ_CHECK_ARG(M >= 0 && K > 0 && N >= 0, "matmul_i4: bad shape %d x %d x %d", M, K, N);
    TQ_CHECK_ARG(mm_group_supported(G), "matmul_i4: group_size %d not 32, 64 or 128", G);
    if (M == 0 || N == 0) return TQB200_OK;
    TQ_CHECK_ARG(((uintptr_t)w & 3) == 0, "matmul_i4: weights not 4-byte aligned");
    TQ_CHECK_ARG(((uintptr_t)scratch & 15) == 0, "matmul_i4: scratch not 16-byte aligned");
    const int npad = (N + 15) & ~15;
    uint8_t *wt = static_cast<uint8_t *>(scratch);
    const size_t wbytes = (mm_repacked_bytes(M, K, G) + 255) & ~(size_t)255;
    const size_t plane = mm_x_planes_bytes(K, N, G) / 2;
    uint16_t *bhi = reinterpret_cast<uint16_t *>(wt + wbytes);
    uint16_t *blo = reinterpret_cast<uint16_t *>(wt + wbytes + plane);
    // the weights in place through a tensor map where their rows allow one, else a
    // repacked copy in the scratch
    alignas(64) uint8_t map[128];
    const bool mapped = mm_encode_weight_map(w, M, K, G, 1, 0, map);
    int r = mapped ? TQB200_OK : launch_mm_repack_w(w, M, K, G, wt, st);
    if (r != TQB200_OK) return r;
    r = launch_mm_pack_x(x, nullptr, K, K, N, G, bhi, blo, st);
    if (r != TQB200_OK) return r;
    const int nt = mm_tile_width(M, N);
    MmJob j{};
    j.w = wt;
    j.y = y;
    j.M = M;
    j.N = N;
    j.ldy = M;
    j.tile_begin = 0;
    j.b_off = 0;
    const int tiles = ((M + kTileRows - 1) / kTileRows) * ((npad + nt - 1) / nt);
    return launch_matmul_i4_grouped(&j, nullptr, 1, K, G, nt, bhi, blo, tiles, status, st,
                                    mapped ? map : nullptr);
}

}  // namespace tqb200
