// kernels.h — internal (C++) launch API shared by capi.cu and engine.cu.
// All launchers are stream-ordered, take device pointers, and return a
// TQB200_* status (errors recorded through set_error).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace tqb200 {

int num_sms();

// ------------------------------------------------------------------ in-graph timeline
// Global-timer stamps of one launch, per decode step: every CTA (up to kStampCtas of
// them) writes three words of its own with plain stores (no atomics): when its last
// thread entered, when that thread got past the dependency wait (griddepcontrol.wait
// returns once the previous kernel has completed), and when it finished.  The host
// takes, per launch, the first wait over the CTAs; a launch's in-step time runs from
// its first wait to the next stamped launch's first wait (the last one's: to its last
// exit), so the times of a step's launches do not overlap and add up to the step.  The
// stamps are compiled only into a kernel's ON = true instantiation, which the launchers
// pick when Stamp::base is set, and the timer values stay in registers until the
// thread's exit, so a stamped CTA waits on no extra memory access or barrier.
constexpr int kStampCtas = 256;  // CTAs of a launch with a record (lower linear index)
struct Stamp {
    unsigned long long *base = nullptr;  // this launch's kStampCtas x 3 words for step 0
    const int *step = nullptr;           // device step counter selecting the record
    int stride = 0;                      // words between consecutive steps' records
    int cap = 0;                         // steps with a record
};

#if defined(__CUDACC__)
struct StampRegs {
    unsigned long long t_enter = 0, t_wait = 0;
    int step = -1;
};
__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// The CTA's last thread stamps: thread 0 of several kernels issues their bulk copies
// at entry, which a timer read must not delay.
__device__ __forceinline__ bool stamp_thread() {
    return threadIdx.x == blockDim.x - 1 && threadIdx.y == blockDim.y - 1 &&
           threadIdx.z == blockDim.z - 1;
}
// At kernel entry.
template <bool ON>
__device__ __forceinline__ void stamp_enter(const Stamp &s, StampRegs &r) {
    if constexpr (ON)
        if (stamp_thread()) r.t_enter = global_timer_ns();
}
// Just before griddepcontrol.wait: the step counter's load (used at the exit).
template <bool ON>
__device__ __forceinline__ void stamp_step(const Stamp &s, StampRegs &r) {
    if constexpr (ON)
        if (stamp_thread()) r.step = *s.step;
}
// Right after griddepcontrol.wait.
template <bool ON>
__device__ __forceinline__ void stamp_waited(const Stamp &s, StampRegs &r) {
    if constexpr (ON)
        if (stamp_thread()) r.t_wait = global_timer_ns();
}
// At the stamping thread's exit.
template <bool ON>
__device__ __forceinline__ void stamp_exit(const Stamp &s, const StampRegs &r) {
    if constexpr (ON) {
        const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
        if (stamp_thread() && r.step >= 0 && r.step < s.cap && cta < (unsigned)kStampCtas) {
            unsigned long long *w = s.base + (size_t)r.step * s.stride + 3 * (size_t)cta;
            w[0] = r.t_enter;
            w[1] = r.t_wait;
            w[2] = global_timer_ns();
        }
    }
}
#endif

// ------------------------------------------------------------------ peer exchange
// Tensor-parallel all-gather fused into the kernel that produces the rows (one process
// per GPU; every rank's exchange arena has the same layout and is mapped into every
// other rank's address space).  The producer stores each of its output rows into its
// own buffer and, at the same offset, into every peer's (NVLink stores); each CTA then
// fences (system scope) and takes a ticket, and the launch's last CTA adds 1 to the
// exchange's arrival counter on every rank (a system-scope release).  A consumer waits,
// after its dependency wait and before reading the buffer, until its own counter reaches
// epoch x ranks (one thread of each CTA polls with an acquire load, bounded in time).
// The counters only grow: epoch counts decode steps (the embed kernel advances it), so
// no counter is ever reset while a peer may still add to it.
constexpr int kMaxPeers = 7;  // up to 8 ranks
struct XPut {
    int n_peers = 0;
    long long delta[kMaxPeers] = {};       // peer arena address minus local (bytes)
    unsigned long long *arrive = nullptr;  // local address of this exchange's counter
    unsigned int *ticket = nullptr;        // local CTA-completion ticket of this exchange
};
struct XWait {
    const unsigned long long *arrive = nullptr;  // this rank's counter of the exchange
    const unsigned int *epoch = nullptr;         // decode steps so far (device)
    unsigned int ranks = 0;                      // arrivals per step
};

#if defined(__CUDACC__)
constexpr unsigned long long kXWaitNs = 20000000000ull;  // 20 s: ranks may start apart

// Stores v at p and at p's offset in every peer's arena.
template <typename T>
__device__ __forceinline__ void xput_val(const XPut &x, T *p, T v) {
    *p = v;
    for (int i = 0; i < x.n_peers; ++i)
        *reinterpret_cast<T *>(reinterpret_cast<char *>(p) + x.delta[i]) = v;
}
// Called by every thread of the CTA after its last store of exchanged rows.
__device__ __forceinline__ void xput_arrive(const XPut &x) {
    if (!x.arrive) return;
    __syncthreads();
    if (threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0) {
        __threadfence_system();  // this CTA's stores, local and remote, before its ticket
        const unsigned int n = gridDim.x * gridDim.y * gridDim.z;
        if ((atomicAdd(x.ticket, 1u) + 1u) % n == 0u) {  // the launch's last CTA
            __threadfence_system();
            asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(x.arrive) : "memory");
            for (int i = 0; i < x.n_peers; ++i) {
                unsigned long long *a = reinterpret_cast<unsigned long long *>(
                    reinterpret_cast<char *>(x.arrive) + x.delta[i]);
                asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(a) : "memory");
            }
        }
    }
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Called by every thread of the CTA; thread 0 polls.  false (and *status set) when the
// peers' rows did not arrive within kXWaitNs or another wait already failed.
__device__ __forceinline__ bool xwait(const XWait &w, int *status) {
    __shared__ int s_xok;
    if (!w.arrive) return true;
    if (threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0) {
        const unsigned long long need =
            (unsigned long long)__ldcg(reinterpret_cast<const unsigned int *>(w.epoch)) * w.ranks;
        int ok = 1;
        if (ld_acquire_sys_u64(w.arrive) < need) {
            const unsigned long long t0 = global_timer_ns();
            for (unsigned int it = 1;; ++it) {
                if (ld_acquire_sys_u64(w.arrive) >= need) break;
                if ((it & 63u) == 0u &&
                    (global_timer_ns() - t0 > kXWaitNs || it > (1u << 30) ||
                     (status && *(volatile int *)status != 0))) {
                    ok = 0;
                    break;
                }
                __nanosleep(100);
            }
        }
        if (!ok && status) atomicCAS(status, 0, kDevTimeoutPeer);
        s_xok = ok;
    }
    __syncthreads();
    return s_xok != 0;
}
#endif

// ------------------------------------------------------------------ i4
// One matrix of a fused i4 matvec launch.  All jobs share x, in_dim and group.
struct I4Job {
    const uint8_t *w;     // interleaved i4 rows
    float *y;             // [rows]
    const float *bias;    // optional [rows], added after the dot (fp32)
    const float *resid;   // optional [rows]: y = resid + dot (residual fused into the store)
    int rows;
};

// Where the kernel's activation vector comes from.
enum XMode : int {
    X_PLAIN = 0,    // x = src
    X_RMSNORM = 1,  // x = rmsnorm(src) * norm_w      (rmsnorm_ref semantics)
    X_SWIGLU = 2,   // x = src / (1 + expf(-src)) * up (swiglu_ref semantics)
};

struct XSource {
    int mode = X_PLAIN;
    const float *src = nullptr;
    const float *norm_w = nullptr;
    float eps = 0.0f;
    const float *up = nullptr;
};

// Greedy-token epilogue: argmax over all rows of job 0 (first index of the max).
struct ArgmaxOut {
    float *part_v = nullptr;        // [>= grid] per-CTA partials
    int *part_i = nullptr;
    unsigned int *ticket = nullptr; // zero-initialised; reset by the last CTA
    int *token = nullptr;           // result index (row + row_offset)
    float *value = nullptr;         // optional: the maximum itself
    int row_offset = 0;             // global index of row 0 (vocabulary shard)
};

struct I4LaunchOpts {
    XSource x;
    ArgmaxOut argmax;
    bool pdl = false;               // launch with programmatic stream serialisation
    bool pair_swiglu = false;       // jobs (gate, up): y_gate = silu(gate x) * (up x)
    int *status = nullptr;          // device error word (bounded-wait timeouts)
    // MoE experts chosen on the device: every job's rows are nslots blocks of erows
    // rows; block b reads expert eidx[b] (device int) at job.w + eidx[b] * estride.
    const int *eidx = nullptr;
    long long estride = 0;
    int erows = 0, nslots = 0, n_experts = 0;
    // per-block activations (one plain job): block b uses x.src + b * in_dim
    bool xslots = false;
    Stamp stamp;                    // in-graph timeline (TMA kernel only)
    // tensor parallelism over peer memory (TMA kernel only; DEVICE descriptors, so the
    // single-GPU kernel instance carries neither their parameters nor their code): wait
    // for x's exchange before reading it; store the written rows (and the argmax pair)
    // into every peer
    const XWait *xwait = nullptr;
    const XPut *put = nullptr;
};

// y_j = W_j x (+bias_j / +resid_j) for up to 3 jobs in one launch (q/k/v, gate/up, ...).
int launch_i4_matvec(const I4Job *jobs, int n_jobs, const float *x, int in_dim, int group_size,
                     cudaStream_t stream);
int launch_i4_matvec_ex(const I4Job *jobs, int n_jobs, int in_dim, int group_size,
                        const I4LaunchOpts &opts, cudaStream_t stream);
int i4_argmax_slots(int rows, int in_dim, int group_size);  // partial slots the epilogue needs
// Symmetric W4A8 ("sdot5") semantics.
int launch_i4_matvec_sym(const uint8_t *w, const float *x, float *y, int rows, int in_dim,
                         int group_size, cudaStream_t stream);
// Bit-exact dequant of `rows` rows to fp32.
int launch_i4_dequant(const uint8_t *w, int rows, int dim, int group_size, float *out,
                      cudaStream_t stream);

// ------------------------------------------------------------------ i4 matmul (tensor cores)
// One weight matrix of a (grouped) tcgen05 matmul: Y[:, n] = W X[:, n] for N columns.
// The weights come either through a tensor map over the interleaved rows themselves
// (tmap set: the decode copy, read in place) or from a tile-contiguous repacked copy (w).
struct MmJob {
    const uint8_t *w;     // tile-contiguous weights (launch_mm_repack_w); unused with tmap
    float *y;             // column n at y + n * ldy
    int M, N, ldy;
    int tile_begin;       // first CTA of this job (jobs in CTA order)
    long long b_off;      // offset (bf16 elements) of this job's X planes
    const float *resid = nullptr;  // optional: y = resid + W x (same layout as y)
    const float *bias = nullptr;   // optional: y = W x + bias[row]
    const void *tmap = nullptr;    // optional: CUtensorMap in device memory (mm_encode_weight_map)
    int tz = 0;                    // the map's matrix index (expert e of a layer: e)
};
constexpr int kMmTileRows = 256;  // weight rows per matmul CTA
constexpr int kMmGroupsPerBlock = 4;  // quantisation groups per staged weight block
// Tensor map (a 128-byte CUtensorMap written to map128) over E matrices of M interleaved
// i4 rows of K columns, matrix x at w + x * stride, for the matmul's weight blocks (256
// rows x kMmGroupsPerBlock groups).  False (nothing written) when the layout cannot be
// mapped: K / G not a multiple of kMmGroupsPerBlock (a row's byte length is then not a
// multiple of 16), w or stride not 16-byte aligned, or the driver refuses the map; the
// caller then repacks.
bool mm_encode_weight_map(const uint8_t *w, int M, int K, int G, int E, size_t stride,
                          void *map128);
// One source of a grouped X pack: column n of the job is x + (cols ? cols[n] : n) * ldx.
struct MmPackJob {
    const float *x;
    const float *u;       // optional: pack SwiGLU(x, u) (u in x's layout) instead of x
    const int *cols;
    int ldx, N;
    long long b_off;      // bf16 elements into the planes
    int col0;             // mapped launch: first padded column of this job among all jobs
};
bool mm_group_supported(int G);  // the tensor-core path covers G = 32, 64, 128
// bytes of the two bf16 X planes (hi, lo) for K x N at group size G
size_t mm_x_planes_bytes(int K, int N, int G);
// interleaved i4 rows -> the GEMM's tile-contiguous weight blocks (same bytes, permuted)
size_t mm_repacked_bytes(int M, int K, int G);
int launch_mm_repack_w(const uint8_t *w, int M, int K, int G, uint8_t *out, cudaStream_t st);
size_t mm_scratch_bytes(int M, int K, int N, int G);  // launch_matmul_i4's scratch
int mm_tile_width(int M, int N);
// X [K x N] (column n at x + (cols ? cols[n] : n) * ldx) -> the bf16 hi/lo planes
int launch_mm_pack_x(const float *x, const int *cols, int ldx, int K, int N, int G,
                     uint16_t *bhi, uint16_t *blo, cudaStream_t st, const float *u = nullptr);
// map128: optional tensor map (host copy) of a single job's weights, passed in the
// kernel's parameters (the job's tmap is then ignored)
int launch_matmul_i4_grouped(const MmJob *host_jobs, const MmJob *dev_jobs, int n_jobs, int K,
                             int G, int nt, const uint16_t *bhi, const uint16_t *blo,
                             int total_tiles, int *status, cudaStream_t st,
                             const void *map128 = nullptr);
// Device-planned launch: the job of tile i is dev_tile_job[i]; tiles at or beyond
// *dev_n_tiles (written on the device, <= max_tiles) return at once.
int launch_matmul_i4_planned(const MmJob *dev_jobs, const int *dev_tile_job, const int *dev_n_tiles,
                             int max_tiles, int K, int G, int nt, const uint16_t *bhi,
                             const uint16_t *blo, int *status, cudaStream_t st);
// ---- prefill (prompt) pieces
// Causal GQA attention of n new tokens at positions p0 .. p0+n-1 whose keys and values
// are already in the cache: out[t] = softmax(q[t] K[0..p0+t]^T * scale) V[0..p0+t].
struct AttnPrefillArgs {
    const float *q;        // [n][n_heads * head_dim] (QK-normed, rotated)
    const void *k, *v;     // [n_kv_heads][max_seq][head_dim] fp32 or fp16
    int kv_fp16;
    int p0, n, max_seq;
    int n_heads, n_kv_heads, head_dim;
    float scale;
    float *out;            // [n][n_heads * head_dim]
};
int launch_attn_prefill(const AttnPrefillArgs &a, cudaStream_t st);
bool attn_prefill_supported(int n_heads, int n_kv_heads, int head_dim);

// MoE layer plan (one CTA on the device): bucket the n*k (token, choice) assignments by
// expert and write the grouped GEMM jobs, pack jobs and tile maps of gate/up and down.
constexpr int kMoePlanMaxExperts = 1024;
struct MoePlanArgs {
    const int *idx;        // [n*k] chosen experts
    int n, k, E;
    int G, H, mi, nt;      // group size, hidden, expert intermediate, tile width
    const uint8_t *wg, *wu, *wd;  // tile-contiguous expert weights, expert e at e * stride
    long long wgu_stride, wd_stride;
    // or tensor maps over the experts' interleaved rows (expert e: coordinate z = e), which
    // take precedence when set
    const void *tmg = nullptr, *tmu = nullptr, *tmd = nullptr;
    const float *xn;       // [n][H] normalised hidden rows (gate/up input)
    float *hbuf, *ubuf;    // [n*k][mi] gate / up outputs in bucket order (down's input is
                           // SwiGLU(h, u), formed by its X pack)
    float *obuf;           // [n*k][H] down outputs in bucket order
    int *rows, *slot;      // [n*k] token of bucket row; bucket row of assignment
    MmJob *jobs_gu, *jobs_dn;     // [2E], [E]
    int *tile_gu, *tile_dn;       // tile -> job maps (moe_plan_max_tiles entries)
    int *ntiles;                  // [3] tiles in use: gate/up, down; 8-column blocks
    MmPackJob *pack_gu, *pack_dn; // [E] each
    int *pack_map;                // 8-column block -> expert (moe_plan_max_cols / 8 entries)
    int *status;
    // expert parallelism: only experts [e0, e0 + e_local) get matmul jobs, their weights at
    // (e - e0) * stride (e_local = 0: every expert); the bucket layout stays that of all E
    // experts, so obuf rows line up across the ranks
    int e0 = 0, e_local = 0;
};
int launch_moe_plan(const MoePlanArgs &a, cudaStream_t st);
// upper bounds for the buffers of a plan: tiles of one job kind of M rows at width nt,
// and X-plane elements (one plane) for K
int moe_plan_max_tiles(int n, int k, int E, int M, int nt);
int moe_plan_max_cols(int n, int k, int E);  // padded columns over all experts
// dynamic shared memory of the plan kernel (at most kMoePlanMaxSmem)
size_t moe_plan_smem_bytes(int n, int k, int E);
constexpr size_t kMoePlanMaxSmem = 160 * 1024;
long long moe_plan_plane_elems(int n, int k, int E, int K, int G);

// X planes of several jobs in one launch: 8-column block b (< *dev_count <= max_blocks)
// belongs to job dev_map[b]; all on the device
int launch_mm_pack_x_mapped(const MmPackJob *dev_jobs, const int *dev_map, const int *dev_count,
                            int max_blocks, int K, int G, uint16_t *bhi, uint16_t *blo, cudaStream_t st);
// tiles of one job of M rows and N columns at tile width nt
int mm_job_tiles(int M, int N, int nt);
// bf16 elements of one plane for N columns (the b_off step between jobs)
long long mm_plane_elems(int K, int N, int G);
// Y = W X (matmul_i4_ref semantics); scratch holds mm_scratch_bytes(M, K, N, G) bytes
int launch_matmul_i4(const uint8_t *w, const float *x, float *y, int M, int K, int N, int G,
                     void *scratch, int *status, cudaStream_t st);

// ------------------------------------------------------------------ VQ2 + BiIP
// One VQ2 matrix of a launch; each job has its own codebook and BiIP rotation.
struct VqJob {
    const uint8_t *w = nullptr;   // [codebook 256x4 f16][rows x K/4 indices]
    float *y = nullptr;
    const float *resid = nullptr; // optional: y = resid + dot
    int rows = 0;
    const float *rot_sign = nullptr, *rot_scale = nullptr;  // BiIP of x (sign null: none)
    int rot_bs = 0;               // 0: the reference's block size for the input width
};
struct VqLaunch {
    VqJob job[3];
    int n_jobs = 1;
    bool pair_swiglu = false;     // jobs (gate, up), equal rows: y_gate = silu(gate) * up
    int K = 0;
    XSource x;
    bool pdl = false;
    int *status = nullptr;        // device error word (bounded-wait timeouts)
    Stamp stamp;                  // in-graph timeline
};
int launch_vq2_matvec(const VqLaunch &a, cudaStream_t st);
int launch_biip(const float *x, float *y, int dim, const float *scale, const float *sign, int bs,
                cudaStream_t st);

// ------------------------------------------------------------------ decode ops
int launch_rmsnorm(const float *x, const float *w, float *y, int rows, int n, float eps,
                   cudaStream_t st);
// Host: the cos/sin row of one position exactly as rope_ref computes it.
void rope_row(float theta, int head_dim, int pos, float *cs, float *sn);
int launch_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim, const float *cs,
                const float *sn, cudaStream_t st);

struct QkRopeKvArgs {
    float *q;                 // [H*hd] in/out
    const float *k, *v;       // [KVH*hd]
    const float *q_norm, *k_norm;  // optional [hd]
    float eps;
    const float *cos_tab, *sin_tab;  // [max_seq][hd/2]
    const int *pos;
    void *kcache, *vcache;    // layer slices [KVH][max_seq][hd]
    int kv_fp16;
    int n_heads, n_kv_heads, head_dim, max_seq;
    int n_tokens = 1;         // consecutive tokens (rows of q/k/v) at *pos, *pos + 1, ...
};
int launch_qk_rope_kv(const QkRopeKvArgs &a, cudaStream_t st);

struct AttnArgs {
    const float *q;           // [H*hd]
    const void *k, *v;        // [KVH][max_seq][hd] fp32 or fp16
    int kv_fp16;
    const int *pos;           // seq = *pos + 1 (nullptr -> seq_len)
    int seq_len, max_seq;
    int n_heads, n_kv_heads, head_dim;
    float scale;
    int nsplit, chunk_max;
    float *partial;           // attn_partial_floats(...)
    unsigned int *tickets;    // [n_kv_heads], zero-initialised
    float *out;               // [H*hd]
    // Engine ("fused") mode, k_new != nullptr: q/k_new/v_new are the step's raw
    // projections; QK-norm (optional), RoPE from the [max_seq][hd/2] tables and
    // the KV append at position seq-1 happen inside the attention launch (one
    // kernel where the shape has a TMA instantiation, else qk_rope_kv first).
    const float *k_new = nullptr, *v_new = nullptr;
    const float *q_norm = nullptr, *k_norm = nullptr;
    float eps = 0.0f;
    const float *cos_tab = nullptr, *sin_tab = nullptr;
    bool pdl = false;         // programmatic dependent launch (TMA kernel only)
    int *status = nullptr;    // device error word (bounded waits, bad position)
    Stamp stamp;              // in-graph timeline (TMA kernel only)
    const XPut *put = nullptr;  // tensor parallelism (device descriptor): out rows also go
                                // to every peer (TMA kernel only)
};
int attn_plan(int n_kv_heads, int max_seq, int *nsplit, int *chunk_max);
size_t attn_partial_floats(int n_heads, int head_dim, int nsplit);
int launch_attention(const AttnArgs &a, cudaStream_t st);
// The TMA-staged, cluster-merged kernel alone (no scratch: partial/tickets unused);
// TQB200_ERR_UNSUPPORTED, with nothing launched, for shapes it does not cover.
int launch_attention_tma(const AttnArgs &a, cudaStream_t st);
// The split kernel alone (plain mode), with AttnArgs' partial/tickets scratch.
int launch_attention_split(const AttnArgs &a, cudaStream_t st);

int launch_swiglu(float *g, const float *u, int n, cudaStream_t st);
int launch_swiglu_out(const float *g, const float *u, float *out, int n, cudaStream_t st);
// (value, index) of every rank's vocabulary shard -> the global first maximum
struct ArgPair {
    float v;
    int i;
};
int launch_argmax_pairs(const ArgPair *pairs, int n, int *out, cudaStream_t st,
                        const XWait &xw = XWait(), int *status = nullptr);
int argmax_blocks(int n);
int launch_argmax(const float *l, int n, float *pv, int *pi, unsigned int *ticket, int *out,
                  cudaStream_t st);
int launch_topk_softmax(const float *logits, int n, int k, int *idx, float *w, cudaStream_t st);
// MoE decode: f32 router over rmsnorm(h) * norm_w, then top-k softmax (ticket: zeroed
// device word, reset by the kernel); and h += sum_t wts[t] * o[t] in router order.
int launch_moe_router(const float *h, const float *norm_w, float eps, int H, const float *W, int E,
                      int k, float *logits, int *idx, float *wts, unsigned int *ticket, bool pdl,
                      cudaStream_t st, const Stamp &stamp = Stamp(), const XWait &xw = XWait(),
                      int *status = nullptr);
int launch_moe_combine(float *h, const float *o, const float *wts, int k, int H, bool pdl,
                       cudaStream_t st, const Stamp &stamp = Stamp(), const XWait &xw = XWait(),
                       int *status = nullptr);
// epoch (optional): advanced by one, the decode step count of the peer exchanges
int launch_embed(const void *table, int dtype, const int *token, int dim, int group_size,
                 float *out, cudaStream_t st, int n_tokens = 1, unsigned int *epoch = nullptr);
// Expert parallelism: local[j] = idx[j] - e0 when this rank owns that expert, else -1;
// o[0 .. k*H) = 0 when o is given (the cross-rank sum of the slots then equals each
// owner's output; the peer exchange, where each owner stores its slots, passes none).
int launch_moe_ep_local(const int *idx, int k, int e0, int e_local, int *local, float *o, int H,
                        bool pdl, cudaStream_t st);
// MoE prefill: router logits of n tokens (f32 router, xn normalised rows), top-k softmax
// per token, and h[t] += sum_j wts[t][j] * o[slot[t*k+j]] per token.
int launch_router_rows(const float *xn, int n, int H, const float *W, int E, float *logits,
                       cudaStream_t st);
int launch_topk_rows(const float *logits, int n, int E, int k, int *idx, float *wts, cudaStream_t st);
int launch_moe_combine_rows(float *h, const float *o, const float *wts, const int *slot, int n,
                            int k, int H, cudaStream_t st);

// ------------------------------------------------------------------ GDN ops (gdn_ops.cu)
// l2norm_inplace / rmsnorm_gated over n_vec vectors of n floats; gdn_step over n_heads
// heads (S [n_heads][qk_dim][v_dim], q/k [n_heads][qk_dim], v/o [n_heads][v_dim], decay =
// exp(g) and beta per head, on the device); partial RoPE with host cos/sin rows.
int launch_l2norm(float *x, int n_vec, int n, float eps, cudaStream_t st);
int launch_causal_conv1d(const float *x, float *state, const float *w, float *out, int dim, int ks,
                         cudaStream_t st);
int launch_gdn_step(float *S, const float *q, const float *k, const float *v, const float *decay,
                    const float *beta, float *o, int n_heads, int qk_dim, int v_dim,
                    cudaStream_t st);
int launch_rmsnorm_gated(const float *x, const float *gate, const float *w, float *y, int n_vec,
                         int n, float eps, cudaStream_t st);
int launch_partial_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim,
                        int rotary_dim, const float *cs, const float *sn, cudaStream_t st);

// ------------------------------------------------------------------ GPTQ, dense (gptq_matvec.cu)
size_t gptq_bytes(int out, int in, int G, bool g_idx);
// Y[:, j] = W X[:, j] for n columns (X [in x n], Y [out x n] column-major)
int launch_gptq_matmul(const uint8_t *w, bool g_idx, const float *x, float *y, int out, int in,
                       int n, int G, cudaStream_t st);
int launch_dense_matvec(const void *w, bool f16, const float *x, float *y, int out, int in,
                        cudaStream_t st);

}  // namespace tqb200
