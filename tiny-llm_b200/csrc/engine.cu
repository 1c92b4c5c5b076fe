// engine.cu — GPU-resident batch-1 greedy decode engine (sm_100a).
//
// Replaces the reference's GPU decode registry entry (kernels/dispatch.h:353-378,
// kernels/cuda/gpu_engine.cu) for quantised (i4) Qwen2/Qwen3-family models and
// runs the same step as QwenModel::forward_token (runtime/qwen_forward_token.cpp:83-742):
//
//   embed -> per layer [ rmsnorm -> q/k/v (+bias) -> QK-norm -> RoPE -> KV append
//            -> attention -> o_proj + residual -> rmsnorm -> gate/up -> SwiGLU
//            -> down + residual ] -> final rmsnorm -> lm_head -> argmax
//
// as 2 + 5 * n_layers kernels for a dense model:
//   embed | qkv (RMSNorm prologue, bias epilogue) | attention (QK-norm, RoPE and KV append
//   fused; split-K over the positions, merged in a cluster) | o_proj (residual epilogue)
//   | gate/up (RMSNorm prologue, SwiGLU epilogue) | down (residual epilogue) | ... |
//   lm_head (RMSNorm prologue, argmax epilogue)
// (a MoE layer: qkv | attention | o_proj | router + top-k | expert gate/up | expert down
// | ordered combine), captured once into a CUDA graph whose nodes are linked by
// programmatic dependent launch, so a kernel's CTAs start (and stream their weights)
// on the SMs its predecessor has left.  Per step the host moves 8 bytes in (token, position) and 8 bytes
// out (next token, device status) through pinned memory, like the reference
// engine's 2 x 4 B H2D + 4 B D2H (kernels/cuda/gpu_engine.cu:332-371).
//
// Tensor parallelism (tp_size > 1, one process per GPU): every projection's
// output rows are split evenly (q/k/v by head, o/down by hidden row, gate/up by
// intermediate row, lm_head by vocabulary row); each rank runs the same kernels
// on its rows and the activations are all-gathered after attention, o_proj,
// SwiGLU and down: by the producing kernels themselves over the ranks' mapped
// arenas once the peer exchange is open (tqb200_engine_open_exchange), else in
// place over NCCL inside the CUDA graph.  Every output
// element is computed by exactly the kernel and order the single-GPU engine
// uses, so tokens and logits do not depend on the number of GPUs.  The greedy
// token is the first maximum over the ranks' (max, index) pairs.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#ifdef TQB200_HAVE_NCCL
#include <nccl.h>
#endif

namespace tqb200 {
namespace {

// Projection order of the per-projection BiIP rotations.
enum Proj { P_Q, P_K, P_V, P_O, P_GATE, P_UP, P_DOWN, P_N };

struct DLayer {
    bool vq2 = false;  // projections are VQ2 (else i4)
    const float *input_ln = nullptr, *post_ln = nullptr;
    const uint8_t *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
    const uint8_t *gate = nullptr, *up = nullptr, *down = nullptr;
    const float *q_bias = nullptr, *k_bias = nullptr, *v_bias = nullptr;
    const float *q_norm = nullptr, *k_norm = nullptr;
    const float *rot_sign[P_N] = {}, *rot_scale[P_N] = {};  // VQ2 BiIP (sign null: none)
    int rot_bs[P_N] = {};
    // MoE FFN: router (f32 or i4) and every expert's matrices back to back
    bool moe = false;
    const float *router_f32 = nullptr;
    const uint8_t *router_i4 = nullptr;
    const uint8_t *ex_gate = nullptr, *ex_up = nullptr, *ex_down = nullptr;
    size_t ex_gu_stride = 0, ex_down_stride = 0;  // bytes between experts
};

// A weight operand of the prefill's tensor-core matmul: a tensor map (device copy)
// over the decode matrix itself, read in place, or, for a matrix no map can cover (K / G
// not a multiple of 4), a tile-contiguous repacked copy (launch_mm_repack_w).
struct PW {
    const uint8_t *w = nullptr;  // repacked copy (null with a map)
    const void *tm = nullptr;    // CUtensorMap in device memory
    explicit operator bool() const { return w || tm; }
};

// A layer's prefill weight operands; experts of a kind under one map (expert x at z = x)
// or repacked back to back, expert x at x * stride.
struct PLayer {
    PW q, k, v, o, gate, up, down, router;
    PW ex_gate, ex_up, ex_down;
    size_t ex_gu_stride = 0, ex_down_stride = 0;
};

// Batched prompt state (allocated by the first prefill): activations of up to `cap`
// tokens, row t of token t, and the X planes of the tensor-core matmul.
struct Prefill {
    bool ready = false;
    int cap = 0;
    std::vector<PLayer> layers;
    float *hidden = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr,
          *attn = nullptr, *gate = nullptr, *up = nullptr;
    int *io = nullptr;  // device [p0, tokens...]
    uint16_t *bhi = nullptr, *blo = nullptr;
    // host-planned jobs of the current chunk size (7 per layer), on the device
    std::vector<MmJob> hjobs;
    MmJob *jobs = nullptr;
    int jobs_n = -1;
    std::vector<int> nt, tiles;  // per job launch: tile width and CTAs (4 launches per layer)
    // MoE
    float *logits = nullptr, *wts = nullptr, *mh = nullptr, *mu = nullptr, *mo = nullptr;
    int *idx = nullptr, *rows = nullptr, *slot = nullptr, *ntiles = nullptr;
    int *tile_gu = nullptr, *tile_dn = nullptr, *pack_map = nullptr;
    MmJob *jobs_gu = nullptr, *jobs_dn = nullptr;
    MmPackJob *pack_gu = nullptr, *pack_dn = nullptr;
    int max_tiles_gu = 0, max_tiles_dn = 0, moe_nt = 64;
    // tensor maps of every layer's matrices (device; 128 bytes each) and the bytes of the
    // repacked copies made for matrices without one
    uint8_t *maps = nullptr;
    size_t n_maps = 0, cap_maps = 0;
    std::vector<uint8_t> hmaps;
    size_t copy_bytes = 0;
};

}  // namespace
}  // namespace tqb200

struct tqb200_engine {
    tqb200_model_desc d{};
    tqb200_engine_opts o{};
    int device = 0;
    cudaStream_t stream = nullptr;
    std::vector<void *> allocs;
    std::vector<tqb200::DLayer> layers;
    const void *embed = nullptr;
    int embed_dtype = 0;
    const uint8_t *lm_head = nullptr;
    const float *final_norm = nullptr;
    float *hidden = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr;
    float *gate = nullptr, *up = nullptr, *logits = nullptr;
    void *kv = nullptr;  // [K|V][L][KVH][max_seq][hd]
    size_t layer_stride = 0;
    float *cos_tab = nullptr, *sin_tab = nullptr;
    int *io_in = nullptr;   // device [token, pos]
    int *io_out = nullptr;  // device [next, status]
    int *h_io = nullptr;    // pinned host [token, pos, next, status]
    float *attn_part = nullptr;
    unsigned int *attn_tickets = nullptr;
    int attn_nsplit = 0, attn_chunk = 0;
    float *am_v = nullptr;
    int *am_i = nullptr;
    unsigned int *am_ticket = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;       // one step, host-fed token/position
    cudaGraph_t loop_graph = nullptr;
    cudaGraphExec_t loop_exec = nullptr;  // one step + device-side feed of the next token
    int *gen_tokens = nullptr;            // device [max_seq] tokens of generate()
    int *gen_count = nullptr;             // device step counter of generate()
    cudaEvent_t ev[2] = {nullptr, nullptr};
    // profiling: events after every launch, tagged with a kernel kind
    bool prof = false;
    bool debug_sync = false;  // TQB200_DEBUG_SYNC=1: no graph, check every kernel
    int cur_layer = -1;
    std::vector<cudaEvent_t> prof_ev;
    std::vector<int> prof_kind;
    int pos = 0;
    size_t weight_bytes = 0;
    // tensor parallelism
    int tp = 1, rank = 0;
    // attention shards: tp for dense models; 1 for MoE models, whose attention runs whole
    // on every rank (expert parallelism shards only the experts), and rank ra in them
    int ga = 1, ra = 0;
    bool xoff = false;  // the batched prefill's exchanges go over NCCL even with p2p open
    float *act = nullptr;              // [inter] SwiGLU output, all-gathered (tp > 1)
    tqb200::ArgPair *pairs = nullptr;  // [tp] per-rank (max, index)
    // MoE decode state: router logits, chosen experts and weights, expert activations
    float *moe_logits = nullptr, *moe_w = nullptr, *moe_h = nullptr, *moe_u = nullptr,
          *moe_o = nullptr;
    int *moe_idx = nullptr;
    int *moe_local = nullptr;  // expert parallelism: chosen experts as local indices (-1: remote)
    unsigned int *moe_ticket = nullptr;
    tqb200::Prefill pf;
    // in-graph timeline of generate() (tqb200_engine_set_timeline): three global-timer
    // words per stamped launch and step, the launches' kinds in step order
    unsigned long long *tl = nullptr;
    int tl_cap = 0, tl_stride = 0, tl_steps = 0;
    bool tl_capture = false;  // true while the stamped generate graph is being captured
    std::vector<int> tl_kind;
#ifdef TQB200_HAVE_NCCL
    ncclComm_t comm = nullptr;
#endif
    // peer exchange (tqb200_engine_open_exchange): the all-gathers fused into the
    // producing kernels over the ranks' mapped arenas instead of NCCL
    void *xarena = nullptr;              // activations, then counters, tickets and epoch
    bool p2p = false;
    int n_peers = 0;
    long long xdelta[tqb200::kMaxPeers] = {};
    std::vector<void *> peer_maps;       // the other ranks' arenas, mapped here
    unsigned long long *xcnt = nullptr;  // [n_xslots] arrival counters
    unsigned int *xticket = nullptr;     // [n_xslots] CTA tickets
    unsigned int *epoch = nullptr;       // decode steps since the exchange opened
    // per exchange slot: the consumer and producer descriptors, on the host (kernels that
    // take them by value) and on the device (the matvec and attention kernels' exchange
    // instances read them from there)
    std::vector<tqb200::XWait> xw_host;
    std::vector<tqb200::XPut> xp_host;
    tqb200::XWait *xw_dev = nullptr;
    tqb200::XPut *xp_dev = nullptr;
};

namespace tqb200 {
namespace {

int dev_alloc(tqb200_engine *e, size_t bytes, void **out) {
    void *p = nullptr;
    TQ_CUDA_TRY(cudaMalloc(&p, bytes + 256));  // +256: bulk copies may round up to 16 B
    e->allocs.push_back(p);
    *out = p;
    return TQB200_OK;
}

int upload_bytes(tqb200_engine *e, const void *host, size_t bytes, const void **out) {
    void *p;
    int st = dev_alloc(e, bytes, &p);
    if (st) return st;
    TQ_CUDA_TRY(cudaMemcpy(p, host, bytes, cudaMemcpyHostToDevice));
    e->weight_bytes += bytes;
    *out = p;
    return TQB200_OK;
}

size_t mat_bytes(const tqb200_matrix &m, int group) {
    switch (m.dtype) {
        case TQB200_DT_I4: return (size_t)m.rows * tqb200_i4_row_bytes(m.cols, group);
        case TQB200_DT_VQ2: return tqb200_vq2_bytes(m.rows, m.cols);
        case TQB200_DT_F16: return (size_t)m.rows * m.cols * 2;
        default: return (size_t)m.rows * m.cols * 4;
    }
}

#define TQ_TRY(expr)         \
    do {                     \
        int s_ = (expr);     \
        if (s_) return s_;   \
    } while (0)

int need_mat(const tqb200_matrix &m, int rows, int cols, int dtype, const char *what, int layer) {
    if (!m.data) return set_error(TQB200_ERR_INVALID_ARG, "layer %d: %s missing", layer, what);
    if (m.dtype != dtype)
        return set_error(TQB200_ERR_UNSUPPORTED,
                         "layer %d: %s dtype %d (the engine needs every projection i4 (3) or "
                         "every projection VQ2 (4); layer 0 has %d)",
                         layer, what, m.dtype, dtype);
    if (m.rows != rows || m.cols != cols)
        return set_error(TQB200_ERR_INVALID_ARG, "layer %d: %s shape %dx%d, expected %dx%d",
                         layer, what, m.rows, m.cols, rows, cols);
    return TQB200_OK;
}

// Rows [r0, r0 + n) of an i4 matrix (a contiguous byte range of the interleaved layout).
int up_i4_rows(tqb200_engine *e, const tqb200_matrix &m, int r0, int n, const uint8_t **out) {
    const size_t rb = tqb200_i4_row_bytes(m.cols, e->d.group_size);
    const void *p;
    TQ_TRY(upload_bytes(e, (const uint8_t *)m.data + (size_t)r0 * rb, (size_t)n * rb, &p));
    *out = (const uint8_t *)p;
    return TQB200_OK;
}

// Rows [r0, r0 + n) of a VQ2 matrix: its codebook followed by those rows' indices.
int up_vq2_rows(tqb200_engine *e, const tqb200_matrix &m, int r0, int n, const uint8_t **out) {
    const size_t rb = (size_t)m.cols / 4, cb = 2048;
    void *p;
    TQ_TRY(dev_alloc(e, cb + (size_t)n * rb, &p));
    TQ_CUDA_TRY(cudaMemcpy(p, m.data, cb, cudaMemcpyHostToDevice));
    TQ_CUDA_TRY(cudaMemcpy((uint8_t *)p + cb, (const uint8_t *)m.data + cb + (size_t)r0 * rb,
                           (size_t)n * rb, cudaMemcpyHostToDevice));
    e->weight_bytes += cb + (size_t)n * rb;
    *out = (const uint8_t *)p;
    return TQB200_OK;
}

int up_vec(tqb200_engine *e, const float *h, int n, const float **out) {
    if (!h) {
        *out = nullptr;
        return TQB200_OK;
    }
    const void *p;
    TQ_TRY(upload_bytes(e, h, (size_t)n * 4, &p));
    *out = (const float *)p;
    return TQB200_OK;
}

// Every expert's gate, up and down matrices into one device buffer per kind, expert x at
// x * stride (stride = the matrix bytes rounded up to 16), and the router.
int up_experts(tqb200_engine *e, const tqb200_layer &s, const tqb200_model_desc &d, DLayer &w) {
    const int E = d.n_experts / e->tp, x0 = e->rank * E;  // this rank's experts (all if tp == 1)
    const size_t gu = (mat_bytes(s.expert_gate[0], d.group_size) + 15) & ~(size_t)15;
    const size_t dn = (mat_bytes(s.expert_down[0], d.group_size) + 15) & ~(size_t)15;
    void *pg, *pu, *pd;
    TQ_TRY(dev_alloc(e, gu * E, &pg));
    TQ_TRY(dev_alloc(e, gu * E, &pu));
    TQ_TRY(dev_alloc(e, dn * E, &pd));
    for (int x = 0; x < E; ++x) {
        const size_t b = mat_bytes(s.expert_gate[x0 + x], d.group_size);
        const size_t bd = mat_bytes(s.expert_down[x0 + x], d.group_size);
        TQ_CUDA_TRY(cudaMemcpy((uint8_t *)pg + x * gu, s.expert_gate[x0 + x].data, b, cudaMemcpyHostToDevice));
        TQ_CUDA_TRY(cudaMemcpy((uint8_t *)pu + x * gu, s.expert_up[x0 + x].data, b, cudaMemcpyHostToDevice));
        TQ_CUDA_TRY(cudaMemcpy((uint8_t *)pd + x * dn, s.expert_down[x0 + x].data, bd, cudaMemcpyHostToDevice));
        e->weight_bytes += 2 * b + bd;
    }
    w.ex_gate = (const uint8_t *)pg;
    w.ex_up = (const uint8_t *)pu;
    w.ex_down = (const uint8_t *)pd;
    w.ex_gu_stride = gu;
    w.ex_down_stride = dn;
    const void *pr;
    TQ_TRY(upload_bytes(e, s.router.data, mat_bytes(s.router, d.group_size), &pr));
    if (s.router.dtype == TQB200_DT_F32) w.router_f32 = (const float *)pr;
    else w.router_i4 = (const uint8_t *)pr;
    return TQB200_OK;
}

int validate(const tqb200_model_desc &d, const tqb200_engine_opts &o) {
    const bool moe = d.model_type == TQB200_MODEL_QWEN3_MOE;
    TQ_CHECK_ARG(d.model_type == TQB200_MODEL_QWEN2 || moe,
                 "engine supports model_type Qwen2/Qwen3 dense (0) and Qwen3-MoE (3), got %d",
                 d.model_type);
    TQ_CHECK_ARG(d.n_layers > 0 && d.hidden > 0 && (moe || d.inter > 0) && d.n_heads > 0 &&
                     d.n_kv_heads > 0 && d.head_dim > 0 && d.vocab > 0 && d.layers,
                 "model description has zero fields");
    if (moe) {
        TQ_CHECK_ARG(d.n_experts > 0 && d.n_experts <= 1024 && d.experts_per_tok > 0 &&
                         d.experts_per_tok <= 64 && d.experts_per_tok <= d.n_experts &&
                         d.moe_inter > 0 && d.moe_inter % 32 == 0,
                     "MoE: n_experts %d, experts_per_tok %d, moe_inter %d", d.n_experts,
                     d.experts_per_tok, d.moe_inter);
        TQ_CHECK_ARG(o.tp_size <= 1 || d.n_experts % o.tp_size == 0,
                     "expert parallelism: tp_size %d must divide n_experts %d", o.tp_size,
                     d.n_experts);
    }
    TQ_CHECK_ARG(d.n_heads % d.n_kv_heads == 0, "n_heads %% n_kv_heads != 0");
    TQ_CHECK_ARG(d.group_size > 0 && d.group_size % 32 == 0,
                 "engine needs group_size %% 32 == 0 (got %d)", d.group_size);
    TQ_CHECK_ARG(d.hidden % 32 == 0 && d.inter % 32 == 0 && (d.n_heads * d.head_dim) % 32 == 0,
                 "engine needs hidden/inter/q_dim multiples of 32");
    TQ_CHECK_ARG(o.max_seq_len > 0 && (d.max_seq_len <= 0 || o.max_seq_len <= d.max_seq_len),
                 "max_seq_len %d exceeds model max %d", o.max_seq_len, d.max_seq_len);
    TQ_CHECK_ARG(d.head_dim % 2 == 0 && d.head_dim <= 512, "head_dim %d", d.head_dim);
    TQ_CHECK_ARG(d.lm_head.data && d.lm_head.dtype == TQB200_DT_I4 && d.lm_head.rows == d.vocab &&
                     d.lm_head.cols == d.hidden,
                 "engine needs an i4 lm_head [vocab x hidden]");
    TQ_CHECK_ARG(d.embed.data && d.embed.rows == d.vocab && d.embed.cols == d.hidden &&
                     (d.embed.dtype == TQB200_DT_F32 || d.embed.dtype == TQB200_DT_F16 ||
                      d.embed.dtype == TQB200_DT_I4),
                 "embed must be f32/f16/i4 [vocab x hidden]");
    TQ_CHECK_ARG(d.final_norm, "final_norm missing");
    return TQB200_OK;
}

// RoPE tables with the reference's exact float operations (kernels/rope/rope_ref.cpp:74-85):
// inv_freq = powf(theta, -(float)(2i)/(float)hd), angle = (float)pos * inv_freq.
int build_rope_tables(tqb200_engine *e) {
    const int half = e->d.head_dim / 2, S = e->o.max_seq_len;
    std::vector<float> cs((size_t)S * half), sn((size_t)S * half);
    for (int p = 0; p < S; ++p)
        rope_row(e->d.rope_theta, e->d.head_dim, p, cs.data() + (size_t)p * half,
                 sn.data() + (size_t)p * half);
    const void *dc, *ds;
    TQ_TRY(upload_bytes(e, cs.data(), cs.size() * 4, &dc));
    TQ_TRY(upload_bytes(e, sn.data(), sn.size() * 4, &ds));
    e->weight_bytes -= (cs.size() + sn.size()) * 4;
    e->cos_tab = (float *)dc;
    e->sin_tab = (float *)ds;
    return TQB200_OK;
}

enum Kind {
    K_EMBED, K_QKV, K_ROPE_KV, K_ATTN, K_OPROJ, K_GATEUP, K_DOWN, K_LMHEAD, K_ROUTER, K_COMBINE,
    K_NORM, K_PACK, K_PLAN, K_SWIGLU, K_NKINDS
};

const char *kind_name(int k) {
    static const char *n[] = {"embed", "qkv", "qk_rope_kv", "attention", "o_proj",
                              "gate_up", "down", "lm_head", "router", "moe_combine",
                              "rmsnorm", "x_pack", "moe_plan", "swiglu"};
    return (k >= 0 && k < K_NKINDS) ? n[k] : "start";
}

int mark(tqb200_engine *e, int kind) {
    if (e->debug_sync) {
        // diagnostic mode (TQB200_DEBUG_SYNC=1): finish every kernel and check it
        const cudaError_t ce = cudaStreamSynchronize(e->stream);
        if (ce != cudaSuccess)
            return set_error(TQB200_ERR_CUDA, "after %s (layer %d, position %d): %s",
                             kind_name(kind), e->cur_layer, e->pos, cudaGetErrorString(ce));
        int stv = 0;
        TQ_CUDA_TRY(cudaMemcpy(&stv, e->io_out + 1, 4, cudaMemcpyDeviceToHost));
        if (stv)
            return set_error(TQB200_ERR_TIMEOUT, "device status %d after %s (layer %d)", stv,
                             kind_name(kind), e->cur_layer);
    }
    if (!e->prof) return TQB200_OK;
    cudaEvent_t ev;
    TQ_CUDA_TRY(cudaEventCreate(&ev));
    TQ_CUDA_TRY(cudaEventRecord(ev, e->stream));
    e->prof_ev.push_back(ev);
    e->prof_kind.push_back(kind);
    return TQB200_OK;
}

// The timeline words of the next stamped launch of kind `kind` (off outside the capture
// of a stamped generate graph).
Stamp tl_next(tqb200_engine *e, int kind) {
    Stamp s;
    if (!e->tl_capture || !e->tl) return s;
    const int i = (int)e->tl_kind.size();
    const int words = 3 * kStampCtas;  // per launch and step
    if (words * (i + 1) > e->tl_stride) return s;
    e->tl_kind.push_back(kind);
    s.base = e->tl + (size_t)words * i;
    s.step = e->gen_count;
    s.stride = e->tl_stride;
    s.cap = e->tl_cap;
    return s;
}

// Device-side token feed for generate(): records the produced token and makes it
// (and position + 1) the input of the next step.
__global__ void feed_next_kernel(int *io_in, const int *io_out, int *tokens, int *count) {
    const int c = *count;
    tokens[c] = io_out[0];
    io_in[0] = io_out[0];
    io_in[1] += 1;
    *count = c + 1;
}

// Peer-exchange slots: four per layer (a MoE layer uses three: its FFN slot carries the
// experts' output slots and the combine runs whole on every rank), then lm_head's.
enum XSlot { XS_ATTN, XS_HID_O, XS_FFN, XS_HID_D, XS_PER_LAYER };
int n_xslots(const tqb200_model_desc &d) { return d.n_layers * XS_PER_LAYER + 1; }
int xslot_lm(const tqb200_model_desc &d) { return d.n_layers * XS_PER_LAYER; }

// The producer and consumer descriptors of exchange `slot` (device copies for the matvec
// and attention kernels, values for the others; none without an open exchange).
bool p2p_on(const tqb200_engine *e) { return e->p2p && !e->xoff; }
const XPut *xput(const tqb200_engine *e, int slot) { return p2p_on(e) ? e->xp_dev + slot : nullptr; }
const XWait *xwait_of(const tqb200_engine *e, int slot) {
    return p2p_on(e) ? e->xw_dev + slot : nullptr;
}
XWait xwait_val(const tqb200_engine *e, int slot) { return p2p_on(e) ? e->xw_host[slot] : XWait(); }

// In-place all-gather of `count` floats per rank (rank r's slice at buf + r * count).
// With the peer exchange open the producing kernel has already stored the rows.
int allgather(tqb200_engine *e, float *buf, size_t count) {
    if (e->tp == 1 || p2p_on(e)) return TQB200_OK;
#ifdef TQB200_HAVE_NCCL
    const ncclResult_t nr =
        ncclAllGather(buf + (size_t)e->rank * count, buf, count, ncclFloat, e->comm, e->stream);
    if (nr != ncclSuccess)
        return set_error(TQB200_ERR_CUDA, "ncclAllGather: %s", ncclGetErrorString(nr));
    return TQB200_OK;
#else
    (void)buf;
    (void)count;
    return set_error(TQB200_ERR_UNSUPPORTED, "built without NCCL");
#endif
}

// In-place sum over the ranks of `count` floats (with the peer exchange open every
// owner has stored its slots in every rank's buffer instead).
int allreduce_sum(tqb200_engine *e, float *buf, size_t count) {
    if (e->tp == 1 || p2p_on(e)) return TQB200_OK;
#ifdef TQB200_HAVE_NCCL
    const ncclResult_t nr = ncclAllReduce(buf, buf, count, ncclFloat, ncclSum, e->comm, e->stream);
    if (nr != ncclSuccess)
        return set_error(TQB200_ERR_CUDA, "ncclAllReduce: %s", ncclGetErrorString(nr));
    return TQB200_OK;
#else
    (void)buf;
    (void)count;
    return set_error(TQB200_ERR_UNSUPPORTED, "built without NCCL");
#endif
}

int launch_lm_head(tqb200_engine *e);

// One decode step's kernels, stream-ordered on e->stream.
int launch_forward(tqb200_engine *e) {
    const tqb200_model_desc &d = e->d;
    cudaStream_t st = e->stream;
    const int G = e->tp, r = e->rank, Ga = e->ga;
    const int H = d.hidden, hd = d.head_dim;
    const int qd = d.n_heads * hd;
    const int Hl = d.n_heads / Ga, KVl = d.n_kv_heads / Ga;
    const int qdl = Hl * hd, kvdl = KVl * hd, Hs = H / Ga, Is = d.inter / G, Vs = d.vocab / G;
    const bool pdl = e->o.pdl != 0;
    const bool xa = Ga > 1;  // attention sharded: its rows and o_proj's are exchanged
    int *status = e->io_out + 1;
    float *attn_mine = e->attn + (size_t)e->ra * qdl;
    float *hidden_mine = e->hidden + (size_t)e->ra * Hs;
    TQ_TRY(mark(e, -1));
    TQ_TRY(launch_embed(e->embed, e->embed_dtype, e->io_in, H, d.group_size, e->hidden, st, 1,
                        p2p_on(e) ? e->epoch : nullptr));
    TQ_TRY(mark(e, K_EMBED));
    for (int l = 0; l < d.n_layers; ++l) {
        const DLayer &w = e->layers[l];
        e->cur_layer = l;
        auto vq = [&](const uint8_t *m, float *y, const float *resid, int rows, int p) {
            VqJob jb;
            jb.w = m;
            jb.y = y;
            jb.resid = resid;
            jb.rows = rows;
            jb.rot_sign = w.rot_sign[p];
            jb.rot_scale = w.rot_scale[p];
            jb.rot_bs = w.rot_bs[p];
            return jb;
        };
        auto vq_launch = [&](VqLaunch &a, int kind) {
            a.pdl = pdl;
            a.status = status;
            a.stamp = tl_next(e, kind);
            return launch_vq2_matvec(a, st);
        };
        if (w.vq2) {  // q/k/v (each with its own rotation) after the input RMSNorm
            VqLaunch a;
            a.job[0] = vq(w.q, e->q, nullptr, qdl, P_Q);
            a.job[1] = vq(w.k, e->k, nullptr, kvdl, P_K);
            a.job[2] = vq(w.v, e->v, nullptr, kvdl, P_V);
            a.n_jobs = 3;
            a.K = H;
            a.x = {X_RMSNORM, e->hidden, w.input_ln, d.rms_eps, nullptr};
            TQ_TRY(vq_launch(a, K_QKV));
            TQ_TRY(mark(e, K_QKV));
        } else {   // q/k/v with the input RMSNorm fused into the prologue, biases into the epilogue
            I4Job j[3] = {{w.q, e->q, w.q_bias, nullptr, qdl},
                          {w.k, e->k, w.k_bias, nullptr, kvdl},
                          {w.v, e->v, w.v_bias, nullptr, kvdl}};
            I4LaunchOpts o;
            o.x = {X_RMSNORM, e->hidden, w.input_ln, d.rms_eps, nullptr};
            o.pdl = pdl;
            o.status = status;
            o.stamp = tl_next(e, K_QKV);
            // the previous dense layer's down rows (a MoE layer's combine is local)
            if (l > 0 && !e->layers[l - 1].moe) o.xwait = xwait_of(e, (l - 1) * XS_PER_LAYER + XS_HID_D);
            TQ_TRY(launch_i4_matvec_ex(j, 3, H, d.group_size, o, st));
            TQ_TRY(mark(e, K_QKV));
        }
        char *kvb = (char *)e->kv;
        const size_t es = e->o.kv_fp16 ? 2 : 4;
        void *kc = kvb + (size_t)l * e->layer_stride * es;
        void *vc = kvb + ((size_t)d.n_layers + l) * e->layer_stride * es;
        {   // QK-norm + RoPE + KV append fused into the attention launch
            AttnArgs a{};
            a.q = e->q;
            a.k = kc;
            a.v = vc;
            a.kv_fp16 = e->o.kv_fp16;
            a.pos = e->io_in + 1;
            a.seq_len = 0;
            a.max_seq = e->o.max_seq_len;
            a.n_heads = Hl;
            a.n_kv_heads = KVl;
            a.head_dim = hd;
            a.scale = 1.0f / sqrtf((float)hd);
            a.nsplit = e->attn_nsplit;
            a.chunk_max = e->attn_chunk;
            a.partial = e->attn_part;
            a.tickets = e->attn_tickets;
            a.out = attn_mine;
            a.k_new = e->k;
            a.v_new = e->v;
            a.q_norm = w.q_norm;
            a.k_norm = w.k_norm;
            a.eps = d.rms_eps;
            a.cos_tab = e->cos_tab;
            a.sin_tab = e->sin_tab;
            a.pdl = pdl;
            a.status = status;
            a.stamp = tl_next(e, K_ATTN);
            a.put = xa ? xput(e, l * XS_PER_LAYER + XS_ATTN) : nullptr;
            TQ_TRY(launch_attention(a, st));
            if (xa) TQ_TRY(allgather(e, e->attn, qdl));
            TQ_TRY(mark(e, K_ATTN));
        }
        if (w.vq2) {
            VqLaunch a;
            a.job[0] = vq(w.o, hidden_mine, hidden_mine, Hs, P_O);
            a.K = qd;
            a.x = {X_PLAIN, e->attn, nullptr, 0.0f, nullptr};
            TQ_TRY(vq_launch(a, K_OPROJ));
            if (xa) TQ_TRY(allgather(e, e->hidden, Hs));
            TQ_TRY(mark(e, K_OPROJ));
        } else {   // o_proj, residual fused: hidden = hidden + W_o attn (this rank's rows)
            I4Job j{w.o, hidden_mine, nullptr, hidden_mine, Hs};
            I4LaunchOpts o;
            o.x = {X_PLAIN, e->attn, nullptr, 0.0f, nullptr};
            o.pdl = pdl;
            o.status = status;
            o.stamp = tl_next(e, K_OPROJ);
            if (xa) {
                o.xwait = xwait_of(e, l * XS_PER_LAYER + XS_ATTN);
                o.put = xput(e, l * XS_PER_LAYER + XS_HID_O);
            }
            TQ_TRY(launch_i4_matvec_ex(&j, 1, qd, d.group_size, o, st));
            if (xa) TQ_TRY(allgather(e, e->hidden, Hs));
            TQ_TRY(mark(e, K_OPROJ));
        }
        if (w.moe) {
            // MoE FFN (runtime/qwen_forward_token.cpp:478-631, no shared expert): router over
            // the post-attention RMSNorm -> top-k softmax -> gate/up of the chosen experts
            // (RMSNorm prologue, SwiGLU epilogue) -> down of each on its own activation ->
            // weighted sum in router order + residual
            const int k = d.experts_per_tok, mi = d.moe_inter, E = d.n_experts;
            // expert parallelism (tp > 1): this rank holds experts [r * El, (r + 1) * El);
            // the router runs whole on every rank (identical choices), each rank computes
            // the chosen experts it holds into zeroed slots, and a cross-rank sum of the
            // slots (exact: one non-zero term each) gives every rank all k outputs for the
            // combine in router order
            const int El = E / G;
            const int *eidx = G > 1 ? e->moe_local : e->moe_idx;
            if (w.router_f32) {
                TQ_TRY(launch_moe_router(e->hidden, w.post_ln, d.rms_eps, H, w.router_f32, E, k,
                                         e->moe_logits, e->moe_idx, e->moe_w, e->moe_ticket, pdl,
                                         st, tl_next(e, K_ROUTER),
                                         xa ? xwait_val(e, l * XS_PER_LAYER + XS_HID_O) : XWait(),
                                         status));
            } else {
                I4Job j{w.router_i4, e->moe_logits, nullptr, nullptr, E};
                I4LaunchOpts o;
                o.x = {X_RMSNORM, e->hidden, w.post_ln, d.rms_eps, nullptr};
                o.pdl = pdl;
                o.status = status;
                o.stamp = tl_next(e, K_ROUTER);
                if (xa) o.xwait = xwait_of(e, l * XS_PER_LAYER + XS_HID_O);
                TQ_TRY(launch_i4_matvec_ex(&j, 1, H, d.group_size, o, st));
                TQ_TRY(launch_topk_softmax(e->moe_logits, E, k, e->moe_idx, e->moe_w, st));
            }
            if (G > 1)
                TQ_TRY(launch_moe_ep_local(e->moe_idx, k, r * El, El, e->moe_local,
                                           e->p2p ? nullptr : e->moe_o, H, pdl, st));
            TQ_TRY(mark(e, K_ROUTER));
            {
                I4Job j[2] = {{w.ex_gate, e->moe_h, nullptr, nullptr, k * mi},
                              {w.ex_up, e->moe_u, nullptr, nullptr, k * mi}};
                I4LaunchOpts o;
                o.x = {X_RMSNORM, e->hidden, w.post_ln, d.rms_eps, nullptr};
                o.pair_swiglu = true;
                o.eidx = eidx;
                o.estride = (long long)w.ex_gu_stride;
                o.erows = mi;
                o.nslots = k;
                o.n_experts = El;
                o.pdl = pdl;
                o.status = status;
                o.stamp = tl_next(e, K_GATEUP);
                if (xa) o.xwait = xwait_of(e, l * XS_PER_LAYER + XS_HID_O);
                TQ_TRY(launch_i4_matvec_ex(j, 2, H, d.group_size, o, st));
                TQ_TRY(mark(e, K_GATEUP));
            }
            {
                I4Job j{w.ex_down, e->moe_o, nullptr, nullptr, k * H};
                I4LaunchOpts o;
                o.x = {X_PLAIN, e->moe_h, nullptr, 0.0f, nullptr};
                o.eidx = eidx;
                o.estride = (long long)w.ex_down_stride;
                o.erows = H;
                o.nslots = k;
                o.n_experts = El;
                o.xslots = true;
                o.pdl = pdl;
                o.status = status;
                o.stamp = tl_next(e, K_DOWN);
                o.put = xput(e, l * XS_PER_LAYER + XS_FFN);
                TQ_TRY(launch_i4_matvec_ex(&j, 1, mi, d.group_size, o, st));
                TQ_TRY(allreduce_sum(e, e->moe_o, (size_t)k * H));
                TQ_TRY(mark(e, K_DOWN));
            }
            TQ_TRY(launch_moe_combine(e->hidden, e->moe_o, e->moe_w, k, H, pdl, st,
                                      tl_next(e, K_COMBINE),
                                      xwait_val(e, l * XS_PER_LAYER + XS_FFN), status));
            TQ_TRY(mark(e, K_COMBINE));
            continue;
        }
        if (w.vq2) {
            VqLaunch a;
            a.job[0] = vq(w.gate, e->act + (size_t)r * Is, nullptr, Is, P_GATE);
            a.job[1] = vq(w.up, e->up, nullptr, Is, P_UP);
            a.n_jobs = 2;
            a.pair_swiglu = true;
            a.K = H;
            a.x = {X_RMSNORM, e->hidden, w.post_ln, d.rms_eps, nullptr};
            TQ_TRY(vq_launch(a, K_GATEUP));
            TQ_TRY(allgather(e, e->act, Is));
            TQ_TRY(mark(e, K_GATEUP));
        } else {   // gate/up in one pass per row block (post-attention RMSNorm in the prologue),
            // SwiGLU of each (gate, up) row pair in the epilogue -> act
            I4Job j[2] = {{w.gate, e->act + (size_t)r * Is, nullptr, nullptr, Is},
                          {w.up, e->up, nullptr, nullptr, Is}};
            I4LaunchOpts o;
            o.x = {X_RMSNORM, e->hidden, w.post_ln, d.rms_eps, nullptr};
            o.pair_swiglu = true;
            o.pdl = pdl;
            o.status = status;
            o.stamp = tl_next(e, K_GATEUP);
            o.xwait = xwait_of(e, l * XS_PER_LAYER + XS_HID_O);
            o.put = xput(e, l * XS_PER_LAYER + XS_FFN);
            TQ_TRY(launch_i4_matvec_ex(j, 2, H, d.group_size, o, st));
            TQ_TRY(allgather(e, e->act, Is));
            TQ_TRY(mark(e, K_GATEUP));
        }
        if (w.vq2) {
            VqLaunch a;
            a.job[0] = vq(w.down, hidden_mine, hidden_mine, Hs, P_DOWN);
            a.K = d.inter;
            a.x = {X_PLAIN, e->act, nullptr, 0.0f, nullptr};
            TQ_TRY(vq_launch(a, K_DOWN));
            TQ_TRY(allgather(e, e->hidden, Hs));
            TQ_TRY(mark(e, K_DOWN));
        } else {   // down with the residual in the epilogue
            I4Job j{w.down, hidden_mine, nullptr, hidden_mine, Hs};
            I4LaunchOpts o;
            o.x = {X_PLAIN, e->act, nullptr, 0.0f, nullptr};
            o.pdl = pdl;
            o.status = status;
            o.stamp = tl_next(e, K_DOWN);
            o.xwait = xwait_of(e, l * XS_PER_LAYER + XS_FFN);
            o.put = xput(e, l * XS_PER_LAYER + XS_HID_D);
            TQ_TRY(launch_i4_matvec_ex(&j, 1, d.inter, d.group_size, o, st));
            TQ_TRY(allgather(e, e->hidden, Hs));
            TQ_TRY(mark(e, K_DOWN));
        }
    }
    return launch_lm_head(e);
}

// lm_head over e->hidden with the final RMSNorm in the prologue and the greedy argmax in
// the epilogue (token -> io_out[0]).
int launch_lm_head(tqb200_engine *e) {
    const tqb200_model_desc &d = e->d;
    cudaStream_t st = e->stream;
    const int G = e->tp, r = e->rank;
    const int H = d.hidden, Vs = d.vocab / G;
    const bool pdl = e->o.pdl != 0;
    int *status = e->io_out + 1;
    {
        I4Job j{e->lm_head, e->logits + (size_t)r * Vs, nullptr, nullptr, Vs};
        I4LaunchOpts o;
        o.x = {X_RMSNORM, e->hidden, e->final_norm, d.rms_eps, nullptr};
        o.argmax.part_v = e->am_v;
        o.argmax.part_i = e->am_i;
        o.argmax.ticket = e->am_ticket;
        o.argmax.row_offset = r * Vs;
        if (G == 1) {
            o.argmax.token = e->io_out;
        } else {
            o.argmax.token = &e->pairs[r].i;
            o.argmax.value = &e->pairs[r].v;
        }
        o.pdl = pdl;
        o.status = status;
        o.stamp = tl_next(e, K_LMHEAD);
        const int L = d.n_layers;
        if (!e->layers[L - 1].moe) o.xwait = xwait_of(e, (L - 1) * XS_PER_LAYER + XS_HID_D);
        o.put = xput(e, xslot_lm(d));
        TQ_TRY(launch_i4_matvec_ex(&j, 1, H, d.group_size, o, st));
        if (G > 1) {
            TQ_TRY(allgather(e, reinterpret_cast<float *>(e->pairs), 2));
            TQ_TRY(allgather(e, e->logits, Vs));
            TQ_TRY(launch_argmax_pairs(e->pairs, G, e->io_out, st, xwait_val(e, xslot_lm(d)),
                                       status));
        }
        TQ_TRY(mark(e, K_LMHEAD));
    }
    return TQB200_OK;
}

int capture(tqb200_engine *e, bool with_feed, cudaGraph_t *graph, cudaGraphExec_t *exec) {
    TQ_CUDA_TRY(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    // the generate graph carries the timeline stamps while a timeline is set
    e->tl_capture = with_feed && e->tl != nullptr;
    e->tl_kind.clear();
    int st = launch_forward(e);
    e->tl_capture = false;
    if (st == TQB200_OK && with_feed) {
        feed_next_kernel<<<1, 1, 0, e->stream>>>(e->io_in, e->io_out, e->gen_tokens, e->gen_count);
        if (cudaGetLastError() != cudaSuccess) st = set_error(TQB200_ERR_CUDA, "feed launch failed");
    }
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
    if (st) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    TQ_CUDA_TRY(ce);
    *graph = g;
    TQ_CUDA_TRY(cudaGraphInstantiate(exec, g, 0));
    return TQB200_OK;
}

int check_status(tqb200_engine *e) {
    if (e->h_io[3] != 0) {
        const int code = e->h_io[3];
        e->h_io[3] = 0;
        cudaMemsetAsync(e->io_out + 1, 0, 4, e->stream);
        cudaStreamSynchronize(e->stream);
        return set_error(TQB200_ERR_TIMEOUT, "device wait timed out (code %d) at position %d",
                         code, e->pos);
    }
    return TQB200_OK;
}

void free_engine(tqb200_engine *e) {
    if (!e) return;
    if (e->exec) cudaGraphExecDestroy(e->exec);
    if (e->graph) cudaGraphDestroy(e->graph);
    if (e->loop_exec) cudaGraphExecDestroy(e->loop_exec);
    if (e->loop_graph) cudaGraphDestroy(e->loop_graph);
    for (auto ev : e->ev)
        if (ev) cudaEventDestroy(ev);
    for (auto ev : e->prof_ev) cudaEventDestroy(ev);
#ifdef TQB200_HAVE_NCCL
    if (e->comm) ncclCommDestroy(e->comm);
#endif
    for (void *p : e->peer_maps) cudaIpcCloseMemHandle(p);
    for (void *p : e->allocs) cudaFree(p);
    if (e->tl) cudaFree(e->tl);
    if (e->h_io) cudaFreeHost(e->h_io);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
}

int create_impl(const tqb200_model_desc *desc, const tqb200_engine_opts *opts, tqb200_engine *e) {
    e->d = *desc;
    e->o = *opts;
    const char *dbg = getenv("TQB200_DEBUG_SYNC");
    if (dbg && dbg[0] == '1') {
        e->debug_sync = true;
        e->o.use_graph = 0;
    }
    const tqb200_model_desc &d = e->d;
    TQ_TRY(validate(d, e->o));
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return set_error(TQB200_ERR_NO_DEVICE, "no CUDA device visible");
    }
    if (e->o.device >= 0) TQ_CUDA_TRY(cudaSetDevice(e->o.device));
    TQ_CUDA_TRY(cudaGetDevice(&e->device));
    TQ_CUDA_TRY(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    const int H = d.hidden, hd = d.head_dim, qd = d.n_heads * hd, kvd = d.n_kv_heads * hd;
    e->tp = e->o.tp_size > 0 ? e->o.tp_size : 1;
    e->rank = e->o.tp_rank;
    const int G = e->tp, r = e->rank;
    TQ_CHECK_ARG(r >= 0 && r < G, "tp_rank %d outside tp_size %d", r, G);
    e->ga = d.model_type == TQB200_MODEL_QWEN3_MOE ? 1 : G;
    e->ra = e->ga > 1 ? r : 0;
    const int Ga = e->ga;
    TQ_CHECK_ARG(d.n_heads % Ga == 0 && d.n_kv_heads % Ga == 0 && H % Ga == 0 &&
                     (Ga == 1 || d.inter % G == 0) && d.vocab % G == 0,
                 "tp_size %d must divide heads %d, kv heads %d, hidden %d, inter %d, vocab %d", G,
                 d.n_heads, d.n_kv_heads, H, d.inter, d.vocab);
    const int ra = e->ra;
    const int qdl = qd / Ga, kvdl = kvd / Ga, Hs = H / Ga, Is = d.inter / G, Vs = d.vocab / G;
#ifdef TQB200_HAVE_NCCL
    if (G > 1) {
        ncclUniqueId id;
        static_assert(sizeof(id) == sizeof(e->o.nccl_id), "NCCL id size");
        memcpy(&id, e->o.nccl_id, sizeof(id));
        const ncclResult_t nr = ncclCommInitRank(&e->comm, G, id, r);
        if (nr != ncclSuccess)
            return set_error(TQB200_ERR_CUDA, "ncclCommInitRank(rank %d of %d): %s", r, G,
                             ncclGetErrorString(nr));
    }
#else
    TQ_CHECK_ARG(G == 1, "this build has no NCCL: tp_size must be 1");
#endif
    e->layers.resize(d.n_layers);
    for (int l = 0; l < d.n_layers; ++l) {
        const tqb200_layer &s = d.layers[l];
        DLayer &w = e->layers[l];
        const int wdt = d.layers[0].q_proj.dtype;
        TQ_CHECK_ARG(wdt == TQB200_DT_I4 || wdt == TQB200_DT_VQ2,
                     "projection dtype %d: the engine path is i4 or VQ2", wdt);
        TQ_TRY(need_mat(s.q_proj, qd, H, wdt, "q_proj", l));
        TQ_TRY(need_mat(s.k_proj, kvd, H, wdt, "k_proj", l));
        TQ_TRY(need_mat(s.v_proj, kvd, H, wdt, "v_proj", l));
        TQ_TRY(need_mat(s.o_proj, H, qd, wdt, "o_proj", l));
        w.moe = d.model_type == TQB200_MODEL_QWEN3_MOE;
        if (w.moe) {
            TQ_CHECK_ARG(wdt == TQB200_DT_I4, "layer %d: MoE layers need i4 projections", l);
            TQ_CHECK_ARG(s.router.data && s.router.rows == d.n_experts && s.router.cols == H &&
                             (s.router.dtype == TQB200_DT_F32 || s.router.dtype == TQB200_DT_I4),
                         "layer %d: router must be f32 or i4 [n_experts x hidden]", l);
            TQ_CHECK_ARG(s.expert_gate && s.expert_up && s.expert_down, "layer %d: experts missing", l);
            for (int x = 0; x < d.n_experts; ++x) {
                TQ_TRY(need_mat(s.expert_gate[x], d.moe_inter, H, TQB200_DT_I4, "expert gate", l));
                TQ_TRY(need_mat(s.expert_up[x], d.moe_inter, H, TQB200_DT_I4, "expert up", l));
                TQ_TRY(need_mat(s.expert_down[x], H, d.moe_inter, TQB200_DT_I4, "expert down", l));
            }
        } else {
            TQ_TRY(need_mat(s.gate_proj, d.inter, H, wdt, "gate_proj", l));
            TQ_TRY(need_mat(s.up_proj, d.inter, H, wdt, "up_proj", l));
            TQ_TRY(need_mat(s.down_proj, H, d.inter, wdt, "down_proj", l));
        }
        TQ_CHECK_ARG(s.input_ln && s.post_ln, "layer %d: norms missing", l);
        TQ_CHECK_ARG((s.q_norm == nullptr) == (s.k_norm == nullptr),
                     "layer %d: q_norm/k_norm must both be present or both absent", l);
        w.vq2 = wdt == TQB200_DT_VQ2;
        const tqb200_rotation *rots[P_N] = {&s.rot_q, &s.rot_k, &s.rot_v, &s.rot_o,
                                            &s.rot_gate, &s.rot_up, &s.rot_down};
        if (!w.vq2) {
            for (int p = 0; p < P_N; ++p)
                TQ_CHECK_ARG(!rots[p]->sign && !rots[p]->scale,
                             "layer %d: BiIP rotations are only on the engine's VQ2 path", l);
        } else {
            TQ_CHECK_ARG(!s.q_bias && !s.k_bias && !s.v_bias,
                         "layer %d: q/k/v biases are not supported with VQ2 projections", l);
            const int rot_dim[P_N] = {H, H, H, qd, H, H, d.inter};
            for (int p = 0; p < P_N; ++p) {
                TQ_CHECK_ARG(rots[p]->sign || !rots[p]->scale,
                             "layer %d: rotation %d has a scale but no sign", l, p);
                const int bs = rots[p]->block_size;
                TQ_CHECK_ARG(bs >= 0 && (bs & (bs - 1)) == 0, "layer %d: rotation block %d", l, bs);
                TQ_TRY(up_vec(e, rots[p]->sign, rot_dim[p], &w.rot_sign[p]));
                TQ_TRY(up_vec(e, rots[p]->scale, rot_dim[p], &w.rot_scale[p]));
                w.rot_bs[p] = bs;
            }
        }
        TQ_TRY(up_vec(e, s.input_ln, H, &w.input_ln));
        TQ_TRY(up_vec(e, s.post_ln, H, &w.post_ln));
        // this rank's rows (all rows when tp == 1)
        auto up_rows = [&](const tqb200_matrix &m, int r0, int n, const uint8_t **o) {
            return w.vq2 ? up_vq2_rows(e, m, r0, n, o) : up_i4_rows(e, m, r0, n, o);
        };
        TQ_TRY(up_rows(s.q_proj, ra * qdl, qdl, &w.q));
        TQ_TRY(up_rows(s.k_proj, ra * kvdl, kvdl, &w.k));
        TQ_TRY(up_rows(s.v_proj, ra * kvdl, kvdl, &w.v));
        TQ_TRY(up_rows(s.o_proj, ra * Hs, Hs, &w.o));
        if (w.moe) {
            TQ_TRY(up_experts(e, s, d, w));
        } else {
            TQ_TRY(up_rows(s.gate_proj, r * Is, Is, &w.gate));
            TQ_TRY(up_rows(s.up_proj, r * Is, Is, &w.up));
            TQ_TRY(up_rows(s.down_proj, r * Hs, Hs, &w.down));
        }
        TQ_TRY(up_vec(e, s.q_bias ? s.q_bias + ra * qdl : nullptr, qdl, &w.q_bias));
        TQ_TRY(up_vec(e, s.k_bias ? s.k_bias + ra * kvdl : nullptr, kvdl, &w.k_bias));
        TQ_TRY(up_vec(e, s.v_bias ? s.v_bias + ra * kvdl : nullptr, kvdl, &w.v_bias));
        TQ_TRY(up_vec(e, s.q_norm, hd, &w.q_norm));
        TQ_TRY(up_vec(e, s.k_norm, hd, &w.k_norm));
    }
    e->embed_dtype = d.embed.dtype;
    TQ_TRY(upload_bytes(e, d.embed.data, mat_bytes(d.embed, d.group_size), &e->embed));
    if (G == 1 && d.lm_head.data == d.embed.data && d.embed.dtype == TQB200_DT_I4)
        e->lm_head = (const uint8_t *)e->embed;  // tied compact-i4 embedding
    else
        TQ_TRY(up_i4_rows(e, d.lm_head, r * Vs, Vs, &e->lm_head));
    TQ_TRY(up_vec(e, d.final_norm, H, &e->final_norm));
    TQ_TRY(build_rope_tables(e));

    // The exchange arena (one allocation, the same layout on every rank, mapped by the
    // peers when the peer exchange opens): the activations, the MoE buffers, then the
    // exchange counters, tickets and epoch.
    void *p;
    const size_t act = ((size_t)H * 2 + qd * 2 + kvd * 2 + (size_t)d.inter * 3 + d.vocab + 64 + 63) &
                       ~(size_t)63;
    const bool moe_model = d.model_type == TQB200_MODEL_QWEN3_MOE;
    const size_t moe_n = moe_model ? ((size_t)d.n_experts + 2 * (size_t)d.experts_per_tok * d.moe_inter +
                                      (size_t)d.experts_per_tok * H + 4 * 64 + 63) & ~(size_t)63
                                   : 0;
    const size_t nx = (size_t)n_xslots(d);
    const size_t arena = (act + moe_n) * 4 + nx * 8 + nx * 4 + 256;
    TQ_TRY(dev_alloc(e, arena, &p));
    TQ_CUDA_TRY(cudaMemset(p, 0, arena));
    e->xarena = p;
    e->xcnt = reinterpret_cast<unsigned long long *>((char *)p + (act + moe_n) * 4);
    e->xticket = reinterpret_cast<unsigned int *>(e->xcnt + nx);
    e->epoch = e->xticket + nx;
    float *f = (float *)p;
    e->hidden = f, f += H;
    e->q = f, f += qd;
    e->k = f, f += kvd;
    e->v = f, f += kvd;
    e->attn = f, f += qd;   // full width: rank r's heads at [r*qdl, (r+1)*qdl)
    e->gate = f, f += d.inter;
    e->up = f, f += d.inter;
    e->act = f, f += d.inter;
    e->logits = f, f += d.vocab;
    e->pairs = reinterpret_cast<ArgPair *>(f);
    TQ_CHECK_ARG(G <= 32, "tp_size %d above 32", G);
    if (moe_model) {
        const int k = d.experts_per_tok, mi = d.moe_inter;
        float *m = (float *)e->xarena + act;  // 256-byte aligned
        e->moe_h = m, m += (size_t)k * mi;       // 16-byte aligned rows of mi floats
        e->moe_u = m, m += (size_t)k * mi;
        e->moe_o = m, m += (size_t)k * H;
        e->moe_logits = m, m += ((d.n_experts + 63) / 64) * 64;
        e->moe_w = m, m += 64;
        e->moe_idx = (int *)m, m += 64;
        e->moe_local = (int *)m, m += 64;
        e->moe_ticket = (unsigned int *)m;
    }
    e->layer_stride = (size_t)(d.n_kv_heads / Ga) * e->o.max_seq_len * hd;
    const size_t kv_bytes = 2 * (size_t)d.n_layers * e->layer_stride * (e->o.kv_fp16 ? 2 : 4);
    TQ_TRY(dev_alloc(e, kv_bytes, &e->kv));
    TQ_CUDA_TRY(cudaMemset(e->kv, 0, kv_bytes));
    TQ_TRY(attn_plan(d.n_kv_heads / Ga, e->o.max_seq_len, &e->attn_nsplit, &e->attn_chunk));
    TQ_TRY(dev_alloc(e, attn_partial_floats(d.n_heads, hd, e->attn_nsplit) * 4, &p));
    e->attn_part = (float *)p;
    const int slots = i4_argmax_slots(d.vocab, H, d.group_size);
    TQ_TRY(dev_alloc(e, (size_t)slots * 8 + 256 + (size_t)d.n_kv_heads * 4 + 64, &p));
    TQ_CUDA_TRY(cudaMemset(p, 0, (size_t)slots * 8 + 256 + (size_t)d.n_kv_heads * 4 + 64));
    e->am_v = (float *)p;
    e->am_i = (int *)((char *)p + (size_t)slots * 4);
    e->am_ticket = (unsigned int *)((char *)p + (size_t)slots * 8);
    e->io_in = (int *)((char *)p + (size_t)slots * 8 + 64);
    e->io_out = (int *)((char *)p + (size_t)slots * 8 + 128);
    e->attn_tickets = (unsigned int *)((char *)p + (size_t)slots * 8 + 256);
    TQ_TRY(dev_alloc(e, (size_t)(e->o.max_seq_len + 8) * 4, &p));
    e->gen_count = (int *)p;
    e->gen_tokens = (int *)p + 8;
    TQ_CUDA_TRY(cudaMallocHost(&e->h_io, 64));
    memset(e->h_io, 0, 64);
    TQ_CUDA_TRY(cudaEventCreate(&e->ev[0]));
    TQ_CUDA_TRY(cudaEventCreate(&e->ev[1]));
    return TQB200_OK;
}

// ------------------------------------------------------------------ prefill
// A prompt runs in chunks of up to Prefill::cap tokens.  Per layer and chunk:
//   rmsnorm rows -> q/k/v (one grouped tensor-core matmul, bias in the epilogue)
//   -> QK-norm + RoPE + KV append (batched) -> causal attention over the cache
//   -> o_proj (residual in the epilogue) -> rmsnorm rows -> FFN:
//      dense: gate/up (grouped) -> SwiGLU -> down (residual in the epilogue)
//      MoE:   router logits -> top-k softmax -> device plan (bucket by expert) ->
//             gate/up of every expert with tokens in one planned launch -> SwiGLU
//             -> down likewise -> weighted sum per token in router order + residual
// then, after the last chunk, the decode lm_head on the last token's hidden state.
// Every projection uses the tile-contiguous copies made by the first prefill.
constexpr int kPrefillChunk = 512;

bool prefill_batched(const tqb200_engine *e) {
    const tqb200_model_desc &d = e->d;
    // tensor parallelism: MoE models only (attention whole on every rank, the experts
    // sharded); dense models under tensor parallelism run the prompt as decode steps
    return (e->tp == 1 || e->ga == 1) && !e->layers[0].vq2 && mm_group_supported(d.group_size) &&
           attn_prefill_supported(d.n_heads, d.n_kv_heads, d.head_dim);
}

// A tensor map over E matrices of M x K (matrix x at w + x * stride) into the next slot
// of the device map array; false when the layout admits none.
bool weight_map(tqb200_engine *e, const uint8_t *w, int M, int K, int E, size_t stride, PW *out) {
    Prefill &P = e->pf;
    if (P.n_maps >= P.cap_maps) return false;
    uint8_t *h = P.hmaps.data() + P.n_maps * 128;
    if (!mm_encode_weight_map(w, M, K, e->d.group_size, E, stride, h)) return false;
    out->w = nullptr;
    out->tm = P.maps + P.n_maps * 128;
    ++P.n_maps;
    return true;
}

int repack(tqb200_engine *e, const uint8_t *w, int M, int K, PW *out) {
    if (weight_map(e, w, M, K, 1, 0, out)) return TQB200_OK;
    const int G = e->d.group_size;
    void *p;
    TQ_TRY(dev_alloc(e, mm_repacked_bytes(M, K, G), &p));
    TQ_TRY(launch_mm_repack_w(w, M, K, G, (uint8_t *)p, e->stream));
    e->pf.copy_bytes += mm_repacked_bytes(M, K, G);
    out->w = (const uint8_t *)p;
    out->tm = nullptr;
    return TQB200_OK;
}

// E experts of M x K at `stride` bytes apart: one map over all of them, or one repacked
// buffer, expert x at x * *ostride.
int repack_experts(tqb200_engine *e, const uint8_t *w, size_t stride, int E, int M, int K,
                   PW *out, size_t *ostride) {
    if (weight_map(e, w, M, K, E, stride, out)) {
        *ostride = stride;
        return TQB200_OK;
    }
    const int G = e->d.group_size;
    const size_t one = (mm_repacked_bytes(M, K, G) + 255) & ~(size_t)255;
    const size_t rb = tqb200_i4_row_bytes(K, G);
    void *p;
    TQ_TRY(dev_alloc(e, one * E, &p));
    e->pf.copy_bytes += one * E;
    if (stride == (size_t)M * rb && M % kMmTileRows == 0 && one == mm_repacked_bytes(M, K, G)) {
        // rows of consecutive experts are contiguous and no tile straddles two experts
        TQ_TRY(launch_mm_repack_w(w, M * E, K, G, (uint8_t *)p, e->stream));
    } else {
        for (int x = 0; x < E; ++x)
            TQ_TRY(launch_mm_repack_w(w + (size_t)x * stride, M, K, G, (uint8_t *)p + (size_t)x * one,
                                      e->stream));
    }
    out->w = (const uint8_t *)p;
    out->tm = nullptr;
    *ostride = one;
    return TQB200_OK;
}

int prefill_setup(tqb200_engine *e) {
    Prefill &P = e->pf;
    if (P.ready) return TQB200_OK;
    const tqb200_model_desc &d = e->d;
    const int H = d.hidden, qd = d.n_heads * d.head_dim, kvd = d.n_kv_heads * d.head_dim;
    const int G = d.group_size;
    const bool moe = d.model_type == TQB200_MODEL_QWEN3_MOE;
    const int k = moe ? d.experts_per_tok : 1, E = moe ? d.n_experts : 0, mi = d.moe_inter;
    const int El = E / e->tp;  // this rank's experts (expert parallelism)
    P.cap = std::min(kPrefillChunk, e->o.max_seq_len);
    if (moe)  // the plan kernel holds the chunk's n*k assignments in shared memory
        while (P.cap > 1 && moe_plan_smem_bytes(P.cap, k, E) > kMoePlanMaxSmem) P.cap /= 2;
    const int cap = P.cap;
    P.layers.resize(d.n_layers);
    void *p;
    P.cap_maps = (size_t)11 * d.n_layers;  // q k v o + gate up down router + 3 expert kinds
    P.hmaps.assign(P.cap_maps * 128, 0);
    TQ_TRY(dev_alloc(e, P.cap_maps * 128, &p));
    P.maps = (uint8_t *)p;
    P.n_maps = 0;
    P.copy_bytes = 0;
    for (int l = 0; l < d.n_layers; ++l) {
        const DLayer &w = e->layers[l];
        PLayer &pl = P.layers[l];
        TQ_TRY(repack(e, w.q, qd, H, &pl.q));
        TQ_TRY(repack(e, w.k, kvd, H, &pl.k));
        TQ_TRY(repack(e, w.v, kvd, H, &pl.v));
        TQ_TRY(repack(e, w.o, H, qd, &pl.o));
        if (w.moe) {
            TQ_TRY(repack_experts(e, w.ex_gate, w.ex_gu_stride, El, mi, H, &pl.ex_gate, &pl.ex_gu_stride));
            TQ_TRY(repack_experts(e, w.ex_up, w.ex_gu_stride, El, mi, H, &pl.ex_up, &pl.ex_gu_stride));
            TQ_TRY(repack_experts(e, w.ex_down, w.ex_down_stride, El, H, mi, &pl.ex_down,
                                  &pl.ex_down_stride));
            if (w.router_i4) TQ_TRY(repack(e, w.router_i4, E, H, &pl.router));
        } else {
            TQ_TRY(repack(e, w.gate, d.inter, H, &pl.gate));
            TQ_TRY(repack(e, w.up, d.inter, H, &pl.up));
            TQ_TRY(repack(e, w.down, H, d.inter, &pl.down));
        }
    }
    if (P.n_maps)
        TQ_CUDA_TRY(cudaMemcpy(P.maps, P.hmaps.data(), P.n_maps * 128, cudaMemcpyHostToDevice));
    const int I = moe ? 0 : d.inter;
    const size_t f = (size_t)cap * (2 * (size_t)H + 2 * (size_t)qd + 2 * (size_t)kvd + 2 * (size_t)I);
    TQ_TRY(dev_alloc(e, f * 4 + 16 * 64, &p));
    float *a = (float *)p;
    auto take = [&](size_t n) {  // 64-byte aligned carve
        float *r = a;
        a += (n + 15) & ~(size_t)15;
        return r;
    };
    P.hidden = take((size_t)cap * H);
    P.xn = take((size_t)cap * H);
    P.q = take((size_t)cap * qd);
    P.attn = take((size_t)cap * qd);
    P.k = take((size_t)cap * kvd);
    P.v = take((size_t)cap * kvd);
    if (I) {
        P.gate = take((size_t)cap * I);
        P.up = take((size_t)cap * I);
    }
    TQ_TRY(dev_alloc(e, (size_t)(cap + 16) * 4, &p));
    P.io = (int *)p;
    long long pe = std::max({mm_plane_elems(H, cap, G), mm_plane_elems(qd, cap, G),
                             I ? mm_plane_elems(I, cap, G) : 0LL});
    if (moe) {
        P.moe_nt = 64;
        pe = std::max({pe, moe_plan_plane_elems(cap, k, E, H, G), moe_plan_plane_elems(cap, k, E, mi, G)});
        const size_t A = (size_t)cap * k;
        P.max_tiles_gu = 2 * moe_plan_max_tiles(cap, k, E, mi, P.moe_nt);
        P.max_tiles_dn = moe_plan_max_tiles(cap, k, E, H, P.moe_nt);
        const size_t mf = (size_t)cap * E + 2 * A + 2 * A * mi + A * H + 64 * 8;
        TQ_TRY(dev_alloc(e, mf * 4, &p));
        float *m = (float *)p;
        auto mt = [&](size_t n) {
            float *r = m;
            m += (n + 15) & ~(size_t)15;
            return r;
        };
        P.logits = mt((size_t)cap * E);
        P.wts = mt(A);
        P.idx = (int *)mt(A);
        P.mh = mt(A * mi);
        P.mu = mt(A * mi);
        P.mo = mt(A * H);
        const size_t mb = (size_t)moe_plan_max_cols(cap, k, E) / 8;
        const size_t ib = (2 * A + 4 + (size_t)P.max_tiles_gu + P.max_tiles_dn + mb) * 4 + 256;
        TQ_TRY(dev_alloc(e, ib, &p));
        int *ip = (int *)p;
        P.rows = ip, ip += A;
        P.slot = ip, ip += A;
        P.ntiles = ip, ip += 4;
        P.tile_gu = ip, ip += P.max_tiles_gu;
        P.tile_dn = ip, ip += P.max_tiles_dn;
        P.pack_map = ip;
        TQ_TRY(dev_alloc(e, sizeof(MmJob) * 3 * E + sizeof(MmPackJob) * 2 * E + 256, &p));
        P.jobs_gu = (MmJob *)p;
        P.jobs_dn = P.jobs_gu + 2 * E;
        P.pack_gu = (MmPackJob *)(P.jobs_dn + E);
        P.pack_dn = P.pack_gu + E;
    }
    TQ_TRY(dev_alloc(e, (size_t)pe * 2 * 2 + 256, &p));
    P.bhi = (uint16_t *)p;
    P.blo = (uint16_t *)((char *)p + (((size_t)pe * 2 + 255) & ~(size_t)255));
    TQ_TRY(dev_alloc(e, sizeof(MmJob) * 7 * d.n_layers, &p));
    P.jobs = (MmJob *)p;
    P.ready = true;
    return TQB200_OK;
}

// Host-planned jobs of every layer for a chunk of n tokens: per layer 7 slots,
// [q, k, v] [o] [gate, up | router] [down], and 4 launches (tile width, CTAs).
int prefill_plan(tqb200_engine *e, int n) {
    Prefill &P = e->pf;
    if (P.jobs_n == n) return TQB200_OK;
    const tqb200_model_desc &d = e->d;
    const int H = d.hidden, qd = d.n_heads * d.head_dim, kvd = d.n_kv_heads * d.head_dim;
    P.hjobs.assign((size_t)7 * d.n_layers, MmJob{});
    P.nt.assign((size_t)4 * d.n_layers, 16);
    P.tiles.assign((size_t)4 * d.n_layers, 0);
    for (int l = 0; l < d.n_layers; ++l) {
        const DLayer &w = e->layers[l];
        const PLayer &pl = P.layers[l];
        MmJob *j = &P.hjobs[(size_t)7 * l];
        auto group = [&](MmJob *js, int nj, int launch) {
            int mtot = 0;
            for (int i = 0; i < nj; ++i) mtot += js[i].M;
            const int nt = mm_tile_width(mtot, n);
            int t = 0;
            for (int i = 0; i < nj; ++i) {
                js[i].N = n;
                js[i].tile_begin = t;
                js[i].b_off = 0;
                t += mm_job_tiles(js[i].M, n, nt);
            }
            P.nt[(size_t)4 * l + launch] = nt;
            P.tiles[(size_t)4 * l + launch] = t;
        };
        auto job = [](const PW &wt, float *y, int M, const float *resid, const float *bias) {
            MmJob x{};
            x.w = wt.w;
            x.tmap = wt.tm;
            x.y = y;
            x.M = M;
            x.ldy = M;
            x.resid = resid;
            x.bias = bias;
            return x;
        };
        j[0] = job(pl.q, P.q, qd, nullptr, w.q_bias);
        j[1] = job(pl.k, P.k, kvd, nullptr, w.k_bias);
        j[2] = job(pl.v, P.v, kvd, nullptr, w.v_bias);
        group(j, 3, 0);
        j[3] = job(pl.o, P.hidden, H, P.hidden, nullptr);
        group(j + 3, 1, 1);
        if (w.moe) {
            if (pl.router) {
                j[4] = job(pl.router, P.logits, d.n_experts, nullptr, nullptr);
                group(j + 4, 1, 2);
            }
        } else {
            j[4] = job(pl.gate, P.gate, d.inter, nullptr, nullptr);
            j[5] = job(pl.up, P.up, d.inter, nullptr, nullptr);
            group(j + 4, 2, 2);
            j[6] = job(pl.down, P.hidden, H, P.hidden, nullptr);
            group(j + 6, 1, 3);
        }
    }
    TQ_CUDA_TRY(cudaMemcpyAsync(P.jobs, P.hjobs.data(), sizeof(MmJob) * P.hjobs.size(),
                                cudaMemcpyHostToDevice, e->stream));
    P.jobs_n = n;
    return TQB200_OK;
}

// One chunk of n tokens at positions p0..p0+n-1 (P.io already holds p0 and the tokens).
int prefill_chunk(tqb200_engine *e, int n, int p0) {
    Prefill &P = e->pf;
    const tqb200_model_desc &d = e->d;
    cudaStream_t st = e->stream;
    const int H = d.hidden, hd = d.head_dim, G = d.group_size;
    const int qd = d.n_heads * hd;
    int *status = e->io_out + 1;
    TQ_TRY(prefill_plan(e, n));
    TQ_TRY(launch_embed(e->embed, e->embed_dtype, P.io + 1, H, G, P.hidden, st, n));
    TQ_TRY(mark(e, K_EMBED));
    auto mm = [&](int l, int slot, int nj, int launch, int K) {
        const MmJob *hj = &P.hjobs[(size_t)7 * l + slot];
        return launch_matmul_i4_grouped(hj, nj > 1 ? P.jobs + (size_t)7 * l + slot : nullptr, nj, K,
                                        G, P.nt[(size_t)4 * l + launch], P.bhi, P.blo,
                                        P.tiles[(size_t)4 * l + launch], status, st);
    };
    auto pack = [&](const float *x, int K, const float *u = nullptr) {
        return launch_mm_pack_x(x, nullptr, K, K, n, G, P.bhi, P.blo, st, u);
    };
    for (int l = 0; l < d.n_layers; ++l) {
        const DLayer &w = e->layers[l];
        const PLayer &pl = P.layers[l];
        e->cur_layer = l;
        TQ_TRY(launch_rmsnorm(P.hidden, w.input_ln, P.xn, n, H, d.rms_eps, st));
        TQ_TRY(mark(e, K_NORM));
        TQ_TRY(pack(P.xn, H));
        TQ_TRY(mark(e, K_PACK));
        TQ_TRY(mm(l, 0, 3, 0, H));
        TQ_TRY(mark(e, K_QKV));
        const size_t es = e->o.kv_fp16 ? 2 : 4;
        char *kvb = (char *)e->kv;
        void *kc = kvb + (size_t)l * e->layer_stride * es;
        void *vc = kvb + ((size_t)d.n_layers + l) * e->layer_stride * es;
        {
            QkRopeKvArgs r{};
            r.q = P.q;
            r.k = P.k;
            r.v = P.v;
            r.q_norm = w.q_norm;
            r.k_norm = w.k_norm;
            r.eps = d.rms_eps;
            r.cos_tab = e->cos_tab;
            r.sin_tab = e->sin_tab;
            r.pos = P.io;
            r.kcache = kc;
            r.vcache = vc;
            r.kv_fp16 = e->o.kv_fp16;
            r.n_heads = d.n_heads;
            r.n_kv_heads = d.n_kv_heads;
            r.head_dim = hd;
            r.max_seq = e->o.max_seq_len;
            r.n_tokens = n;
            TQ_TRY(launch_qk_rope_kv(r, st));
            TQ_TRY(mark(e, K_ROPE_KV));
        }
        {
            AttnPrefillArgs a{};
            a.q = P.q;
            a.k = kc;
            a.v = vc;
            a.kv_fp16 = e->o.kv_fp16;
            a.p0 = p0;
            a.n = n;
            a.max_seq = e->o.max_seq_len;
            a.n_heads = d.n_heads;
            a.n_kv_heads = d.n_kv_heads;
            a.head_dim = hd;
            a.scale = 1.0f / sqrtf((float)hd);
            a.out = P.attn;
            TQ_TRY(launch_attn_prefill(a, st));
            TQ_TRY(mark(e, K_ATTN));
        }
        TQ_TRY(pack(P.attn, qd));
        TQ_TRY(mark(e, K_PACK));
        TQ_TRY(mm(l, 3, 1, 1, qd));
        TQ_TRY(mark(e, K_OPROJ));
        TQ_TRY(launch_rmsnorm(P.hidden, w.post_ln, P.xn, n, H, d.rms_eps, st));
        TQ_TRY(mark(e, K_NORM));
        if (!w.moe) {
            TQ_TRY(pack(P.xn, H));
            TQ_TRY(mark(e, K_PACK));
            TQ_TRY(mm(l, 4, 2, 2, H));
            TQ_TRY(mark(e, K_GATEUP));
            TQ_TRY(pack(P.gate, d.inter, P.up));  // SwiGLU formed by the pack
            TQ_TRY(mark(e, K_PACK));
            TQ_TRY(mm(l, 6, 1, 3, d.inter));
            TQ_TRY(mark(e, K_DOWN));
            continue;
        }
        const int k = d.experts_per_tok, E = d.n_experts, mi = d.moe_inter;
        if (pl.router) {
            TQ_TRY(pack(P.xn, H));
            TQ_TRY(mark(e, K_PACK));
            TQ_TRY(mm(l, 4, 1, 2, H));
        } else {
            TQ_TRY(launch_router_rows(P.xn, n, H, w.router_f32, E, P.logits, st));
        }
        TQ_TRY(launch_topk_rows(P.logits, n, E, k, P.idx, P.wts, st));
        TQ_TRY(mark(e, K_ROUTER));
        MoePlanArgs a{};
        a.idx = P.idx;
        a.n = n;
        a.k = k;
        a.E = E;
        a.G = G;
        a.H = H;
        a.mi = mi;
        a.nt = P.moe_nt;
        a.wg = pl.ex_gate.w;
        a.wu = pl.ex_up.w;
        a.wd = pl.ex_down.w;
        a.tmg = pl.ex_gate.tm;
        a.tmu = pl.ex_up.tm;
        a.tmd = pl.ex_down.tm;
        a.wgu_stride = (long long)pl.ex_gu_stride;
        a.wd_stride = (long long)pl.ex_down_stride;
        a.xn = P.xn;
        a.hbuf = P.mh;
        a.ubuf = P.mu;
        a.obuf = P.mo;
        a.rows = P.rows;
        a.slot = P.slot;
        a.jobs_gu = P.jobs_gu;
        a.jobs_dn = P.jobs_dn;
        a.tile_gu = P.tile_gu;
        a.tile_dn = P.tile_dn;
        a.ntiles = P.ntiles;
        a.pack_gu = P.pack_gu;
        a.pack_dn = P.pack_dn;
        a.pack_map = P.pack_map;
        a.status = status;
        if (e->tp > 1) {  // expert parallelism: this rank's experts only
            a.e0 = e->rank * (E / e->tp);
            a.e_local = E / e->tp;
        }
        TQ_TRY(launch_moe_plan(a, st));
        TQ_TRY(mark(e, K_PLAN));
        const int nbk = moe_plan_max_cols(n, k, E) / 8;
        const int tgu = 2 * moe_plan_max_tiles(n, k, E, mi, P.moe_nt);
        const int tdn = moe_plan_max_tiles(n, k, E, H, P.moe_nt);
        TQ_TRY(launch_mm_pack_x_mapped(P.pack_gu, P.pack_map, P.ntiles + 2, nbk, H, G, P.bhi, P.blo, st));
        TQ_TRY(mark(e, K_PACK));
        TQ_TRY(launch_matmul_i4_planned(P.jobs_gu, P.tile_gu, P.ntiles, tgu, H, G, P.moe_nt, P.bhi,
                                        P.blo, status, st));
        TQ_TRY(mark(e, K_GATEUP));
        TQ_TRY(launch_mm_pack_x_mapped(P.pack_dn, P.pack_map, P.ntiles + 2, nbk, mi, G, P.bhi, P.blo, st));
        TQ_TRY(mark(e, K_PACK));
        // expert parallelism: the bucket rows of other ranks' experts stay zero here, and
        // a cross-rank sum (exact: one non-zero term per row) gives every rank all rows
        if (e->tp > 1) TQ_CUDA_TRY(cudaMemsetAsync(P.mo, 0, (size_t)n * k * H * 4, st));
        TQ_TRY(launch_matmul_i4_planned(P.jobs_dn, P.tile_dn, P.ntiles + 1, tdn, mi, G, P.moe_nt,
                                        P.bhi, P.blo, status, st));
        if (e->tp > 1) TQ_TRY(allreduce_sum(e, P.mo, (size_t)n * k * H));
        TQ_TRY(mark(e, K_DOWN));
        TQ_TRY(launch_moe_combine_rows(P.hidden, P.mo, P.wts, P.slot, n, k, H, st));
        TQ_TRY(mark(e, K_COMBINE));
    }
    return TQB200_OK;
}

}  // namespace
}  // namespace tqb200

using namespace tqb200;

extern "C" {

void tqb200_engine_default_opts(tqb200_engine_opts *o) {
    if (!o) return;
    memset(o, 0, sizeof *o);
    o->max_seq_len = 512;
    o->kv_fp16 = 0;
    o->use_graph = 1;
    o->pdl = 1;
    o->device = -1;
    o->tp_size = 1;
    o->tp_rank = 0;
}

int tqb200_nccl_unique_id(unsigned char id[128]) {
    TQ_CHECK_ARG(id, "null id buffer");
#ifdef TQB200_HAVE_NCCL
    ncclUniqueId u;
    const ncclResult_t nr = ncclGetUniqueId(&u);
    if (nr != ncclSuccess)
        return set_error(TQB200_ERR_CUDA, "ncclGetUniqueId: %s", ncclGetErrorString(nr));
    memcpy(id, &u, sizeof u);
    return TQB200_OK;
#else
    return set_error(TQB200_ERR_UNSUPPORTED, "built without NCCL");
#endif
}

int tqb200_engine_create(const tqb200_model_desc *desc, const tqb200_engine_opts *opts,
                         tqb200_engine **out) {
    TQ_CHECK_ARG(desc && out, "null argument");
    *out = nullptr;
    tqb200_engine_opts o;
    if (opts)
        o = *opts;
    else
        tqb200_engine_default_opts(&o);
    auto *e = new tqb200_engine();
    const int st = create_impl(desc, &o, e);
    if (st) {
        free_engine(e);
        return st;
    }
    *out = e;
    return TQB200_OK;
}

int tqb200_engine_step(tqb200_engine *e, int token_id, int *next_token) {
    TQ_CHECK_ARG(e, "null engine");
    TQ_CHECK_ARG(token_id >= 0 && token_id < e->d.vocab, "token_id %d out of range [0, %d)",
                 token_id, e->d.vocab);
    TQ_CHECK_ARG(e->pos < e->o.max_seq_len, "position %d exceeds max_seq_len %d", e->pos,
                 e->o.max_seq_len);
    TQ_CUDA_TRY(cudaSetDevice(e->device));
    e->h_io[0] = token_id;
    e->h_io[1] = e->pos;
    TQ_CUDA_TRY(cudaMemcpyAsync(e->io_in, e->h_io, 8, cudaMemcpyHostToDevice, e->stream));
    if (e->o.use_graph) {
        if (!e->exec) TQ_TRY(capture(e, false, &e->graph, &e->exec));
        TQ_CUDA_TRY(cudaGraphLaunch(e->exec, e->stream));
    } else {
        TQ_TRY(launch_forward(e));
    }
    TQ_CUDA_TRY(cudaMemcpyAsync(e->h_io + 2, e->io_out, 8, cudaMemcpyDeviceToHost, e->stream));
    TQ_CUDA_TRY(cudaStreamSynchronize(e->stream));
    TQ_TRY(check_status(e));
    e->pos += 1;
    if (next_token) *next_token = e->h_io[2];
    return TQB200_OK;
}

int tqb200_engine_profile_prefill(tqb200_engine *e, const int *tokens, int n, float *ms_by_kind,
                                  int n_kinds, int *next_token) {
    TQ_CHECK_ARG(e && ms_by_kind && n_kinds > 0, "bad profile arguments");
    TQ_CHECK_ARG(prefill_batched(e), "this engine's prefill runs as decode steps");
    TQ_CUDA_TRY(cudaSetDevice(e->device));
    TQ_TRY(prefill_setup(e));  // first-use weight repack stays outside the timed launches
    e->prof = true;
    TQ_TRY(mark(e, -1));
    const int st = tqb200_engine_prefill(e, tokens, n, next_token);
    e->prof = false;
    for (int k = 0; k < n_kinds; ++k) ms_by_kind[k] = 0.0f;
    int rc = st;
    for (size_t i = 1; i < e->prof_ev.size() && rc == TQB200_OK; ++i) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, e->prof_ev[i - 1], e->prof_ev[i]) != cudaSuccess) {
            rc = set_error(TQB200_ERR_CUDA, "profile events");
            break;
        }
        const int k = e->prof_kind[i];
        if (k >= 0 && k < n_kinds) ms_by_kind[k] += ms;
    }
    for (auto ev : e->prof_ev) cudaEventDestroy(ev);
    e->prof_ev.clear();
    e->prof_kind.clear();
    return rc;
}

int tqb200_engine_prefill(tqb200_engine *e, const int *tokens, int n, int *next_token) {
    TQ_CHECK_ARG(e && tokens && n > 0, "bad prefill arguments");
    TQ_CHECK_ARG(e->pos + n <= e->o.max_seq_len, "positions %d..%d exceed max_seq_len %d", e->pos,
                 e->pos + n, e->o.max_seq_len);
    for (int i = 0; i < n; ++i)
        TQ_CHECK_ARG(tokens[i] >= 0 && tokens[i] < e->d.vocab, "token %d (%d) out of range [0, %d)",
                     i, tokens[i], e->d.vocab);
    if (!prefill_batched(e)) {  // token by token through the decode step
        int next = 0;
        for (int i = 0; i < n; ++i) TQ_TRY(tqb200_engine_step(e, tokens[i], &next));
        if (next_token) *next_token = next;
        return TQB200_OK;
    }
    TQ_CUDA_TRY(cudaSetDevice(e->device));
    TQ_TRY(prefill_setup(e));
    Prefill &P = e->pf;
    // expert parallelism: the prompt's cross-rank sums go over NCCL (the decode step's
    // peer-exchange counters stay in step with its epoch)
    struct XOff {
        tqb200_engine *e;
        explicit XOff(tqb200_engine *x) : e(x) { e->xoff = true; }
        ~XOff() { e->xoff = false; }
    } xoff_guard(e);
    std::vector<int> io((size_t)P.cap + 1);
    for (int c0 = 0; c0 < n; c0 += P.cap) {
        const int m = std::min(P.cap, n - c0);
        io[0] = e->pos + c0;
        std::copy(tokens + c0, tokens + c0 + m, io.begin() + 1);
        // pageable source: the call returns once the bytes are staged, so `io` is reusable
        TQ_CUDA_TRY(cudaMemcpyAsync(P.io, io.data(), (size_t)(m + 1) * 4, cudaMemcpyHostToDevice,
                                    e->stream));
        TQ_TRY(prefill_chunk(e, m, e->pos + c0));
        if (c0 + m == n) {  // the prompt's last token -> logits and the greedy next token
            TQ_CUDA_TRY(cudaMemcpyAsync(e->hidden, P.hidden + (size_t)(m - 1) * e->d.hidden,
                                        (size_t)e->d.hidden * 4, cudaMemcpyDeviceToDevice, e->stream));
            TQ_TRY(launch_lm_head(e));
            TQ_TRY(mark(e, K_LMHEAD));
        }
    }
    TQ_CUDA_TRY(cudaMemcpyAsync(e->h_io + 2, e->io_out, 8, cudaMemcpyDeviceToHost, e->stream));
    TQ_CUDA_TRY(cudaStreamSynchronize(e->stream));
    TQ_TRY(check_status(e));
    e->pos += n;
    if (next_token) *next_token = e->h_io[2];
    return TQB200_OK;
}

int tqb200_engine_generate(tqb200_engine *e, int token_id, int n_steps, int *out_tokens,
                           float *device_ms) {
    TQ_CHECK_ARG(e && out_tokens && n_steps >= 0, "bad generate arguments");
    TQ_CHECK_ARG(token_id >= 0 && token_id < e->d.vocab, "token_id %d out of range", token_id);
    TQ_CHECK_ARG(e->pos + n_steps <= e->o.max_seq_len, "positions %d..%d exceed max_seq_len %d",
                 e->pos, e->pos + n_steps, e->o.max_seq_len);
    if (n_steps == 0) return TQB200_OK;
    TQ_CUDA_TRY(cudaSetDevice(e->device));
    if (e->o.use_graph && !e->loop_exec) TQ_TRY(capture(e, true, &e->loop_graph, &e->loop_exec));
    e->h_io[0] = token_id;
    e->h_io[1] = e->pos;
    TQ_CUDA_TRY(cudaMemcpyAsync(e->io_in, e->h_io, 8, cudaMemcpyHostToDevice, e->stream));
    TQ_CUDA_TRY(cudaMemsetAsync(e->gen_count, 0, 4, e->stream));
    if (e->tl) {  // a fresh timeline record for the first tl_cap steps of this call
        TQ_CUDA_TRY(cudaMemsetAsync(e->tl, 0xFF, (size_t)e->tl_cap * e->tl_stride * 8, e->stream));
        e->tl_steps = std::min(n_steps, e->tl_cap);
    }
    TQ_CUDA_TRY(cudaEventRecord(e->ev[0], e->stream));
    for (int i = 0; i < n_steps; ++i) {
        if (e->o.use_graph) {
            TQ_CUDA_TRY(cudaGraphLaunch(e->loop_exec, e->stream));
        } else {
            TQ_TRY(launch_forward(e));
            feed_next_kernel<<<1, 1, 0, e->stream>>>(e->io_in, e->io_out, e->gen_tokens,
                                                     e->gen_count);
            TQ_CUDA_TRY(cudaGetLastError());
        }
    }
    TQ_CUDA_TRY(cudaEventRecord(e->ev[1], e->stream));
    TQ_CUDA_TRY(cudaMemcpyAsync(out_tokens, e->gen_tokens, (size_t)n_steps * 4,
                                cudaMemcpyDeviceToHost, e->stream));
    TQ_CUDA_TRY(cudaMemcpyAsync(e->h_io + 2, e->io_out, 8, cudaMemcpyDeviceToHost, e->stream));
    TQ_CUDA_TRY(cudaStreamSynchronize(e->stream));
    TQ_TRY(check_status(e));
    if (device_ms) TQ_CUDA_TRY(cudaEventElapsedTime(device_ms, e->ev[0], e->ev[1]));
    e->pos += n_steps;
    return TQB200_OK;
}

int tqb200_engine_profile_step(tqb200_engine *e, int token_id, float *ms_by_kind, int n_kinds,
                               int *next_token) {
    TQ_CHECK_ARG(e && ms_by_kind && n_kinds > 0, "bad profile arguments");
    TQ_CHECK_ARG(token_id >= 0 && token_id < e->d.vocab && e->pos < e->o.max_seq_len,
                 "bad token/position");
    TQ_CUDA_TRY(cudaSetDevice(e->device));
    e->h_io[0] = token_id;
    e->h_io[1] = e->pos;
    TQ_CUDA_TRY(cudaMemcpyAsync(e->io_in, e->h_io, 8, cudaMemcpyHostToDevice, e->stream));
    e->prof = true;
    const int st = launch_forward(e);
    e->prof = false;
    if (st) return st;
    TQ_CUDA_TRY(cudaMemcpyAsync(e->h_io + 2, e->io_out, 8, cudaMemcpyDeviceToHost, e->stream));
    TQ_CUDA_TRY(cudaStreamSynchronize(e->stream));
    for (int k = 0; k < n_kinds; ++k) ms_by_kind[k] = 0.0f;
    for (size_t i = 1; i < e->prof_ev.size(); ++i) {
        float ms = 0.0f;
        TQ_CUDA_TRY(cudaEventElapsedTime(&ms, e->prof_ev[i - 1], e->prof_ev[i]));
        const int k = e->prof_kind[i];
        if (k >= 0 && k < n_kinds) ms_by_kind[k] += ms;
    }
    for (auto ev : e->prof_ev) cudaEventDestroy(ev);
    e->prof_ev.clear();
    e->prof_kind.clear();
    TQ_TRY(check_status(e));
    e->pos += 1;
    if (next_token) *next_token = e->h_io[2];
    return TQB200_OK;
}

int tqb200_engine_reset(tqb200_engine *e) {
    TQ_CHECK_ARG(e, "null engine");
    e->pos = 0;  // KvCache::reset only rewinds seq_len (runtime/kv_cache.cpp:63-65)
    return TQB200_OK;
}

int tqb200_engine_destroy(tqb200_engine *e) {
    if (e) {
        cudaSetDevice(e->device);
        free_engine(e);
    }
    return TQB200_OK;
}

const float *tqb200_engine_logits(const tqb200_engine *e) { return e ? e->logits : nullptr; }

int tqb200_engine_copy_logits(const tqb200_engine *e, float *host, int n) {
    TQ_CHECK_ARG(e && host && n >= 0 && n <= e->d.vocab, "bad logits copy");
    TQ_CUDA_TRY(cudaSetDevice(e->device));
    TQ_CUDA_TRY(cudaMemcpy(host, e->logits, (size_t)n * 4, cudaMemcpyDeviceToHost));
    return TQB200_OK;
}

int tqb200_engine_position(const tqb200_engine *e) { return e ? e->pos : -1; }

int tqb200_engine_set_position(tqb200_engine *e, int pos) {
    TQ_CHECK_ARG(e && pos >= 0 && pos < e->o.max_seq_len, "bad position");
    e->pos = pos;
    return TQB200_OK;
}

int tqb200_engine_stream(const tqb200_engine *e, void **stream) {
    TQ_CHECK_ARG(e && stream, "null argument");
    *stream = e->stream;
    return TQB200_OK;
}

int tqb200_engine_kv_cache(const tqb200_engine *e, void **kv, size_t *bytes) {
    TQ_CHECK_ARG(e && kv && bytes, "null argument");
    *kv = e->kv;
    *bytes = 2 * (size_t)e->d.n_layers * e->layer_stride * (e->o.kv_fp16 ? 2 : 4);
    return TQB200_OK;
}

int tqb200_engine_weight_bytes(const tqb200_engine *e, size_t *bytes) {
    TQ_CHECK_ARG(e && bytes, "null argument");
    *bytes = e->weight_bytes;
    return TQB200_OK;
}

int tqb200_engine_prefill_copy_bytes(const tqb200_engine *e, size_t *bytes) {
    TQ_CHECK_ARG(e && bytes, "null argument");
    *bytes = e->pf.copy_bytes;
    return TQB200_OK;
}

int tqb200_engine_exchange_handle(tqb200_engine *e, unsigned char handle[64]) {
    TQ_CHECK_ARG(e && handle, "null argument");
    TQ_CUDA_TRY(cudaSetDevice(e->device));
    TQ_CUDA_TRY(cudaDeviceSynchronize());  // the arena's zeroed counters are in place
    cudaIpcMemHandle_t h;
    static_assert(sizeof(h) == 64, "CUDA IPC handle size");
    TQ_CUDA_TRY(cudaIpcGetMemHandle(&h, e->xarena));
    memcpy(handle, &h, 64);
    return TQB200_OK;
}

int tqb200_engine_open_exchange(tqb200_engine *e, const unsigned char *handles, int n_ranks) {
    TQ_CHECK_ARG(e && handles, "null argument");
    TQ_CHECK_ARG(n_ranks == e->tp && e->tp > 1, "open_exchange: %d handles for tp_size %d",
                 n_ranks, e->tp);
    TQ_CHECK_ARG(e->tp - 1 <= kMaxPeers, "open_exchange: tp_size %d above %d", e->tp,
                 kMaxPeers + 1);
    TQ_CHECK_ARG(!e->p2p, "open_exchange: already open");
    TQ_CHECK_ARG(!e->layers[0].vq2, "open_exchange: VQ2 models keep the NCCL all-gathers");
    TQ_CUDA_TRY(cudaSetDevice(e->device));
    TQ_CUDA_TRY(cudaStreamSynchronize(e->stream));
    int np = 0;
    for (int r = 0; r < n_ranks; ++r) {
        if (r == e->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, handles + 64 * (size_t)r, 64);
        void *peer = nullptr;
        const cudaError_t ce = cudaIpcOpenMemHandle(&peer, h, cudaIpcMemLazyEnablePeerAccess);
        if (ce != cudaSuccess) {
            for (void *q : e->peer_maps) cudaIpcCloseMemHandle(q);
            e->peer_maps.clear();
            return set_error(TQB200_ERR_CUDA, "open_exchange: rank %d's arena: %s", r,
                             cudaGetErrorString(ce));
        }
        e->peer_maps.push_back(peer);
        e->xdelta[np++] = (long long)((char *)peer - (char *)e->xarena);
    }
    e->n_peers = np;
    const int nx = n_xslots(e->d);
    e->xw_host.assign(nx, XWait());
    e->xp_host.assign(nx, XPut());
    for (int s = 0; s < nx; ++s) {
        XWait &w = e->xw_host[s];
        w.arrive = e->xcnt + s;
        w.epoch = e->epoch;
        w.ranks = (unsigned int)e->tp;
        XPut &p = e->xp_host[s];
        p.n_peers = np;
        for (int i = 0; i < np; ++i) p.delta[i] = e->xdelta[i];
        p.arrive = e->xcnt + s;
        p.ticket = e->xticket + s;
    }
    void *dw = nullptr, *dp = nullptr;
    TQ_TRY(dev_alloc(e, sizeof(XWait) * nx, &dw));
    TQ_TRY(dev_alloc(e, sizeof(XPut) * nx, &dp));
    TQ_CUDA_TRY(cudaMemcpy(dw, e->xw_host.data(), sizeof(XWait) * nx, cudaMemcpyHostToDevice));
    TQ_CUDA_TRY(cudaMemcpy(dp, e->xp_host.data(), sizeof(XPut) * nx, cudaMemcpyHostToDevice));
    e->xw_dev = (XWait *)dw;
    e->xp_dev = (XPut *)dp;
    e->p2p = true;
    // the step graphs are captured again on their next use, with the exchange
    for (cudaGraphExec_t *x : {&e->exec, &e->loop_exec})
        if (*x) cudaGraphExecDestroy(*x), *x = nullptr;
    for (cudaGraph_t *g : {&e->graph, &e->loop_graph})
        if (*g) cudaGraphDestroy(*g), *g = nullptr;
    return TQB200_OK;
}

int tqb200_engine_set_timeline(tqb200_engine *e, int max_steps) {
    TQ_CHECK_ARG(e && max_steps >= 0 && max_steps <= 1 << 16, "bad timeline arguments");
    TQ_CHECK_ARG(max_steps == 0 || e->o.use_graph, "the timeline needs the graph-replayed step");
    TQ_CUDA_TRY(cudaSetDevice(e->device));
    TQ_CUDA_TRY(cudaStreamSynchronize(e->stream));
    // the generate graph is captured again on its next use, with or without stamps
    if (e->loop_exec) cudaGraphExecDestroy(e->loop_exec);
    if (e->loop_graph) cudaGraphDestroy(e->loop_graph);
    e->loop_exec = nullptr;
    e->loop_graph = nullptr;
    if (e->tl) cudaFree(e->tl);
    e->tl = nullptr;
    e->tl_cap = e->tl_steps = 0;
    e->tl_kind.clear();
    if (max_steps == 0) return TQB200_OK;
    // room for every launch of a step (at most 8 per layer plus the head), kStampCtas
    // CTAs of three words each
    e->tl_stride = 3 * kStampCtas * (8 * e->d.n_layers + 16);
    const size_t bytes = (size_t)max_steps * e->tl_stride * 8;
    TQ_CUDA_TRY(cudaMalloc(&e->tl, bytes));
    TQ_CUDA_TRY(cudaMemset(e->tl, 0xFF, bytes));
    e->tl_cap = max_steps;
    return TQB200_OK;
}

int tqb200_engine_timeline_launches(const tqb200_engine *e, int step, int max_launches,
                                    int *kinds, double *us, int *n_launches) {
    TQ_CHECK_ARG(e && kinds && us && n_launches && max_launches > 0, "bad timeline arguments");
    TQ_CHECK_ARG(e->tl && step >= 0 && step < e->tl_steps, "no timeline record for step %d", step);
    const int nl = std::min((int)e->tl_kind.size(), max_launches);
    const int words = 3 * kStampCtas;
    std::vector<unsigned long long> h((size_t)e->tl_stride);
    TQ_CUDA_TRY(cudaSetDevice(e->device));
    TQ_CUDA_TRY(cudaStreamSynchronize(e->stream));
    TQ_CUDA_TRY(cudaMemcpy(h.data(), e->tl + (size_t)step * e->tl_stride, h.size() * 8,
                           cudaMemcpyDeviceToHost));
    const unsigned long long none = ~0ull;
    unsigned long long t0 = none;
    for (int i = 0; i < nl; ++i)
        for (int c = 0; c < kStampCtas; ++c)
            if (h[(size_t)i * words + 3 * c] != none) t0 = std::min(t0, h[(size_t)i * words + 3 * c]);
    for (int i = 0; i < nl; ++i) {
        unsigned long long v[6] = {none, 0, none, 0, none, 0};  // entry, wait, exit: min, max
        for (int c = 0; c < kStampCtas; ++c) {
            const unsigned long long *r = h.data() + (size_t)i * words + 3 * c;
            if (r[0] == none) continue;
            for (int j = 0; j < 3; ++j) {
                v[2 * j] = std::min(v[2 * j], r[j]);
                v[2 * j + 1] = std::max(v[2 * j + 1], r[j]);
            }
        }
        kinds[i] = e->tl_kind[i];
        for (int j = 0; j < 6; ++j)
            us[6 * i + j] = v[j] == none || t0 == none ? -1.0 : (double)(v[j] - t0) * 1e-3;
    }
    *n_launches = nl;
    return TQB200_OK;
}

int tqb200_engine_timeline(const tqb200_engine *e, int n_kinds, double *excl_ms, double *incl_ms,
                           int *launches, int *steps, double *span_ms) {
    TQ_CHECK_ARG(e && n_kinds > 0 && excl_ms && incl_ms && launches && steps && span_ms,
                 "bad timeline arguments");
    TQ_CHECK_ARG(e->tl, "no timeline set (tqb200_engine_set_timeline)");
    for (int k = 0; k < n_kinds; ++k) excl_ms[k] = incl_ms[k] = 0.0, launches[k] = 0;
    *steps = 0;
    *span_ms = 0.0;
    const int ns = e->tl_steps, nl = (int)e->tl_kind.size();
    if (ns == 0 || nl == 0) return TQB200_OK;
    std::vector<unsigned long long> h((size_t)ns * e->tl_stride);
    TQ_CUDA_TRY(cudaSetDevice(e->device));
    TQ_CUDA_TRY(cudaStreamSynchronize(e->stream));
    TQ_CUDA_TRY(cudaMemcpy(h.data(), e->tl, h.size() * 8, cudaMemcpyDeviceToHost));
    const unsigned long long none = ~0ull;
    const int words = 3 * kStampCtas;
    int good = 0;
    for (int s = 0; s < ns; ++s) {
        // per launch: first CTA in, first CTA past its wait, last CTA out
        std::vector<unsigned long long> entry(nl, none), wait(nl, none), exit(nl, 0);
        bool complete = true;
        for (int i = 0; i < nl; ++i) {
            const unsigned long long *r = h.data() + (size_t)s * e->tl_stride + (size_t)i * words;
            for (int c = 0; c < kStampCtas; ++c) {
                if (r[3 * c] == none) continue;
                entry[i] = std::min(entry[i], r[3 * c]);
                wait[i] = std::min(wait[i], r[3 * c + 1]);
                exit[i] = std::max(exit[i], r[3 * c + 2]);
            }
            complete = complete && entry[i] != none;
        }
        if (!complete) continue;  // a launch left no record (error path): skip the step
        // in-step time of launch i: its first wait to the next launch's first wait (the
        // last launch: to its last exit); time from launch: first entry to last exit
        unsigned long long first = none, last = 0;
        for (int i = 0; i < nl; ++i) {
            first = std::min(first, entry[i]);
            last = std::max(last, exit[i]);
            const int k = e->tl_kind[i];
            if (k < 0 || k >= n_kinds) continue;
            const unsigned long long end = i + 1 < nl ? wait[i + 1] : exit[i];
            excl_ms[k] += end > wait[i] ? (double)(end - wait[i]) * 1e-6 : 0.0;
            incl_ms[k] += exit[i] > entry[i] ? (double)(exit[i] - entry[i]) * 1e-6 : 0.0;
            if (good == 0) launches[k] += 1;
        }
        *span_ms += (double)(last - first) * 1e-6;
        ++good;
    }
    if (good > 0) {
        for (int k = 0; k < n_kinds; ++k) excl_ms[k] /= good, incl_ms[k] /= good;
        *span_ms /= good;
    }
    *steps = good;
    return TQB200_OK;
}

}  // extern "C"
