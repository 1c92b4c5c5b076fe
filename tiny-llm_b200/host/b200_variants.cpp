// b200_variants.cpp — binds libtqb200.so into the reference's own registries.
//
// Compiled together with the reference sources (kernels/dispatch.h, runtime/*) and
// linked with libtqb200.so, this file self-registers, under the name "b200":
//   * the per-op variants: i4 matvec / pair / qkv (kernels/dispatch.h:151-175),
//     VQ2 matvec (:187), BiIP rotate (:227) and the ops rmsnorm, rope, attention,
//     swiglu, argmax, top-k softmax (:298-307), selected by
//     --matvec-impl b200 / --ops-impl b200;
//   * the Qwen3.5 GDN ops (:389-396, with --ops-impl b200) and the GPTQ-INT4 matvec /
//     matmul (:211-258, --matvec-gptq-impl b200);
//   * the whole-step GPU decode engine (:353-378), selected by --engine b200;
// and defines create_b200_backend() (b200_backend.h): an IBackend
// (runtime/backend.h:73-392) whose every op runs on the GPU through libtqb200.so,
// fp16-KV attention (attention_decode_f16kv) included, for QwenModel::create's backend
// argument (main.cpp's --backend).
// Per-op calls use host pointers with resident weights: a weight is uploaded the
// first time its (mmap'd, immutable) host pointer is seen, as the reference's own
// resident CUDA variants do (kernels/matvec/matvec_f32_cuda_resident.cu).
// Errors abort with a message, the reference's convention
// (kernels/dispatch.cpp:393-398, kernels/cuda/gpu_engine.cu:38-45).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "b200_backend.h"
#include "dispatch.h"
#include "model_loader.h"
#include "ref_ops.h"
#include "tqb200.h"

namespace tinyqwen {
int g_matmul_calls = 0;  // calls that reached matmul_i4_b200 (read by drop_in_check)
}

namespace {

[[noreturn]] void die(const char *what) {
    std::fprintf(stderr, "tinyqwen b200 %s failed: %s\n", what, tqb200_last_error());
    std::abort();
}

struct ResidentOn {
    ResidentOn() { tqb200_set_resident_weights(1); }
} g_resident_on;

// ------------------------------------------------------------------ per-op variants
void matvec_i4_b200(const uint8_t *w, const float *x, float *y, int out, int in, int g) {
    if (tqb200_matvec_i4(w, x, y, out, in, g)) die("matvec_i4");
}
void matvec_pair_i4_b200(const uint8_t *w1, const uint8_t *w2, const float *x, float *y1,
                         float *y2, int out, int in, int g) {
    if (tqb200_matvec_pair_i4(w1, w2, x, y1, y2, out, in, g)) die("matvec_pair_i4");
}
void matvec_qkv_i4_b200(const uint8_t *wq, const uint8_t *wk, const uint8_t *wv, const float *x,
                        float *yq, float *yk, float *yv, int qd, int kvd, int in, int g) {
    if (tqb200_matvec_qkv_i4(wq, wk, wv, x, yq, yk, yv, qd, kvd, in, g)) die("matvec_qkv_i4");
}
// MatmulI4Fn (kernels/dispatch.h:248-249).  The reference has no by-name selector for
// it: the first registration becomes current (kernels/dispatch.cpp:651-660), so this one
// is current when this file is linked ahead of the reference's kernel objects.
void matmul_i4_b200(const uint8_t *w, const float *x, float *y, int M, int K, int N, int g) {
    ++tinyqwen::g_matmul_calls;
    if (tqb200_matmul_i4(w, x, y, M, K, N, g)) die("matmul_i4");
}
void matvec_vq2_b200(const uint8_t *w, const float *x, float *y, int out, int in) {
    if (tqb200_matvec_vq2(w, x, y, out, in)) die("matvec_vq2");
}
void biip_b200(const float *x, float *y, int dim, const float *scale, const float *sign, int bs) {
    if (tqb200_biip_rotate(x, y, dim, scale, sign, bs)) die("biip_rotate");
}
void rmsnorm_b200(const float *x, const float *w, float *y, int n, float eps) {
    if (tqb200_rmsnorm(x, w, y, n, eps)) die("rmsnorm");
}
void rope_b200(float *q, float *k, int nh, int nkv, int hd, int pos, float theta) {
    if (tqb200_rope(q, k, nh, nkv, hd, pos, theta)) die("rope");
}
void attention_b200(const float *q, const float *kc, const float *vc, int seq, int maxs, int nh,
                    int nkv, int hd, float scale, float *out) {
    if (tqb200_attention_decode(q, kc, vc, seq, maxs, nh, nkv, hd, scale, out)) die("attention");
}
void swiglu_b200(float *g, const float *u, int n) {
    if (tqb200_swiglu(g, u, n)) die("swiglu");
}
int argmax_b200(const float *l, int n) {
    int i = 0;
    if (tqb200_argmax(l, n, &i)) die("argmax");
    return i;
}
void topk_softmax_b200(const float *l, int n, int k, int *idx, float *w) {
    if (tqb200_topk_softmax(l, n, k, idx, w)) die("topk_softmax");
}

void matvec_gptq_b200(const uint8_t *w, const float *x, float *y, int out, int in, int g) {
    if (tqb200_matvec_gptq(w, x, y, out, in, g)) die("matvec_gptq");
}
void matmul_gptq_b200(const uint8_t *w, const float *x, float *y, int M, int K, int N, int g) {
    if (tqb200_matmul_gptq(w, x, y, M, K, N, g)) die("matmul_gptq");
}
void causal_conv1d_b200(const float *x, float *st, const float *w, float *out, int dim, int ks) {
    if (tqb200_causal_conv1d_update(x, st, w, out, dim, ks)) die("causal_conv1d_update");
}
void l2norm_b200(float *x, int n, float eps) {
    if (tqb200_l2norm_inplace(x, n, eps)) die("l2norm_inplace");
}
void gdn_step_b200(float *S, const float *q, const float *k, const float *v, float g, float beta,
                   float *o, int dk, int dv) {
    if (tqb200_gdn_step(S, q, k, v, g, beta, o, dk, dv)) die("gdn_step");
}
void rmsnorm_gated_b200(const float *x, const float *gate, const float *w, float *y, int n,
                        float eps) {
    if (tqb200_rmsnorm_gated(x, gate, w, y, n, eps)) die("rmsnorm_gated");
}

// ------------------------------------------------------------------ IBackend
// Every op on the GPU through the C ABI, weights resident by host pointer: the
// CUDABackend the reference leaves incomplete (runtime/backend_cuda.cpp:151-154 aborts on
// i4, :253-258 on partial_rope) and the fp16-KV attention its CPU backend lacks off
// aarch64 (runtime/backend_cpu.cpp:142-156).
class B200Backend final : public tinyqwen::IBackend {
    using WT = tinyqwen::WeightTensor;
    using QT = tinyqwen::QuantType;

  public:
    void matvec(const WT &w, const float *x, float *y, int out, int in) override {
        switch (w.quant_type) {
            case QT::kI4: matvec_i4_b200(u8(w), x, y, out, in, w.group_size); break;
            case QT::kVQ2: matvec_vq2_b200(u8(w), x, y, out, in); break;
            case QT::kGPTQ: matvec_gptq_b200(u8(w), x, y, out, in, w.group_size); break;
            case QT::kF16:
                if (tqb200_matvec_f16(static_cast<const uint16_t *>(w.data), x, y, out, in))
                    die("matvec_f16");
                break;
            default:
                if (tqb200_matvec_f32(static_cast<const float *>(w.data), x, y, out, in))
                    die("matvec_f32");
        }
    }
    void matvec_pair(const WT &w1, const WT &w2, const float *x, float *y1, float *y2, int out,
                     int in) override {
        if (w1.quant_type == QT::kI4 && w2.quant_type == QT::kI4 && w1.group_size == w2.group_size) {
            matvec_pair_i4_b200(u8(w1), u8(w2), x, y1, y2, out, in, w1.group_size);
            return;
        }
        matvec(w1, x, y1, out, in);
        matvec(w2, x, y2, out, in);
    }
    void matvec_qkv(const WT &wq, const WT &wk, const WT &wv, const float *x, float *yq, float *yk,
                    float *yv, int qd, int kvd, int in) override {
        if (wq.quant_type == QT::kI4 && wk.quant_type == QT::kI4 && wv.quant_type == QT::kI4 &&
            wq.group_size == wk.group_size && wk.group_size == wv.group_size) {
            matvec_qkv_i4_b200(u8(wq), u8(wk), u8(wv), x, yq, yk, yv, qd, kvd, in, wq.group_size);
            return;
        }
        matvec(wq, x, yq, qd, in);
        matvec(wk, x, yk, kvd, in);
        matvec(wv, x, yv, kvd, in);
    }
    void matmul(const WT &w, const float *x, float *y, int M, int K, int N) override {
        if (w.quant_type == QT::kI4) {
            if (tqb200_matmul_i4(u8(w), x, y, M, K, N, w.group_size)) die("matmul_i4");
        } else if (w.quant_type == QT::kGPTQ) {
            matmul_gptq_b200(u8(w), x, y, M, K, N, w.group_size);
        } else {  // one matvec per column (column-major X / Y), as CUDABackend::matmul
            for (int c = 0; c < N; ++c) matvec(w, x + (size_t)c * K, y + (size_t)c * M, M, K);
        }
    }
    void rmsnorm(const float *x, const float *w, float *y, int n, float eps) override {
        rmsnorm_b200(x, w, y, n, eps);
    }
    void rope(float *q, float *k, int nh, int nkv, int hd, int pos, float theta) override {
        rope_b200(q, k, nh, nkv, hd, pos, theta);
    }
    void partial_rope(float *q, float *k, int nh, int nkv, int hd, int rd, int pos,
                      float theta) override {
        if (tqb200_partial_rope(q, k, nh, nkv, hd, rd, pos, theta)) die("partial_rope");
    }
    void attention_decode(const float *q, const float *kc, const float *vc, int seq, int maxs,
                          int nh, int nkv, int hd, float scale, float *out) override {
        attention_b200(q, kc, vc, seq, maxs, nh, nkv, hd, scale, out);
    }
    void attention_decode_f16kv(const float *q, const uint16_t *kc, const uint16_t *vc, int seq,
                                int maxs, int nh, int nkv, int hd, float scale,
                                float *out) override {
        if (tqb200_attention_decode_f16kv(q, kc, vc, seq, maxs, nh, nkv, hd, scale, out))
            die("attention_decode_f16kv");
    }
    void swiglu(float *g, const float *u, int n) override { swiglu_b200(g, u, n); }
    int argmax(const float *l, int n) override { return argmax_b200(l, n); }
    // unused by the reference's decode (CPUBackend::top_k_logits writes nothing either,
    // runtime/backend_cpu.cpp:168-171)
    void top_k_logits(const float *, int, int, int *, float *) override {}
    void topk_softmax(const float *g, int n, int k, int *idx, float *w) override {
        topk_softmax_b200(g, n, k, idx, w);
    }
    void causal_conv1d_update(float *x, float *state, const float *w, float *out, int dim,
                              int ks) override {
        causal_conv1d_b200(x, state, w, out, dim, ks);
    }
    void l2norm_inplace(float *x, int n, float eps) override { l2norm_b200(x, n, eps); }
    void gdn_step(float *S, const float *q, const float *k, const float *v, float g, float beta,
                  float *o, int dk, int dv) override {
        gdn_step_b200(S, q, k, v, g, beta, o, dk, dv);
    }
    void rmsnorm_gated(float *x, const float *gate, const float *w, float *y, int n,
                       float eps) override {
        rmsnorm_gated_b200(x, gate, w, y, n, eps);
    }

  private:
    static const uint8_t *u8(const WT &w) { return static_cast<const uint8_t *>(w.data); }
};

// ------------------------------------------------------------------ engine
// The reference treats GpuDecodeEngine as opaque (kernels/dispatch.h:341-351); this
// holder is handed out behind that type.
struct Holder {
    tqb200_engine *e = nullptr;
    std::vector<tqb200_layer> layers;
    std::vector<std::vector<tqb200_matrix>> experts;
    std::vector<std::vector<float>> owned;  // fp16 norm vectors decoded to fp32
};

const float *vec_f32(Holder *h, const tinyqwen::TensorView *t) {
    if (!t) return nullptr;
    if (t->dtype == tinyqwen::Dtype::kF32) return reinterpret_cast<const float *>(t->data);
    std::vector<float> v(t->nbytes / 2);
    for (size_t i = 0; i < v.size(); ++i) {
        uint16_t hb;
        std::memcpy(&hb, t->data + 2 * i, 2);
        v[i] = tinyqwen::half_to_float(hb);
    }
    h->owned.push_back(std::move(v));
    return h->owned.back().data();
}

tqb200_matrix mat(const tinyqwen::TensorView *t) {
    tqb200_matrix m{};
    if (!t) return m;
    m.data = t->data;
    m.dtype = static_cast<int>(t->dtype);
    m.rows = static_cast<int>(t->shape[0]);
    m.cols = static_cast<int>(t->ndim > 1 ? t->shape[1] : 1);
    return m;
}

tqb200_rotation rot(Holder *h, const tinyqwen::ModelFile &f, const std::string &prefix) {
    tqb200_rotation r{};
    r.sign = vec_f32(h, f.get(prefix + ".rot_sign"));
    r.scale = vec_f32(h, f.get(prefix + ".rot_scale"));
    return r;  // block_size 0: derived from the input width (runtime/qwen_model.cpp:61-67)
}

// GpuDecodeCreateFn: a tqb200_model_desc from the ModelFile's tensor table, using the
// tensor names QwenModel::create binds (runtime/qwen_model.cpp:438-649).
bool create_b200(const void *model_file, int max_seq_len, std::string *err,
                 tinyqwen::GpuDecodeEngine **out) {
    const auto &f = *static_cast<const tinyqwen::ModelFile *>(model_file);
    const tinyqwen::ModelConfig &c = f.config();
    auto h = std::make_unique<Holder>();
    tqb200_model_desc d{};
    d.model_type = c.is_moe() ? TQB200_MODEL_QWEN3_MOE : TQB200_MODEL_QWEN2;
    d.n_layers = (int)c.n_layers;
    d.hidden = (int)c.hidden_size;
    d.inter = (int)c.intermediate_size;
    d.n_heads = (int)c.n_heads;
    d.n_kv_heads = (int)c.n_kv_heads;
    d.head_dim = (int)c.head_dim;
    d.vocab = (int)c.vocab_size;
    d.group_size = (int)c.quant_group_size;
    d.max_seq_len = (int)c.max_seq_len;
    d.rms_eps = c.rms_norm_eps;
    d.rope_theta = c.rope_theta;
    d.n_experts = (int)c.n_routed_experts;
    d.experts_per_tok = (int)c.num_experts_per_tok;
    d.moe_inter = (int)c.moe_intermediate_size;
    d.embed = mat(f.get("model.embed_tokens.weight"));
    const tinyqwen::TensorView *lm = f.get("lm_head.weight");
    d.lm_head = lm ? mat(lm) : d.embed;
    d.final_norm = vec_f32(h.get(), f.get("model.norm.weight"));
    h->layers.resize(c.n_layers);
    h->experts.resize(3 * (size_t)c.n_layers);
    for (uint32_t i = 0; i < c.n_layers; ++i) {
        const std::string p = "model.layers." + std::to_string(i) + ".";
        tqb200_layer &L = h->layers[i];
        L.input_ln = vec_f32(h.get(), f.get(p + "input_layernorm.weight"));
        L.post_ln = vec_f32(h.get(), f.get(p + "post_attention_layernorm.weight"));
        L.q_proj = mat(f.get(p + "self_attn.q_proj.weight"));
        L.k_proj = mat(f.get(p + "self_attn.k_proj.weight"));
        L.v_proj = mat(f.get(p + "self_attn.v_proj.weight"));
        L.o_proj = mat(f.get(p + "self_attn.o_proj.weight"));
        L.q_bias = vec_f32(h.get(), f.get(p + "self_attn.q_proj.bias"));
        L.k_bias = vec_f32(h.get(), f.get(p + "self_attn.k_proj.bias"));
        L.v_bias = vec_f32(h.get(), f.get(p + "self_attn.v_proj.bias"));
        L.q_norm = vec_f32(h.get(), f.get(p + "self_attn.q_norm.weight"));
        L.k_norm = vec_f32(h.get(), f.get(p + "self_attn.k_norm.weight"));
        L.gate_proj = mat(f.get(p + "mlp.gate_proj.weight"));
        L.up_proj = mat(f.get(p + "mlp.up_proj.weight"));
        L.down_proj = mat(f.get(p + "mlp.down_proj.weight"));
        L.rot_q = rot(h.get(), f, p + "self_attn.q_proj");
        L.rot_k = rot(h.get(), f, p + "self_attn.k_proj");
        L.rot_v = rot(h.get(), f, p + "self_attn.v_proj");
        L.rot_o = rot(h.get(), f, p + "self_attn.o_proj");
        L.rot_gate = rot(h.get(), f, p + "mlp.gate_proj");
        L.rot_up = rot(h.get(), f, p + "mlp.up_proj");
        L.rot_down = rot(h.get(), f, p + "mlp.down_proj");
        if (c.is_moe()) {
            L.router = mat(f.get(p + "mlp.gate.weight"));
            auto &eg = h->experts[3 * i], &eu = h->experts[3 * i + 1], &ed = h->experts[3 * i + 2];
            for (uint32_t e = 0; e < c.n_routed_experts; ++e) {
                const std::string pe = p + "mlp.experts." + std::to_string(e) + ".";
                eg.push_back(mat(f.get(pe + "gate_proj.weight")));
                eu.push_back(mat(f.get(pe + "up_proj.weight")));
                ed.push_back(mat(f.get(pe + "down_proj.weight")));
            }
            L.expert_gate = eg.data();
            L.expert_up = eu.data();
            L.expert_down = ed.data();
        }
    }
    d.layers = h->layers.data();
    tqb200_engine_opts o;
    tqb200_engine_default_opts(&o);
    o.max_seq_len = max_seq_len > 0 ? max_seq_len : (int)c.max_seq_len;
    if (tqb200_engine_create(&d, &o, &h->e) != TQB200_OK) {
        if (err) *err = std::string("tqb200_engine_create: ") + tqb200_last_error();
        return false;
    }
    *out = reinterpret_cast<tinyqwen::GpuDecodeEngine *>(h.release());
    return true;
}

int step_b200(tinyqwen::GpuDecodeEngine *e, int token) {
    int next = -1;
    if (tqb200_engine_step(reinterpret_cast<Holder *>(e)->e, token, &next)) die("engine_step");
    return next;
}
void reset_b200(tinyqwen::GpuDecodeEngine *e) {
    if (tqb200_engine_reset(reinterpret_cast<Holder *>(e)->e)) die("engine_reset");
}
void destroy_b200(tinyqwen::GpuDecodeEngine *e) {
    auto *h = reinterpret_cast<Holder *>(e);
    tqb200_engine_destroy(h->e);
    delete h;
}
const float *logits_b200(const tinyqwen::GpuDecodeEngine *e) {
    return tqb200_engine_logits(reinterpret_cast<const Holder *>(e)->e);
}

}  // namespace

TINYQWEN_MATVEC_I4_VARIANT(matvec_i4_b200, "b200");
TINYQWEN_MATVEC_I4_PAIR_VARIANT(matvec_pair_i4_b200, "b200");
TINYQWEN_MATVEC_QKV_I4_VARIANT(matvec_qkv_i4_b200, "b200");
TINYQWEN_MATVEC_VQ2_VARIANT(matvec_vq2_b200, "b200");
TINYQWEN_MATMUL_I4_VARIANT(matmul_i4_b200, "b200");
TINYQWEN_BIIP_ROTATE_VARIANT(biip_b200, "b200");
TINYQWEN_RMSNORM_VARIANT(rmsnorm_b200, "b200");
TINYQWEN_ROPE_VARIANT(rope_b200, "b200");
TINYQWEN_ATTENTION_DECODE_VARIANT(attention_b200, "b200");
TINYQWEN_SWIGLU_VARIANT(swiglu_b200, "b200");
TINYQWEN_ARGMAX_VARIANT(argmax_b200, "b200");
TINYQWEN_TOPK_SOFTMAX_VARIANT(topk_softmax_b200, "b200");
TINYQWEN_MATVEC_GPTQ_VARIANT(matvec_gptq_b200, "b200");
TINYQWEN_MATMUL_GPTQ_VARIANT(matmul_gptq_b200, "b200");
TINYQWEN_CAUSAL_CONV1D_UPDATE_VARIANT(causal_conv1d_b200, "b200");
TINYQWEN_L2NORM_INPLACE_VARIANT(l2norm_b200, "b200");
TINYQWEN_GDN_STEP_VARIANT(gdn_step_b200, "b200");
TINYQWEN_RMSNORM_GATED_VARIANT(rmsnorm_gated_b200, "b200");
TINYQWEN_GPU_DECODE_VARIANT("b200", create_b200, step_b200, reset_b200, destroy_b200, logits_b200);

std::unique_ptr<tinyqwen::IBackend> create_b200_backend() {
    return std::make_unique<B200Backend>();
}
