// ref_harness.cpp — extern "C" wrappers around the reference's own CPU code,
// compiled together with the reference sources (oracle/Makefile) into
// oracle/_ref/libtqref.so.
//
// TEST INFRASTRUCTURE ONLY.  The compiled reference pins the C restatement
// (oracle/tq_oracle.c) and serves as the timed CPU baseline; nothing in the
// product library links or loads it.
//
// Only reference entry points are called (matvec_i4_ref, matvec_vq2_ref,
// biip_rotate_activation_ref, the ops *_ref, the dispatch entries, ModelFile
// and QwenModel::forward_token); nothing from the reference is modified.
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "backend_cpu.h"
#include "dispatch.h"
#include "gdn_ops.h"
#include "model_loader.h"
#include "profiler.h"
#include "qwen_model.h"
#include "ref_ops.h"

namespace tinyqwen {
// Defined with external linkage in kernels/matvec/matvec_i4_ref.cpp:45 and
// kernels/matvec/matvec_vq2_ref.cpp:52; the reference declares them only for
// registration, so they are declared here.
void matvec_i4_ref(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                   int group_size);
void matvec_vq2_ref(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim);
// kernels/matvec/matvec_gptq_ref.cpp, likewise registration-only
void matvec_gptq_ref(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                     int group_size);
}  // namespace tinyqwen

namespace {

using tinyqwen::IBackend;
using tinyqwen::WeightTensor;

// CPUBackend::attention_decode_f16kv aborts off aarch64 (runtime/backend_cpu.cpp:142-156).
// The reference's own x86 check of that path decodes the stored halves and
// runs attention_decode_ref (tests/test_attention.cpp:192-226); this backend
// does the same and forwards every other op to the stock CPU backend.
class F16KvCheckBackend : public IBackend {
  public:
    F16KvCheckBackend() : inner_(tinyqwen::create_cpu_backend()) {}
    void matvec(const WeightTensor &w, const float *x, float *y, int o, int i) override {
        inner_->matvec(w, x, y, o, i);
    }
    void matvec_pair(const WeightTensor &w1, const WeightTensor &w2, const float *x, float *y1,
                     float *y2, int o, int i) override {
        inner_->matvec_pair(w1, w2, x, y1, y2, o, i);
    }
    void matvec_qkv(const WeightTensor &wq, const WeightTensor &wk, const WeightTensor &wv,
                    const float *x, float *yq, float *yk, float *yv, int qd, int kvd,
                    int in) override {
        inner_->matvec_qkv(wq, wk, wv, x, yq, yk, yv, qd, kvd, in);
    }
    void matmul(const WeightTensor &w, const float *x, float *y, int M, int K, int N) override {
        inner_->matmul(w, x, y, M, K, N);
    }
    void rmsnorm(const float *x, const float *w, float *y, int n, float eps) override {
        inner_->rmsnorm(x, w, y, n, eps);
    }
    void rope(float *q, float *k, int nh, int nkv, int hd, int pos, float theta) override {
        inner_->rope(q, k, nh, nkv, hd, pos, theta);
    }
    void partial_rope(float *q, float *k, int nh, int nkv, int hd, int rd, int pos,
                      float theta) override {
        inner_->partial_rope(q, k, nh, nkv, hd, rd, pos, theta);
    }
    void attention_decode(const float *q, const float *kc, const float *vc, int seq, int maxs,
                          int nh, int nkv, int hd, float scale, float *out) override {
        inner_->attention_decode(q, kc, vc, seq, maxs, nh, nkv, hd, scale, out);
    }
    void attention_decode_f16kv(const float *q, const uint16_t *kc, const uint16_t *vc, int seq,
                                int maxs, int nh, int nkv, int hd, float scale,
                                float *out) override {
        const size_t n = static_cast<size_t>(nkv) * maxs * hd;
        kf_.resize(n);
        vf_.resize(n);
        for (size_t i = 0; i < n; ++i) {
            kf_[i] = tinyqwen::half_to_float(kc[i]);
            vf_[i] = tinyqwen::half_to_float(vc[i]);
        }
        tinyqwen::attention_decode_ref(q, kf_.data(), vf_.data(), seq, maxs, nh, nkv, hd, scale,
                                       out);
    }
    void swiglu(float *g, const float *u, int n) override { inner_->swiglu(g, u, n); }
    int argmax(const float *l, int n) override { return inner_->argmax(l, n); }
    void top_k_logits(const float *l, int n, int k, int *idx, float *vals) override {
        inner_->top_k_logits(l, n, k, idx, vals);
    }
    void topk_softmax(const float *g, int n, int k, int *idx, float *w) override {
        inner_->topk_softmax(g, n, k, idx, w);
    }
    void causal_conv1d_update(float *x, float *state, const float *weight, float *out, int dim,
                              int kernel) override {
        inner_->causal_conv1d_update(x, state, weight, out, dim, kernel);
    }
    void l2norm_inplace(float *x, int n, float eps) override { inner_->l2norm_inplace(x, n, eps); }
    void gdn_step(float *S, const float *q, const float *k, const float *v, float g, float beta,
                  float *out, int dk, int dv) override {
        inner_->gdn_step(S, q, k, v, g, beta, out, dk, dv);
    }
    void rmsnorm_gated(float *x, const float *gate, const float *weight, float *out, int n,
                       float eps) override {
        inner_->rmsnorm_gated(x, gate, weight, out, n, eps);
    }

  private:
    std::unique_ptr<IBackend> inner_;
    std::vector<float> kf_, vf_;
};

struct RefModel {
    tinyqwen::ModelFile file;
    tinyqwen::Profiler profiler{false};
    std::unique_ptr<tinyqwen::QwenModel> model;
};

}  // namespace

extern "C" {

void tqref_matvec_i4(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                     int group_size) {
    tinyqwen::matvec_i4_ref(w, x, y, out_dim, in_dim, group_size);
}

void tqref_matmul_i4(const uint8_t *w, const float *x, float *y, int M, int K, int N,
                     int group_size) {
    tinyqwen::set_matvec_i4_impl_by_name("ref");
    tinyqwen::matmul_i4(w, x, y, M, K, N, group_size);
}

void tqref_dequant_i4_row(const uint8_t *w, int row, int dim, int group_size, float *out) {
    tinyqwen::dequant_i4_row(w, row, dim, group_size, out);
}

void tqref_matvec_vq2(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim) {
    tinyqwen::matvec_vq2_ref(w, x, y, out_dim, in_dim);
}

void tqref_matvec_f32(const float *w, const float *x, float *y, int out_dim, int in_dim) {
    tinyqwen::matvec_f32_ref(w, x, y, out_dim, in_dim);
}

void tqref_biip_rotate(const float *x, float *y, int dim, const float *scale, const float *sign,
                       int block_size) {
    tinyqwen::biip_rotate_activation_ref(x, y, dim, scale, sign, block_size);
}

void tqref_rmsnorm(const float *x, const float *w, float *y, int n, float eps) {
    tinyqwen::rmsnorm_ref(x, w, y, n, eps);
}

void tqref_rope(float *q, float *k, int nh, int nkv, int hd, int pos, float theta) {
    tinyqwen::rope_ref(q, k, nh, nkv, hd, pos, theta);
}

void tqref_attention_decode(const float *q, const float *kc, const float *vc, int seq, int maxs,
                            int nh, int nkv, int hd, float scale, float *out) {
    tinyqwen::attention_decode_ref(q, kc, vc, seq, maxs, nh, nkv, hd, scale, out);
}

void tqref_swiglu(float *g, const float *u, int n) { tinyqwen::swiglu_ref(g, u, n); }

int tqref_argmax(const float *l, int n) { return tinyqwen::argmax_ref(l, n); }

void tqref_topk_softmax(const float *g, int n, int k, int *idx, float *w) {
    tinyqwen::topk_softmax_ref(g, n, k, idx, w);
}

void tqref_matvec_gptq(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                       int group_size) {
    tinyqwen::matvec_gptq_ref(w, x, y, out_dim, in_dim, group_size);
}

void tqref_l2norm_inplace(float *x, int n, float eps) { tinyqwen::l2norm_inplace_ref(x, n, eps); }

void tqref_causal_conv1d_update(const float *x, float *state, const float *w, float *out, int dim,
                                int kernel_size) {
    tinyqwen::causal_conv1d_update_ref(x, state, w, out, dim, kernel_size);
}

void tqref_gdn_step(float *S, const float *q, const float *k, const float *v, float g, float beta,
                    float *o, int qk_dim, int v_dim) {
    tinyqwen::gdn_step_ref(S, q, k, v, g, beta, o, qk_dim, v_dim);
}

void tqref_rmsnorm_gated(const float *x, const float *gate, const float *w, float *y, int n,
                         float eps) {
    tinyqwen::rmsnorm_gated_ref(x, gate, w, y, n, eps);
}

void tqref_partial_rope(float *q, float *k, int nh, int nkv, int hd, int rd, int pos, float theta) {
    tinyqwen::partial_rope_ref(q, k, nh, nkv, hd, rd, pos, theta);
}

uint16_t tqref_float_to_half(float f) { return tinyqwen::float_to_half(f); }
float tqref_half_to_float(uint16_t h) { return tinyqwen::half_to_float(h); }

// Whole-model decode through the reference's loader and QwenModel::forward_token.
void *tqref_model_open(const char *path, int max_seq_len, int kv_fp16, char *err, int err_len) {
    auto *rm = new RefModel();
    std::string e;
    if (!rm->file.load(path, &e)) {
        std::snprintf(err, static_cast<size_t>(err_len), "%s", e.c_str());
        delete rm;
        return nullptr;
    }
    std::unique_ptr<IBackend> be;
    if (kv_fp16) be.reset(new F16KvCheckBackend());
    if (!tinyqwen::QwenModel::create(rm->file, max_seq_len, rm->profiler, &e, &rm->model,
                                     std::move(be), kv_fp16 != 0)) {
        std::snprintf(err, static_cast<size_t>(err_len), "%s", e.c_str());
        delete rm;
        return nullptr;
    }
    return rm;
}

int tqref_model_step(void *h, int token) {
    return static_cast<RefModel *>(h)->model->forward_token(token, nullptr, 5, true);
}

const float *tqref_model_logits(void *h) {
    return static_cast<RefModel *>(h)->model->last_logits();
}

void tqref_model_reset(void *h) { static_cast<RefModel *>(h)->model->reset(); }

void tqref_model_close(void *h) { delete static_cast<RefModel *>(h); }

}  // extern "C"
