/*
 * tq_oracle.h — CPU restatement of the tinyqwen quantised decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker the CUDA path is compared
 * against; it is never linked into, loaded by, or called from the product
 * library (libtqb200.so).  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference legs may load it.
 *
 * Every function restates one reference function (file:line given at each
 * definition in tq_oracle.c) with the same rounding points: same float/double
 * promotions, same accumulation order within a row, no FMA contraction
 * (built with -ffp-contract=off).  Row loops are parallel (OpenMP) because
 * rows are independent; each row's arithmetic is unchanged, so results do not
 * depend on the thread count.
 */
#ifndef TQ_ORACLE_H
#define TQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "../include/tqb200_model.h"

#ifdef __cplusplus
extern "C" {
#endif

float tqo_half_to_float(uint16_t h);
uint16_t tqo_float_to_half(float f);
void tqo_set_threads(int n);

void tqo_matvec_i4(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                   int group_size);
void tqo_matvec_i4_w4a8(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                        int group_size);
void tqo_matmul_i4(const uint8_t *w, const float *x, float *y, int M, int K, int N,
                   int group_size);
void tqo_dequant_i4(const uint8_t *w, int rows, int dim, int group_size, float *out);
void tqo_matvec_vq2(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim);
void tqo_matvec_f32(const float *w, const float *x, float *y, int out_dim, int in_dim);
void tqo_matvec_f16(const uint16_t *w, const float *x, float *y, int out_dim, int in_dim);
void tqo_biip_rotate(const float *x, float *y, int dim, const float *scale, const float *sign,
                     int block_size);
int tqo_hadamard_block_size(int dim);
void tqo_rmsnorm(const float *x, const float *weight, float *y, int n, float eps);
void tqo_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim, int pos,
              float theta);
void tqo_attention_decode(const float *q, const float *k_cache, const float *v_cache, int seq_len,
                          int max_seq_len, int n_heads, int n_kv_heads, int head_dim, float scale,
                          float *out);
void tqo_attention_decode_f16kv(const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                                int seq_len, int max_seq_len, int n_heads, int n_kv_heads,
                                int head_dim, float scale, float *out);
void tqo_swiglu(float *gate, const float *up, int n);
int tqo_argmax(const float *logits, int n);
void tqo_topk_softmax(const float *gate_logits, int n, int k, int *indices, float *weights);

void tqo_matvec_gptq(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                     int group_size);
void tqo_matmul_gptq(const uint8_t *w, const float *x, float *y, int M, int K, int N,
                     int group_size);
void tqo_l2norm_inplace(float *x, int n, float eps);
void tqo_causal_conv1d_update(const float *x, float *state, const float *weight, float *out,
                              int dim, int kernel_size);
void tqo_gdn_step(float *S, const float *q, const float *k, const float *v, float g, float beta,
                  float *o, int qk_dim, int v_dim);
void tqo_rmsnorm_gated(const float *x, const float *gate, const float *weight, float *y, int n,
                       float eps);
void tqo_partial_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim,
                      int rotary_dim, int pos, float theta);

/* Whole-model greedy decode (runtime/qwen_forward_token.cpp:83-742). */
typedef struct tqo_model tqo_model;
tqo_model *tqo_model_create(const tqb200_model_desc *desc, int max_seq_len, int kv_fp16);
int tqo_model_step(tqo_model *m, int token_id);           /* returns argmax id, -1 on error */
const float *tqo_model_logits(const tqo_model *m);        /* [vocab] of the last step */
const float *tqo_model_hidden(const tqo_model *m);        /* residual stream after last step */
void tqo_model_reset(tqo_model *m);
void *tqo_model_kv(tqo_model *m, size_t *bytes);          /* KV arena, engine layout */
int tqo_model_set_position(tqo_model *m, int pos);        /* 0, or -1 out of range */
/* fp16 cache guide for comparisons (see tq_oracle.c); NULL = off. */
void tqo_model_set_kv_guide(tqo_model *m, const uint16_t *guide, float tol);
void tqo_model_kv_guide_counts(const tqo_model *m, long long *flips, long long *mismatches,
                               double *max_dev);
void tqo_model_destroy(tqo_model *m);
/* Runs only layers [0, n_layers_run) and skips the head when head == 0: a bounded
 * sample of one step, used by the timed CPU baseline. */
void tqo_model_set_partial(tqo_model *m, int n_layers_run, int head);

#ifdef __cplusplus
}
#endif
#endif
