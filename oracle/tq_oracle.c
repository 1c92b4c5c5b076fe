/*
 * tq_oracle.c — CPU restatement of the tinyqwen quantised decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see tq_oracle.h): the checker for the CUDA path,
 * never part of the product library.
 *
 * Each function names the reference function it restates, as
 * path:line inside the 918822019/tiny-llm source tree.  Rounding points are
 * kept: fp16 fields decode exactly, dequant is (float(q) - zero) * scale in
 * fp32, dot products accumulate in double in row order, and the file is built
 * with -ffp-contract=off so no multiply-add is fused unless the reference
 * fuses it.  Row loops run in parallel; a row's arithmetic never depends on
 * the thread count.
 */
#include "tq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32 (kernels/ref_ops.h:51-105)                                  */
/* ------------------------------------------------------------------------ */

/* Exact binary16 -> binary32 decode.  Same values as half_to_float
 * (kernels/ref_ops.h:51-74); subnormals are scaled by 2^-24 instead of being
 * renormalised bit by bit, which yields the identical float. */
float tqo_half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu;
    const uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            const float f = (float)m * 5.9604644775390625e-8f; /* m * 2^-24, exact */
            return sign ? -f : f;
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* binary32 -> binary16, round to nearest even, with the reference's two
 * deliberate choices (kernels/ref_ops.h:78-105): every NaN becomes the quiet
 * NaN 0x7E00 (with sign), and magnitudes below 2^-24 flush to signed zero. */
uint16_t tqo_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, sizeof x);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t a = x & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return (uint16_t)(sign | 0x7E00u);
    if (a >= 0x47800000u) return (uint16_t)(sign | 0x7C00u);
    if (a >= 0x38800000u) {
        /* normal half: rebias exponent, round the 13 dropped mantissa bits */
        uint32_t base = (a >> 13) - (112u << 10);
        const uint32_t rem = a & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (base & 1u))) base += 1u;
        return (uint16_t)(sign | base);
    }
    if (a < 0x33800000u) return sign;
    {
        const int e = (int)(a >> 23) - 127;             /* -24 .. -15 */
        const uint32_t mant = (a & 0x7FFFFFu) | 0x800000u;
        const int sh = -1 - e;                           /* 14 .. 23 */
        uint32_t q = mant >> sh;
        const uint32_t rem = mant & ((1u << sh) - 1u);
        const uint32_t halfway = 1u << (sh - 1);
        if (rem > halfway || (rem == halfway && (q & 1u))) q += 1u;
        return (uint16_t)(sign | q);
    }
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

void tqo_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------------ */
/* matvecs                                                                   */
/* ------------------------------------------------------------------------ */

/* One i4 row dot x (kernels/matvec/matvec_i4_ref.cpp:57-101). */
static float i4_row_dot(const uint8_t *row, const float *x, int in_dim, int group_size) {
    const int gpr = (in_dim + group_size - 1) / group_size;
    const int gbytes = 4 + group_size / 2;
    double acc = 0.0;
    int col = 0;
    for (int g = 0; g < gpr; ++g) {
        const uint8_t *gp = row + (size_t)g * gbytes;
        const float scale = tqo_half_to_float(rd16(gp));
        const float zero = tqo_half_to_float(rd16(gp + 2));
        const uint8_t *pk = gp + 4;
        const int elems = (col + group_size <= in_dim) ? group_size : (in_dim - col);
        for (int i = 0; i < elems; ++i) {
            const uint8_t v = (i & 1) ? (uint8_t)((pk[i >> 1] >> 4) & 0x0F)
                                      : (uint8_t)(pk[i >> 1] & 0x0F);
            const float dq = ((float)v - zero) * scale;
            acc += (double)dq * (double)x[col + i];
        }
        col += group_size;
    }
    return (float)acc;
}

/* matvec_i4_ref (kernels/matvec/matvec_i4_ref.cpp:45-103). */
void tqo_matvec_i4(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                   int group_size) {
    const size_t rb = tqb200_i4_row_bytes(in_dim, group_size);
#pragma omp parallel for schedule(static)
    for (int o = 0; o < out_dim; ++o) y[o] = i4_row_dot(w + (size_t)o * rb, x, in_dim, group_size);
}

/* W4A8 semantics of the symmetric "sdot5" family, restated from the reference's
 * own naive checker matvec_i4_w4a8_naive (tests/test_matvec_i4.cpp:252-306):
 * x -> int8 with scale amax/127 (round half away from zero, clamp +-127), per
 * group an exact integer dot of (q-8)*xq, fp32 accumulation of
 * A*dot - C*xqsum with A = scale_w*scale_x, C = A*(zero-8).  For symmetric
 * weights (zero == 8) C == 0 and this is matvec_i4_sdot5
 * (kernels/matvec/matvec_i4_sdot5.cpp:113-180, 276). */
void tqo_matvec_i4_w4a8(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                        int group_size) {
    float amax = 0.0f;
    for (int i = 0; i < in_dim; ++i) {
        const float a = x[i] < 0 ? -x[i] : x[i];
        if (a > amax) amax = a;
    }
    const float scale_x = amax > 0.0f ? amax / 127.0f : 1.0f;
    const float inv = 1.0f / scale_x;
    int *xq = (int *)malloc(sizeof(int) * (size_t)(in_dim > 0 ? in_dim : 1));
    int *prefix = (int *)malloc(sizeof(int) * (size_t)(in_dim + 1));
    prefix[0] = 0;
    for (int i = 0; i < in_dim; ++i) {
        float v = x[i] * inv;
        v = v > 127.0f ? 127.0f : (v < -127.0f ? -127.0f : v);
        const int q = (int)(v >= 0 ? v + 0.5f : v - 0.5f);
        xq[i] = q;
        prefix[i + 1] = prefix[i] + q;
    }
    const int gpr = (in_dim + group_size - 1) / group_size;
    const int gbytes = 4 + group_size / 2;
    const size_t rb = (size_t)gpr * gbytes;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < out_dim; ++o) {
        const uint8_t *row = w + (size_t)o * rb;
        float acc = 0.0f;
        int col = 0;
        for (int g = 0; g < gpr; ++g) {
            const uint8_t *gp = row + (size_t)g * gbytes;
            const float scale_w = tqo_half_to_float(rd16(gp));
            const float zero_w = tqo_half_to_float(rd16(gp + 2));
            const float A = scale_w * scale_x;
            const float C = A * (zero_w - 8.0f);
            const uint8_t *pk = gp + 4;
            const int elems = (col + group_size <= in_dim) ? group_size : (in_dim - col);
            int dot = 0;
            for (int i = 0; i < elems; ++i) {
                const int q = (i & 1) ? ((pk[i >> 1] >> 4) & 0x0F) : (pk[i >> 1] & 0x0F);
                dot += (q - 8) * xq[col + i];
            }
            const int xqsum = prefix[col + elems] - prefix[col];
            const float t1 = A * (float)dot;
            const float t2 = C * (float)xqsum;
            acc += t1 - t2;
            col += group_size;
        }
        y[o] = acc;
    }
    free(xq);
    free(prefix);
}

/* matmul_i4_ref (kernels/matvec/matmul_i4_ref.cpp:53-114): X, Y column-major,
 * each column is one matvec_i4_ref. */
void tqo_matmul_i4(const uint8_t *w, const float *x, float *y, int M, int K, int N,
                   int group_size) {
    const size_t rb = tqb200_i4_row_bytes(K, group_size);
    const long total = (long)M * N;
#pragma omp parallel for schedule(static)
    for (long t = 0; t < total; ++t) {
        const int col = (int)(t / M), row = (int)(t % M);
        y[(size_t)col * M + row] = i4_row_dot(w + (size_t)row * rb, x + (size_t)col * K, K, group_size);
    }
}

/* dequant_i4_row (kernels/ref_ops.h:183-205) applied to `rows` rows. */
void tqo_dequant_i4(const uint8_t *w, int rows, int dim, int group_size, float *out) {
    const int gpr = (dim + group_size - 1) / group_size;
    const int gbytes = 4 + group_size / 2;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const uint8_t *row = w + (size_t)r * gpr * gbytes;
        float *o = out + (size_t)r * dim;
        int col = 0;
        for (int g = 0; g < gpr; ++g) {
            const uint8_t *gp = row + (size_t)g * gbytes;
            const float scale = tqo_half_to_float(rd16(gp));
            const float zero = tqo_half_to_float(rd16(gp + 2));
            const int elems = (col + group_size <= dim) ? group_size : (dim - col);
            for (int i = 0; i < elems; ++i) {
                const uint8_t v = (i & 1) ? (uint8_t)((gp[4 + (i >> 1)] >> 4) & 0x0F)
                                          : (uint8_t)(gp[4 + (i >> 1)] & 0x0F);
                o[col + i] = ((float)v - zero) * scale;
            }
            col += group_size;
        }
    }
}

/* matvec_vq2_ref (kernels/matvec/matvec_vq2_ref.cpp:52-82): codebook
 * [256][4] fp16 in-band, then one uint8 index per 4 weights, row-major. */
void tqo_matvec_vq2(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim) {
    float cb[256][4];
    for (int k = 0; k < 256; ++k)
        for (int j = 0; j < 4; ++j) cb[k][j] = tqo_half_to_float(rd16(w + (k * 4 + j) * 2));
    const int nb = in_dim / 4;
    const uint8_t *idx = w + 2048;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < out_dim; ++o) {
        const uint8_t *row = idx + (size_t)o * nb;
        double acc = 0.0;
        for (int b = 0; b < nb; ++b) {
            const float *cv = cb[row[b]];
            for (int j = 0; j < 4; ++j) acc += (double)cv[j] * (double)x[b * 4 + j];
        }
        y[o] = (float)acc;
    }
}

/* matvec_f32_ref (kernels/matvec/matvec_f32_ref.cpp:41-58). */
void tqo_matvec_f32(const float *w, const float *x, float *y, int out_dim, int in_dim) {
#pragma omp parallel for schedule(static)
    for (int o = 0; o < out_dim; ++o) {
        const float *row = w + (size_t)o * in_dim;
        double acc = 0.0;
        for (int i = 0; i < in_dim; ++i) acc += (double)row[i] * x[i];
        y[o] = (float)acc;
    }
}

/* matvec_f16_ref (kernels/matvec/matvec_f16_ref.cpp:33-50). */
void tqo_matvec_f16(const uint16_t *w, const float *x, float *y, int out_dim, int in_dim) {
#pragma omp parallel for schedule(static)
    for (int o = 0; o < out_dim; ++o) {
        const uint16_t *row = w + (size_t)o * in_dim;
        double acc = 0.0;
        for (int i = 0; i < in_dim; ++i) acc += (double)tqo_half_to_float(row[i]) * x[i];
        y[o] = (float)acc;
    }
}

/* ------------------------------------------------------------------------ */
/* BiIP (kernels/biip/biip_rotate.cpp:36-69; block size runtime/qwen_model.cpp:61-67) */
/* ------------------------------------------------------------------------ */

int tqo_hadamard_block_size(int dim) {
    static const int cand[] = {256, 128, 64, 32, 16, 8, 4, 2};
    for (int i = 0; i < 8; ++i)
        if (dim % cand[i] == 0) return cand[i];
    return 1;
}

void tqo_biip_rotate(const float *x, float *y, int dim, const float *scale, const float *sign,
                     int block_size) {
    if (scale) {
        for (int j = 0; j < dim; ++j) y[j] = (x[j] / scale[j]) * sign[j];
    } else {
        for (int j = 0; j < dim; ++j) y[j] = x[j] * sign[j];
    }
    const int nblk = dim / block_size;
    const float inv_sqrt = 1.0f / sqrtf((float)block_size);
    for (int b = 0; b < nblk; ++b) {
        float *blk = y + (size_t)b * block_size;
        for (int h = 1; h < block_size; h <<= 1)
            for (int i = 0; i < block_size; i += 2 * h)
                for (int j = i; j < i + h; ++j) {
                    const float a = blk[j], c = blk[j + h];
                    blk[j] = a + c;
                    blk[j + h] = a - c;
                }
        for (int j = 0; j < block_size; ++j) blk[j] *= inv_sqrt;
    }
}

/* ------------------------------------------------------------------------ */
/* decode ops                                                                */
/* ------------------------------------------------------------------------ */

/* rmsnorm_ref (kernels/rmsnorm/rmsnorm_ref.cpp:48-78). */
void tqo_rmsnorm(const float *x, const float *weight, float *y, int n, float eps) {
    double sumsq = 0.0;
    for (int i = 0; i < n; ++i) {
        const double xi = (double)x[i];
        sumsq += xi * xi;
    }
    const float mean_sq = (float)(sumsq / n);
    const float rms = sqrtf(mean_sq + eps);
    const float scale = 1.0f / rms;
    for (int i = 0; i < n; ++i) {
        const float normed = x[i] * scale;
        y[i] = normed * weight[i];
    }
}

/* rope_ref (kernels/rope/rope_ref.cpp:56-117): rotate-half pairs (i, i+hd/2). */
void tqo_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim, int pos,
              float theta) {
    const int half = head_dim / 2;
    if (half <= 0 || half > 256) return;
    float cs[256], sn[256];
    for (int i = 0; i < half; ++i) {
        const float exponent = -(float)(2 * i) / (float)head_dim;
        const float inv_freq = powf(theta, exponent);
        const float angle = (float)pos * inv_freq;
        cs[i] = cosf(angle);
        sn[i] = sinf(angle);
    }
    for (int h = 0; h < n_heads + n_kv_heads; ++h) {
        float *v = (h < n_heads) ? q + (size_t)h * head_dim : k + (size_t)(h - n_heads) * head_dim;
        for (int i = 0; i < half; ++i) {
            const float x0 = v[i], x1 = v[i + half];
            const float a = x0 * cs[i], b = x1 * sn[i];
            const float c = x1 * cs[i], d = x0 * sn[i];
            v[i] = a - b;
            v[i + half] = c + d;
        }
    }
}

/* attention_decode_ref (kernels/attention/attention_decode_ref.cpp:53-143):
 * one pass of online softmax per query head, double q.k, fp32 rescaling. */
static void attention_core(const float *q, const void *kc, const void *vc, int f16, int seq_len,
                           int max_seq_len, int n_heads, int n_kv_heads, int head_dim, float scale,
                           float *out) {
    const int hpk = n_heads / n_kv_heads;
    const size_t stride = (size_t)max_seq_len * head_dim;
#pragma omp parallel for schedule(static)
    for (int h = 0; h < n_heads; ++h) {
        const int kv = h / hpk;
        const float *qh = q + (size_t)h * head_dim;
        float *oh = out + (size_t)h * head_dim;
        float *kt = (float *)malloc(sizeof(float) * (size_t)head_dim * 2);
        float *vt = kt + head_dim;
        float m = -INFINITY, l = 0.0f;
        for (int i = 0; i < head_dim; ++i) oh[i] = 0.0f;
        for (int t = 0; t < seq_len; ++t) {
            const size_t off = (size_t)kv * stride + (size_t)t * head_dim;
            if (f16) {
                for (int i = 0; i < head_dim; ++i) {
                    kt[i] = tqo_half_to_float(((const uint16_t *)kc)[off + i]);
                    vt[i] = tqo_half_to_float(((const uint16_t *)vc)[off + i]);
                }
            } else {
                memcpy(kt, (const float *)kc + off, sizeof(float) * (size_t)head_dim);
                memcpy(vt, (const float *)vc + off, sizeof(float) * (size_t)head_dim);
            }
            double dot = 0.0;
            for (int i = 0; i < head_dim; ++i) dot += (double)qh[i] * kt[i];
            const float s = (float)dot * scale;
            const float m_new = s > m ? s : m;
            const float rescale = expf(m - m_new);
            const float p = expf(s - m_new);
            for (int i = 0; i < head_dim; ++i) {
                const float ro = oh[i] * rescale;
                const float c = p * vt[i];
                oh[i] = ro + c;
            }
            const float rl = l * rescale;
            l = rl + p;
            m = m_new;
        }
        const float inv_l = 1.0f / l;
        for (int i = 0; i < head_dim; ++i) oh[i] = oh[i] * inv_l;
        free(kt);
    }
}

void tqo_attention_decode(const float *q, const float *k_cache, const float *v_cache, int seq_len,
                          int max_seq_len, int n_heads, int n_kv_heads, int head_dim, float scale,
                          float *out) {
    attention_core(q, k_cache, v_cache, 0, seq_len, max_seq_len, n_heads, n_kv_heads, head_dim,
                   scale, out);
}

/* fp16-KV attention: the reference's x86 check of the fp16 path is "decode the
 * stored halves, then attention_decode_ref" (tests/test_attention.cpp:192-226). */
void tqo_attention_decode_f16kv(const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                                int seq_len, int max_seq_len, int n_heads, int n_kv_heads,
                                int head_dim, float scale, float *out) {
    attention_core(q, k_cache, v_cache, 1, seq_len, max_seq_len, n_heads, n_kv_heads, head_dim,
                   scale, out);
}

/* swiglu_ref (kernels/silu/swiglu_ref.cpp:41-52). */
void tqo_swiglu(float *gate, const float *up, int n) {
    for (int i = 0; i < n; ++i) {
        const float denom = 1.0f + expf(-gate[i]);
        const float s = gate[i] / denom;
        gate[i] = s * up[i];
    }
}

/* argmax_ref (kernels/argmax/argmax_ref.cpp:42-54): first index of the max. */
int tqo_argmax(const float *logits, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (logits[i] > logits[best]) best = i;
    return best;
}

/* topk_softmax_ref (kernels/topk_softmax/topk_softmax_ref.cpp:41-78): top-k by
 * logit (ties: lower index first), softmax over those k in double, weights
 * rounded to float; slots beyond n get index -1 and weight 0. */
void tqo_topk_softmax(const float *gate_logits, int n, int k, int *indices, float *weights) {
    if (k <= 0 || n <= 0) return;
    const int kk = k > n ? n : k;
    int *sel = (int *)malloc(sizeof(int) * (size_t)kk);
    unsigned char *used = (unsigned char *)calloc((size_t)n, 1);
    for (int t = 0; t < kk; ++t) {
        int best = -1;
        for (int i = 0; i < n; ++i) {
            if (used[i]) continue;
            if (best < 0 || gate_logits[i] > gate_logits[best]) best = i;
        }
        sel[t] = best;
        used[best] = 1;
    }
    float m = gate_logits[sel[0]];
    for (int i = 1; i < kk; ++i)
        if (gate_logits[sel[i]] > m) m = gate_logits[sel[i]];
    double sum = 0.0;
    for (int i = 0; i < kk; ++i) {
        const float e = (float)exp((double)gate_logits[sel[i]] - (double)m);
        weights[i] = e;
        sum += (double)e;
    }
    const double inv = (sum > 0.0) ? 1.0 / sum : 0.0;
    for (int i = 0; i < kk; ++i) {
        indices[i] = sel[i];
        weights[i] = (float)((double)weights[i] * inv);
    }
    for (int i = kk; i < k; ++i) {
        indices[i] = -1;
        weights[i] = 0.0f;
    }
    free(sel);
    free(used);
}

/* ------------------------------------------------------------------------ */
/* GPTQ-INT4 (kernels/matvec/matvec_gptq_ref.cpp:52-96, matmul_gptq_ref.cpp;   */
/* layout runtime/tiny_format.h:140-182)                                       */
/* ------------------------------------------------------------------------ */

static uint32_t rd_u32(const uint8_t *p) {
    uint32_t v;
    memcpy(&v, p, 4);
    return v;
}
static float rd_f16(const uint8_t *p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return tqo_half_to_float(h);
}

void tqo_matvec_gptq(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                     int group_size) {
    const uint32_t flags = rd_u32(w + 4);
    const int has_g_idx = (flags & 1u) != 0;
    const int n_groups = in_dim / group_size;
    const size_t sq = (size_t)n_groups * out_dim * 2;
    const uint8_t *scales = w + 8, *qzeros = scales + sq;
    const uint8_t *g_idx = has_g_idx ? qzeros + sq : NULL;
    const uint8_t *qweight = has_g_idx ? g_idx + (size_t)in_dim * 4 : qzeros + sq;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < out_dim; ++o) {
        double acc = 0.0;
        for (int c8 = 0; c8 < in_dim / 8; ++c8) {
            const uint32_t word = rd_u32(qweight + ((size_t)c8 * out_dim + o) * 4);
            for (int k = 0; k < 8; ++k) {
                const int c = c8 * 8 + k;
                const uint32_t nib = (word >> (k * 4)) & 0xFu;
                const int g = has_g_idx ? (int)rd_u32(g_idx + (size_t)c * 4) : c / group_size;
                const float s = rd_f16(scales + ((size_t)g * out_dim + o) * 2);
                const float z = rd_f16(qzeros + ((size_t)g * out_dim + o) * 2);
                const float dq = ((float)nib - z) * s;
                acc += (double)dq * (double)x[c];
            }
        }
        y[o] = (float)acc;
    }
}

/* matmul_gptq_ref: column n of X/Y (column-major, one token per column) is a matvec. */
void tqo_matmul_gptq(const uint8_t *w, const float *x, float *y, int M, int K, int N,
                     int group_size) {
    for (int n = 0; n < N; ++n)
        tqo_matvec_gptq(w, x + (size_t)n * K, y + (size_t)n * M, M, K, group_size);
}

/* ------------------------------------------------------------------------ */
/* Qwen3.5 GDN ops and partial RoPE (kernels/gdn/gdn_ops_ref.cpp)             */
/* ------------------------------------------------------------------------ */

static float silu_f(float x) { return x / (1.0f + expf(-x)); }

/* l2norm_inplace_ref (:44-57) */
void tqo_l2norm_inplace(float *x, int n, float eps) {
    double sumsq = 0.0;
    for (int i = 0; i < n; ++i) sumsq += (double)x[i] * (double)x[i];
    const float inv = 1.0f / sqrtf((float)sumsq + eps);
    for (int i = 0; i < n; ++i) x[i] *= inv;
}

/* causal_conv1d_update_ref (:82-105) */
void tqo_causal_conv1d_update(const float *x, float *state, const float *weight, float *out,
                              int dim, int kernel_size) {
    const int sl = kernel_size - 1;
    for (int c = 0; c < dim; ++c) {
        float *st = state + (size_t)c * sl;
        const float *w = weight + (size_t)c * kernel_size;
        const float xc = x[c];
        float acc = 0.0f;
        for (int i = 0; i < sl; ++i) acc += w[i] * st[i];
        acc += w[sl] * xc;
        out[c] = silu_f(acc);
        for (int i = 0; i < sl - 1; ++i) st[i] = st[i + 1];
        st[sl - 1] = xc;
    }
}

/* gdn_step_ref (:134-176) */
void tqo_gdn_step(float *S, const float *q, const float *k, const float *v, float g, float beta,
                  float *o, int qk_dim, int v_dim) {
    if (v_dim <= 0 || v_dim > 512) return;
    const float decay = expf(g);
    float kv[512], delta[512];
    for (int d = 0; d < v_dim; ++d) kv[d] = 0.0f;
    for (int j = 0; j < qk_dim; ++j) {
        float *row = S + (size_t)j * v_dim;
        for (int d = 0; d < v_dim; ++d) {
            row[d] *= decay;
            kv[d] += row[d] * k[j];
        }
    }
    for (int d = 0; d < v_dim; ++d) delta[d] = beta * (v[d] - kv[d]);
    for (int j = 0; j < qk_dim; ++j) {
        float *row = S + (size_t)j * v_dim;
        for (int d = 0; d < v_dim; ++d) row[d] += k[j] * delta[d];
    }
    for (int d = 0; d < v_dim; ++d) {
        double acc = 0.0;
        for (int j = 0; j < qk_dim; ++j) acc += (double)S[(size_t)j * v_dim + d] * (double)q[j];
        o[d] = (float)acc;
    }
}

/* rmsnorm_gated_ref (:203-218) */
void tqo_rmsnorm_gated(const float *x, const float *gate, const float *weight, float *y, int n,
                       float eps) {
    double sumsq = 0.0;
    for (int i = 0; i < n; ++i) sumsq += (double)x[i] * (double)x[i];
    const float scale = 1.0f / sqrtf((float)(sumsq / n) + eps);
    for (int i = 0; i < n; ++i) {
        const float normed = x[i] * scale * weight[i];
        y[i] = normed * silu_f(gate[i]);
    }
}

/* partial_rope_ref (:233-277) */
void tqo_partial_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim,
                      int rotary_dim, int pos, float theta) {
    const int half = rotary_dim / 2;
    if (rotary_dim <= 0 || rotary_dim > head_dim || rotary_dim % 2 || half > 256) return;
    float cs[256], sn[256];
    for (int i = 0; i < half; ++i) {
        const float exponent = -(float)(2 * i) / (float)rotary_dim;
        const float inv_freq = powf(theta, exponent);
        const float angle = (float)pos * inv_freq;
        cs[i] = cosf(angle);
        sn[i] = sinf(angle);
    }
    for (int h = 0; h < n_heads + n_kv_heads; ++h) {
        float *v = (h < n_heads) ? q + (size_t)h * head_dim : k + (size_t)(h - n_heads) * head_dim;
        for (int i = 0; i < half; ++i) {
            const float x0 = v[i], x1 = v[i + half];
            v[i] = x0 * cs[i] - x1 * sn[i];
            v[i + half] = x1 * cs[i] + x0 * sn[i];
        }
    }
}

/* ------------------------------------------------------------------------ */
/* whole-model decode step (runtime/qwen_forward_token.cpp:83-742)            */
/* ------------------------------------------------------------------------ */

struct tqo_model {
    tqb200_model_desc d;
    int max_seq_len, kv_fp16, pos;
    int n_layers_run, head;
    float *kv32;
    uint16_t *kv16;
    size_t layer_stride;
    float *hidden, *normed, *q, *k, *v, *attn, *o, *gate, *up, *ffn, *logits, *rot_buf;
    float *router, *acc, *eg, *eu, *eo, *topk_w;
    int *topk_i;
    /* fp16 cache guide (tests): another implementation's arena for the step; see
     * tqo_model_set_kv_guide */
    const uint16_t *guide;
    float guide_tol;
    long long guide_flips, guide_mismatches;
    double guide_max_dev;
};

/* QwenModel::mv / mv_typed (runtime/qwen_model.cpp:212-221) -> CPUBackend::matvec
 * (runtime/backend_cpu.cpp:19-33) -> the dtype's ref matvec. */
static void mv(const tqo_model *m, const tqb200_matrix *w, const float *x, float *y) {
    switch (w->dtype) {
        case TQB200_DT_I4:
            tqo_matvec_i4((const uint8_t *)w->data, x, y, w->rows, w->cols, m->d.group_size);
            break;
        case TQB200_DT_VQ2:
            tqo_matvec_vq2((const uint8_t *)w->data, x, y, w->rows, w->cols);
            break;
        case TQB200_DT_F16:
            tqo_matvec_f16((const uint16_t *)w->data, x, y, w->rows, w->cols);
            break;
        default:
            tqo_matvec_f32((const float *)w->data, x, y, w->rows, w->cols);
            break;
    }
}

/* QwenModel::mv_rot (runtime/qwen_model.cpp:229-238). */
static void mv_rot(const tqo_model *m, const tqb200_matrix *w, const float *x, float *y,
                   const tqb200_rotation *rot) {
    const float *xr = x;
    if (rot->sign) {
        const int bs = rot->block_size > 0 ? rot->block_size : tqo_hadamard_block_size(w->cols);
        tqo_biip_rotate(x, m->rot_buf, w->cols, rot->scale, rot->sign, bs);
        xr = m->rot_buf;
    }
    mv(m, w, xr, y);
}

static float *fz(size_t n) { return (float *)calloc(n ? n : 1, sizeof(float)); }

tqo_model *tqo_model_create(const tqb200_model_desc *desc, int max_seq_len, int kv_fp16) {
    if (desc->head_dim > 1024) return NULL; /* kv_write's row buffers */
    tqo_model *m = (tqo_model *)calloc(1, sizeof(tqo_model));
    m->d = *desc;
    m->max_seq_len = max_seq_len;
    m->kv_fp16 = kv_fp16;
    m->n_layers_run = desc->n_layers;
    m->head = 1;
    const size_t H = (size_t)desc->hidden, qd = (size_t)desc->n_heads * desc->head_dim;
    const size_t kvd = (size_t)desc->n_kv_heads * desc->head_dim;
    size_t inter = (size_t)desc->inter;
    if ((size_t)desc->moe_inter > inter) inter = (size_t)desc->moe_inter;
    m->layer_stride = (size_t)desc->n_kv_heads * max_seq_len * desc->head_dim;
    const size_t total = 2 * (size_t)desc->n_layers * m->layer_stride;
    if (kv_fp16)
        m->kv16 = (uint16_t *)calloc(total, sizeof(uint16_t));
    else
        m->kv32 = fz(total);
    m->hidden = fz(H);
    m->normed = fz(H);
    m->q = fz(qd);
    m->k = fz(kvd);
    m->v = fz(kvd);
    m->attn = fz(qd);
    m->o = fz(H);
    m->gate = fz(inter);
    m->up = fz(inter);
    m->ffn = fz(H);
    m->logits = fz((size_t)desc->vocab);
    size_t rb = H > inter ? H : inter;
    if (qd > rb) rb = qd;
    m->rot_buf = fz(rb);
    m->router = fz((size_t)(desc->n_experts > 0 ? desc->n_experts : 1));
    m->acc = fz(H);
    m->eg = fz(inter);
    m->eu = fz(inter);
    m->eo = fz(H);
    m->topk_w = fz((size_t)(desc->experts_per_tok > 0 ? desc->experts_per_tok : 1));
    m->topk_i = (int *)calloc((size_t)(desc->experts_per_tok > 0 ? desc->experts_per_tok : 1),
                              sizeof(int));
    return m;
}

void tqo_model_set_partial(tqo_model *m, int n_layers_run, int head) {
    m->n_layers_run = n_layers_run < m->d.n_layers ? n_layers_run : m->d.n_layers;
    m->head = head;
}

/* Spacing of binary16 values at the magnitude of h (its ulp). */
static double half_ulp(uint16_t h) {
    const int e = (h & 0x7FFF) >> 10;
    return ldexp(1.0, (e == 0 ? 1 : e) - 25);
}

/* One head row of the current position, n values written at dst[i] (binary16 bits): with
 * a guide set, the guide's row is taken (every cached element then equals the other
 * implementation's), and each element's distance from this model's own rounding is
 * measured beyond one ulp, in units of the row's largest magnitude. */
static void guided_row(tqo_model *m, uint16_t *dst, size_t idx, const uint16_t *own, int n) {
    if (!m->guide) {
        memcpy(dst, own, sizeof(uint16_t) * (size_t)n);
        return;
    }
    double rmax = 0.0;
    for (int i = 0; i < n; ++i) {
        const double a = fabs((double)tqo_half_to_float(own[i]));
        if (a > rmax) rmax = a;
    }
    for (int i = 0; i < n; ++i) {
        const uint16_t g = m->guide[idx + i];
        dst[i] = g;
        if (g == own[i]) continue;
        m->guide_flips += 1;
        const double d = fabs((double)tqo_half_to_float(g) - (double)tqo_half_to_float(own[i]));
        const double u = half_ulp(g) > half_ulp(own[i]) ? half_ulp(g) : half_ulp(own[i]);
        const double dev = rmax > 0.0 ? (d - u) / rmax : (d > u ? INFINITY : 0.0);
        if (dev > m->guide_max_dev) m->guide_max_dev = dev;
        if (dev > m->guide_tol) m->guide_mismatches += 1;
    }
}

/* KvCache::write_token (runtime/kv_cache.cpp:120-135): layout [K|V][L][KVH][max_seq][hd],
 * fp16 mode stores float_to_half. */
static void kv_write(tqo_model *m, int layer) {
    const tqb200_model_desc *d = &m->d;
    const size_t plane = (size_t)m->max_seq_len * d->head_dim;
    const size_t koff = (size_t)layer * m->layer_stride;
    const size_t voff = ((size_t)d->n_layers + layer) * m->layer_stride;
    uint16_t hk[1024], hv[1024];
    for (int h = 0; h < d->n_kv_heads; ++h) {
        const size_t base = (size_t)h * plane + (size_t)m->pos * d->head_dim;
        for (int i = 0; i < d->head_dim; ++i) {
            const float kvk = m->k[h * d->head_dim + i], kvv = m->v[h * d->head_dim + i];
            if (m->kv_fp16) {
                hk[i] = tqo_float_to_half(kvk);
                hv[i] = tqo_float_to_half(kvv);
            } else {
                m->kv32[koff + base + i] = kvk;
                m->kv32[voff + base + i] = kvv;
            }
        }
        if (m->kv_fp16) {
            guided_row(m, m->kv16 + koff + base, koff + base, hk, d->head_dim);
            guided_row(m, m->kv16 + voff + base, voff + base, hv, d->head_dim);
        }
    }
}

int tqo_model_step(tqo_model *m, int token_id) {
    const tqb200_model_desc *d = &m->d;
    const int H = d->hidden, hd = d->head_dim;
    const int qd = d->n_heads * hd, kvd = d->n_kv_heads * hd;
    if (token_id < 0 || token_id >= d->vocab || m->pos >= m->max_seq_len) return -1;

    /* embed (qwen_forward_token.cpp:121-164) */
    if (d->embed.dtype == TQB200_DT_F32) {
        memcpy(m->hidden, (const float *)d->embed.data + (size_t)token_id * H, sizeof(float) * H);
    } else if (d->embed.dtype == TQB200_DT_I4) {
        tqo_dequant_i4((const uint8_t *)d->embed.data + (size_t)token_id *
                                                           tqb200_i4_row_bytes(H, d->group_size),
                       1, H, d->group_size, m->hidden);
    } else {
        const uint16_t *row = (const uint16_t *)d->embed.data + (size_t)token_id * H;
        for (int j = 0; j < H; ++j) m->hidden[j] = tqo_half_to_float(row[j]);
    }

    const float attn_scale = 1.0f / sqrtf((float)hd);
    for (int li = 0; li < m->n_layers_run; ++li) {
        const tqb200_layer *w = &d->layers[li];
        tqo_rmsnorm(m->hidden, w->input_ln, m->normed, H, d->rms_eps);
        /* q/k/v (rotated :388-397, fused/unfused :398-420: identical numerics) */
        mv_rot(m, &w->q_proj, m->normed, m->q, &w->rot_q);
        mv_rot(m, &w->k_proj, m->normed, m->k, &w->rot_k);
        mv_rot(m, &w->v_proj, m->normed, m->v, &w->rot_v);
        if (w->q_bias) for (int j = 0; j < qd; ++j) m->q[j] += w->q_bias[j];
        if (w->k_bias) for (int j = 0; j < kvd; ++j) m->k[j] += w->k_bias[j];
        if (w->v_bias) for (int j = 0; j < kvd; ++j) m->v[j] += w->v_bias[j];
        if (w->q_norm) { /* QK-norm per head (:423-431) */
            for (int h = 0; h < d->n_heads; ++h)
                tqo_rmsnorm(m->q + h * hd, w->q_norm, m->q + h * hd, hd, d->rms_eps);
            for (int h = 0; h < d->n_kv_heads; ++h)
                tqo_rmsnorm(m->k + h * hd, w->k_norm, m->k + h * hd, hd, d->rms_eps);
        }
        tqo_rope(m->q, m->k, d->n_heads, d->n_kv_heads, hd, m->pos, d->rope_theta);
        kv_write(m, li);
        {
            const size_t koff = (size_t)li * m->layer_stride;
            const size_t voff = ((size_t)d->n_layers + li) * m->layer_stride;
            if (m->kv_fp16)
                tqo_attention_decode_f16kv(m->q, m->kv16 + koff, m->kv16 + voff, m->pos + 1,
                                           m->max_seq_len, d->n_heads, d->n_kv_heads, hd,
                                           attn_scale, m->attn);
            else
                tqo_attention_decode(m->q, m->kv32 + koff, m->kv32 + voff, m->pos + 1,
                                     m->max_seq_len, d->n_heads, d->n_kv_heads, hd, attn_scale,
                                     m->attn);
        }
        mv_rot(m, &w->o_proj, m->attn, m->o, &w->rot_o);
        for (int j = 0; j < H; ++j) m->hidden[j] += m->o[j];
        tqo_rmsnorm(m->hidden, w->post_ln, m->normed, H, d->rms_eps);

        if (d->model_type == TQB200_MODEL_QWEN3_MOE) {
            /* MoE FFN, no shared expert (:478-629) */
            mv(m, &w->router, m->normed, m->router);
            tqo_topk_softmax(m->router, d->n_experts, d->experts_per_tok, m->topk_i, m->topk_w);
            for (int j = 0; j < H; ++j) m->acc[j] = 0.0f;
            for (int t = 0; t < d->experts_per_tok; ++t) {
                const int e = m->topk_i[t];
                mv(m, &w->expert_gate[e], m->normed, m->eg);
                mv(m, &w->expert_up[e], m->normed, m->eu);
                tqo_swiglu(m->eg, m->eu, d->moe_inter);
                mv(m, &w->expert_down[e], m->eg, m->eo);
                const float wt = m->topk_w[t];
                for (int j = 0; j < H; ++j) {
                    const float c = wt * m->eo[j];
                    m->acc[j] += c;
                }
            }
            for (int j = 0; j < H; ++j) m->hidden[j] += m->acc[j];
        } else {
            /* dense FFN (:630-665) */
            mv_rot(m, &w->gate_proj, m->normed, m->gate, &w->rot_gate);
            mv_rot(m, &w->up_proj, m->normed, m->up, &w->rot_up);
            tqo_swiglu(m->gate, m->up, d->inter);
            mv_rot(m, &w->down_proj, m->gate, m->ffn, &w->rot_down);
            for (int j = 0; j < H; ++j) m->hidden[j] += m->ffn[j];
        }
    }

    int next = 0;
    if (m->head) {
        /* final norm, lm_head, argmax (:694-734) */
        tqo_rmsnorm(m->hidden, d->final_norm, m->normed, H, d->rms_eps);
        mv(m, &d->lm_head, m->normed, m->logits);
        next = tqo_argmax(m->logits, d->vocab);
    }
    m->pos += 1;
    return next;
}

const float *tqo_model_logits(const tqo_model *m) { return m->logits; }
const float *tqo_model_hidden(const tqo_model *m) { return m->hidden; }
void tqo_model_reset(tqo_model *m) { m->pos = 0; }

/* The KV arena (KvCache layout [K|V][L][KVH][max_seq][hd], fp32 or binary16 bits) and its
 * byte size, so a test can compare it with the engine's or load it from there. */
void *tqo_model_kv(tqo_model *m, size_t *bytes) {
    const size_t n = 2 * (size_t)m->d.n_layers * m->layer_stride;
    if (bytes) *bytes = n * (m->kv_fp16 ? 2 : 4);
    return m->kv_fp16 ? (void *)m->kv16 : (void *)m->kv32;
}

/* fp16 cache guide, for comparing another implementation's cache with this one step by
 * step: while set, the K/V rows this model writes are taken from the guide (an arena of
 * the same layout holding the other implementation's cache after the same step), so
 * both continue from the same cache.  Each element that differs from this model's own
 * rounding counts as a flip; its distance beyond one binary16 ulp, in units of its head
 * row's largest magnitude, is tracked (the maximum), and counts as a mismatch above tol.
 * NULL turns the guide off; the counts add up over steps. */
void tqo_model_set_kv_guide(tqo_model *m, const uint16_t *guide, float tol) {
    m->guide = guide;
    m->guide_tol = tol;
}
void tqo_model_kv_guide_counts(const tqo_model *m, long long *flips, long long *mismatches,
                               double *max_dev) {
    if (flips) *flips = m->guide_flips;
    if (mismatches) *mismatches = m->guide_mismatches;
    if (max_dev) *max_dev = m->guide_max_dev;
}

/* Position of the next step (KvCache::seq_len; rows below it must hold K/V). */
int tqo_model_set_position(tqo_model *m, int pos) {
    if (pos < 0 || pos >= m->max_seq_len) return -1;
    m->pos = pos;
    return 0;
}

void tqo_model_destroy(tqo_model *m) {
    if (!m) return;
    free(m->kv32);
    free(m->kv16);
    free(m->hidden); free(m->normed); free(m->q); free(m->k); free(m->v); free(m->attn);
    free(m->o); free(m->gate); free(m->up); free(m->ffn); free(m->logits); free(m->rot_buf);
    free(m->router); free(m->acc); free(m->eg); free(m->eu); free(m->eo); free(m->topk_w);
    free(m->topk_i);
    free(m);
}
