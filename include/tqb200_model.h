/*
 * tqb200_model.h — plain-C description of a tinyqwen decoder whose weights
 * already sit in memory (host or device).
 *
 * This is the argument of tqb200_engine_create().  It replaces the
 * `const void *model_file` (a tinyqwen::ModelFile) that the reference passes
 * to GpuDecodeCreateFn (kernels/dispatch.h:356): the reference-side adapter
 * (tiny-llm_b200/host/b200_variants.cpp) fills this struct from the
 * ModelFile's tensor table using exactly the tensor names QwenModel::create
 * binds (runtime/qwen_model.cpp:438-649), so the engine never links the
 * reference's loader.  All pointers are borrowed; the engine copies what it
 * needs to the device (repacking quantised matrices) during create.
 *
 * Byte layouts are the reference's in-band formats:
 *   TQB200_DT_I4   rows of ceil(in/G) groups, each [scale f16][zero f16][G/2 nibble bytes],
 *                  low nibble = even column      (runtime/tiny_format.h:66-77)
 *   TQB200_DT_VQ2  [codebook 256x4 f16 = 2048 B][rows x in/4 uint8 indices]
 *                                                (runtime/tiny_format.h:91-103)
 *   TQB200_DT_F32 / TQB200_DT_F16  dense row-major.
 */
#ifndef TQB200_MODEL_H
#define TQB200_MODEL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Dtype codes: the numeric values of tinyqwen::Dtype (runtime/tiny_format.h:197-205). */
enum {
    TQB200_DT_F32 = 0,
    TQB200_DT_F16 = 1,
    TQB200_DT_I4 = 3,
    TQB200_DT_VQ2 = 4
};

/* Model families: the numeric values of tinyqwen::ModelType (runtime/tiny_format.h:185-193).
 * Qwen2 covers Qwen2.x and dense Qwen3 (QK-norm is keyed on q_norm != NULL, as in
 * runtime/qwen_model.cpp:628-637); Qwen3MoE is the all-full-attention MoE family. */
enum {
    TQB200_MODEL_QWEN2 = 0,
    TQB200_MODEL_QWEN3_MOE = 3
};

/* A quantised or dense matrix [rows x cols]. */
typedef struct tqb200_matrix {
    const void *data;   /* bytes in the layout named by dtype; NULL = absent */
    int dtype;          /* TQB200_DT_* */
    int rows;
    int cols;
} tqb200_matrix;

/* BiIP activation rotation of one projection's input (runtime/qwen_model.cpp:427-435).
 * sign == NULL means the projection is not rotated. scale may be NULL. */
typedef struct tqb200_rotation {
    const float *sign;   /* [dim] +-1 */
    const float *scale;  /* [dim] or NULL */
    int block_size;      /* Hadamard block; 0 = derive as the reference does */
} tqb200_rotation;

typedef struct tqb200_layer {
    const float *input_ln;     /* [hidden] */
    const float *post_ln;      /* [hidden] */
    tqb200_matrix q_proj, k_proj, v_proj, o_proj;
    const float *q_bias, *k_bias, *v_bias;   /* optional (Qwen2) */
    const float *q_norm, *k_norm;            /* optional (Qwen3 QK-norm), [head_dim] */
    /* dense FFN */
    tqb200_matrix gate_proj, up_proj, down_proj;
    /* BiIP rotations (VQ2 / rotated models) */
    tqb200_rotation rot_q, rot_k, rot_v, rot_o, rot_gate, rot_up, rot_down;
    /* MoE FFN (model_type == TQB200_MODEL_QWEN3_MOE) */
    tqb200_matrix router;                    /* [n_experts x hidden] */
    const tqb200_matrix *expert_gate;        /* n_experts entries, [moe_inter x hidden] */
    const tqb200_matrix *expert_up;          /* n_experts entries, [moe_inter x hidden] */
    const tqb200_matrix *expert_down;        /* n_experts entries, [hidden x moe_inter] */
} tqb200_layer;

typedef struct tqb200_model_desc {
    int model_type;          /* TQB200_MODEL_* */
    int n_layers;
    int hidden;
    int inter;               /* dense FFN width (unused by MoE layers) */
    int n_heads;
    int n_kv_heads;
    int head_dim;
    int vocab;
    int group_size;          /* i4 group size of every i4 matrix */
    int max_seq_len;         /* model limit (header max_seq_len) */
    float rms_eps;
    float rope_theta;
    /* MoE */
    int n_experts;
    int experts_per_tok;
    int moe_inter;
    /* embeddings / head */
    tqb200_matrix embed;     /* [vocab x hidden], f32 / f16 / i4 */
    tqb200_matrix lm_head;   /* [vocab x hidden]; may alias embed (tied) */
    const float *final_norm; /* [hidden] */
    const tqb200_layer *layers;  /* n_layers entries */
} tqb200_model_desc;

/* Bytes of an i4 matrix row (runtime/tiny_format.h:73-77). */
static inline size_t tqb200_i4_row_bytes(int cols, int group_size) {
    const int groups = (cols + group_size - 1) / group_size;
    return (size_t)groups * (size_t)(4 + group_size / 2);
}

/* Bytes of a VQ2 tensor (runtime/tiny_format.h:100-103). */
static inline size_t tqb200_vq2_bytes(int rows, int cols) {
    return 2048u + (size_t)rows * (size_t)(cols / 4);
}

#ifdef __cplusplus
}
#endif
#endif /* TQB200_MODEL_H */
