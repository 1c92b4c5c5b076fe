/*
 * tqb200.h — C ABI of libtqb200.so, the B200-native (sm_100a) quantised decode
 * hot path for tinyqwen (918822019/tiny-llm).
 *
 * Plain C: pointers, sizes, int status codes; no CUDA or torch types.  Every
 * entry point names the reference interface it replaces (path:line inside the
 * reference tree).  Per-op entry points take HOST pointers and keep the
 * reference's argument meaning, so the reference's dispatch registries can
 * bind them through the adapter in tiny-llm_b200/host/b200_variants.cpp;
 * tqb200_dev_* twins take DEVICE pointers and a cudaStream_t passed as void*.
 *
 * Errors: every function returns TQB200_OK (0) or a TQB200_ERR_* code and
 * records a message readable with tqb200_last_error() (thread-local).  The
 * reference aborts instead (kernels/dispatch.cpp:393-398,
 * kernels/cuda/gpu_engine.cu:38-45); the adapter converts codes back to that
 * behaviour.  Nothing here falls back to a CPU implementation.
 */
#ifndef TQB200_H
#define TQB200_H

#include <stddef.h>
#include <stdint.h>

#include "tqb200_model.h"

#ifdef __cplusplus
extern "C" {
#endif

#define TQB200_OK 0
#define TQB200_ERR_INVALID_ARG 1
#define TQB200_ERR_CUDA 2
#define TQB200_ERR_UNSUPPORTED 3
#define TQB200_ERR_NO_DEVICE 4
#define TQB200_ERR_TIMEOUT 5

/* ----------------------------------------------------------------- library */
int tqb200_version(void);
const char *tqb200_last_error(void);
const char *tqb200_status_string(int status);
/* Number of visible CUDA devices (0 on a GPU-less host; never an error). */
int tqb200_device_count(int *count);

/* Per-op host-pointer calls copy every argument to the device on each call.
 * With resident weights on, a weight blob is uploaded once and reused while
 * the same host pointer and byte size come back (the reference's mmap'd
 * tensors never change; kernels/matvec/matvec_f32_cuda_resident.cu keys its
 * device copies the same way).  Off by default.  */
int tqb200_set_resident_weights(int enabled);
int tqb200_clear_resident_weights(void);

/* ------------------------------------------------------ i4 (HQQ/RTN, group G)
 * Layout: rows of ceil(in/G) groups [scale f16][zero f16][G/2 bytes], low
 * nibble = even column (runtime/tiny_format.h:66-77).  y = W x with
 * w = (q - zero) * scale.  */

/* MatvecI4Fn (kernels/dispatch.h:151); semantics of matvec_i4_ref
 * (kernels/matvec/matvec_i4_ref.cpp:45-103). */
int tqb200_matvec_i4(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                     int group_size);
/* MatvecPairI4Fn (kernels/dispatch.h:162): two matrices, one x, one launch. */
int tqb200_matvec_pair_i4(const uint8_t *w1, const uint8_t *w2, const float *x, float *y1,
                          float *y2, int out_dim, int in_dim, int group_size);
/* MatvecQkvI4Fn (kernels/dispatch.h:169): q/k/v, one launch. */
int tqb200_matvec_qkv_i4(const uint8_t *wq, const uint8_t *wk, const uint8_t *wv,
                         const float *x, float *yq, float *yk, float *yv, int q_dim, int kv_dim,
                         int in_dim, int group_size);
/* Symmetric W4A8 ("sdot5", kernels/matvec/matvec_i4_sdot5.cpp:276): x quantised to
 * int8 with amax/127, integer group dots of (q-8)*xq; the zero field is ignored
 * exactly as sdot5 ignores it. */
int tqb200_matvec_i4_sym(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                         int group_size);
/* dequant_i4_row (kernels/ref_ops.h:183-205) over `rows` rows: bit-exact fp32. */
int tqb200_dequant_i4(const uint8_t *w, int rows, int dim, int group_size, float *out);

/* Device-pointer twins (stream = cudaStream_t or NULL). */
int tqb200_dev_matvec_i4(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                         int group_size, void *stream);
int tqb200_dev_matvec_i4_sym(const uint8_t *w, const float *x, float *y, int out_dim,
                             int in_dim, int group_size, void *stream);
int tqb200_dev_dequant_i4(const uint8_t *w, int rows, int dim, int group_size, float *out,
                          void *stream);

#ifdef __cplusplus
}
#endif
#endif /* TQB200_H */
