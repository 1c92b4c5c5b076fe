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
/* tqb200_dev_matvec_i4 launched with programmatic dependent launch (no reference
 * counterpart): the kernel may start while the preceding kernel on the stream still runs
 * and read W then (its first weight loads overlap that kernel's tail, as the engine's
 * matvecs do); x is read, and y written, only after that kernel has completed.  For
 * weights that the preceding kernel does not write, such as the reference's immutable
 * model tensors. */
int tqb200_dev_matvec_i4_pdl(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                             int group_size, void *stream);
int tqb200_dev_dequant_i4(const uint8_t *w, int rows, int dim, int group_size, float *out,
                          void *stream);

/* MatmulI4Fn (kernels/dispatch.h:248-249); semantics of matmul_i4_ref
 * (kernels/matvec/matmul_i4_ref.cpp:53-114): Y[:, n] = W X[:, n] for n < N, X [in_dim x N]
 * and Y [out_dim x N] column-major (one token per column).  Runs on the tensor cores
 * (tcgen05: exact bf16 codes against bf16 hi/lo activations, per-group partials in TMEM,
 * fp32 accumulation); group_size 32, 64 or 128 (TQB200_ERR_INVALID_ARG otherwise). */
int tqb200_matmul_i4(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim, int n,
                     int group_size);
/* Device twin.  `scratch` (16-byte aligned) holds
 * tqb200_matmul_i4_scratch_bytes(out_dim, in_dim, n, group_size) bytes for the weights in
 * the kernel's tile order and the split activations (0 for an unsupported group size);
 * no reference counterpart. */
size_t tqb200_matmul_i4_scratch_bytes(int out_dim, int in_dim, int n, int group_size);
int tqb200_dev_matmul_i4(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                         int n, int group_size, void *scratch, void *stream);

/* ------------------------------------------------------ VQ2 + BiIP rotation
 * VQ2 tensor: [codebook 256x4 fp16 = 2048 B][one uint8 index per 4 weights, row-major]
 * (runtime/tiny_format.h:91-103).  in_dim % 4 == 0. */

/* MatvecVQ2Fn (kernels/dispatch.h:187); matvec_vq2_ref, kernels/matvec/matvec_vq2_ref.cpp:52-82. */
int tqb200_matvec_vq2(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim);
/* BiipRotateFn (kernels/dispatch.h:227); biip_rotate_activation_ref,
 * kernels/biip/biip_rotate.cpp:36-69.  scale may be NULL; x == y allowed. */
int tqb200_biip_rotate(const float *x, float *y, int dim, const float *scale, const float *sign,
                       int block_size);
/* Fused: y = W_vq2 * BiIP(x) in one launch (QwenModel::mv_rot, runtime/qwen_model.cpp:229-238);
 * sign == NULL skips the rotation. */
int tqb200_matvec_vq2_rot(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                          const float *scale, const float *sign, int block_size);
int tqb200_dev_matvec_vq2_rot(const uint8_t *w, const float *x, float *y, int out_dim,
                              int in_dim, const float *scale, const float *sign, int block_size,
                              void *stream);

/* -------------------------------------------------- decode ops (host pointers)
 * Same signatures and meaning as the reference's ops dispatch entries
 * (kernels/dispatch.h:298-307, shared --ops-impl name); status instead of abort. */

/* RmsnormFn (kernels/dispatch.h:298); rmsnorm_ref, kernels/rmsnorm/rmsnorm_ref.cpp:48-78. In-place safe. */
int tqb200_rmsnorm(const float *x, const float *weight, float *y, int n, float eps);
/* RopeFn (kernels/dispatch.h:299); rope_ref, kernels/rope/rope_ref.cpp:56-117.  q, k in place. */
int tqb200_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim, int pos,
                float theta);
/* AttentionDecodeFn (kernels/dispatch.h:301); attention_decode_ref,
 * kernels/attention/attention_decode_ref.cpp:53-143.  k/v: one layer, [KVH][max_seq_len][hd]. */
int tqb200_attention_decode(const float *q, const float *k_cache, const float *v_cache,
                            int seq_len, int max_seq_len, int n_heads, int n_kv_heads,
                            int head_dim, float scale, float *out);
/* IBackend::attention_decode_f16kv (runtime/backend.h:246-249): fp16 (binary16 bits) KV. */
int tqb200_attention_decode_f16kv(const float *q, const uint16_t *k_cache,
                                  const uint16_t *v_cache, int seq_len, int max_seq_len,
                                  int n_heads, int n_kv_heads, int head_dim, float scale,
                                  float *out);
/* Decode attention on DEVICE pointers (fp32 KV, the arguments of AttentionDecodeFn plus a
 * cudaStream_t) that allocates nothing.  It has no counterpart in the reference.  It is for
 * callers that cannot allocate device memory on the call path: an allocator that forbids
 * allocations it does not track, every device byte reserved up front, or a loop that cannot
 * afford an allocation call.  Its split-K scratch is a fixed file-scope device array of 4 MiB
 * plus 256 KV-head tickets per device, held until the process exits; shapes needing more than
 * 4 MiB for one split or more than 256 KV heads are rejected with TQB200_ERR_INVALID_ARG, as
 * are k/v caches that are not 16-byte aligned.  Every call clears the tickets on its stream.
 * The first call on a device looks up the array's address, so make it outside any stream
 * capture.  CUDA loads a library's device code lazily by default, so that first call is
 * also when the driver loads this library's kernels and places the arrays in device
 * memory: make it before reserving the rest of the device, or set
 * CUDA_MODULE_LOADING=EAGER so that the arrays are placed when the library is loaded.
 * All calls share the array: calls that overlap on the GPU race. */
int tqb200_dev_attention_decode_noalloc(const float *q, const float *k_cache,
                                        const float *v_cache, int seq_len, int max_seq_len,
                                        int n_heads, int n_kv_heads, int head_dim, float scale,
                                        float *out, void *stream);
/* SwigluFn (kernels/dispatch.h:304); swiglu_ref, kernels/silu/swiglu_ref.cpp:41-52.  gate in place. */
int tqb200_swiglu(float *gate, const float *up, int n);
/* ArgmaxFn (kernels/dispatch.h:305) returns the index; here via *index (first maximum). */
int tqb200_argmax(const float *logits, int n, int *index);
/* TopKSoftmaxFn (kernels/dispatch.h:306); topk_softmax_ref,
 * kernels/topk_softmax/topk_softmax_ref.cpp:41-78 (n <= 1024, k <= 64; ties -> lower index). */
int tqb200_topk_softmax(const float *gate_logits, int n, int k, int *indices, float *weights);

/* ---------------------------------------------- Qwen3.5 GDN ops and partial RoPE
 * Same signatures and meaning as the reference's GDN dispatch entries
 * (kernels/dispatch.h:389-396, the --ops-impl name) and IBackend::partial_rope
 * (runtime/backend.h:211); semantics of kernels/gdn/gdn_ops_ref.cpp. */

/* L2normInplaceFn; l2norm_inplace_ref (gdn_ops_ref.cpp:44-57). */
int tqb200_l2norm_inplace(float *x, int n, float eps);
/* CausalConv1dUpdateFn; causal_conv1d_update_ref (gdn_ops_ref.cpp:82-105): conv_state
 * [dim][kernel_size-1] is updated in place, out[dim] = silu(conv). */
int tqb200_causal_conv1d_update(const float *x, float *conv_state, const float *weight, float *out,
                                int dim, int kernel_size);
/* GdnStepFn; gdn_step_ref (gdn_ops_ref.cpp:134-176): one head, S [qk_dim][v_dim] in place,
 * v_dim <= 512 (TQB200_ERR_INVALID_ARG otherwise). */
int tqb200_gdn_step(float *S, const float *q, const float *k, const float *v, float g, float beta,
                    float *o, int qk_dim, int v_dim);
/* Device twin over n_heads heads at once (S [n_heads][qk_dim][v_dim], q/k [n_heads][qk_dim],
 * v/o [n_heads][v_dim]); decay[h] = exp(g_h) and beta[h] on the device.  No reference
 * counterpart (the reference calls gdn_step once per head). */
int tqb200_dev_gdn_step(float *S, const float *q, const float *k, const float *v,
                        const float *decay, const float *beta, float *o, int n_heads, int qk_dim,
                        int v_dim, void *stream);
/* RmsnormGatedFn; rmsnorm_gated_ref (gdn_ops_ref.cpp:203-218). */
int tqb200_rmsnorm_gated(const float *x, const float *gate, const float *weight, float *y, int n,
                         float eps);
/* IBackend::partial_rope (runtime/backend.h:211); partial_rope_ref (gdn_ops_ref.cpp:233-277):
 * rotate-half RoPE over the first rotary_dim dimensions of every head. */
int tqb200_partial_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim,
                        int rotary_dim, int pos, float theta);

/* ------------------------------------------------------ GPTQ-INT4, dense f32 / f16
 * GPTQ tensor (runtime/tiny_format.h:140-182): [u32 magic][u32 flags][scales f16
 * [n_groups][out]][qzeros f16 [n_groups][out]][g_idx u32 [in], when flags & 1]
 * [qweight u32 [in/8][out], column-major]; in % group_size == 0, group_size % 8 == 0. */

/* MatvecGPTQFn (kernels/dispatch.h:211); matvec_gptq_ref (kernels/matvec/matvec_gptq_ref.cpp). */
int tqb200_matvec_gptq(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                       int group_size);
/* MatmulGPTQFn (kernels/dispatch.h:258); matmul_gptq_ref: X [in x n], Y [out x n] column-major. */
int tqb200_matmul_gptq(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim, int n,
                       int group_size);
int tqb200_dev_matvec_gptq(const uint8_t *w, int has_g_idx, const float *x, float *y, int out_dim,
                           int in_dim, int group_size, void *stream);
/* MatvecFn (kernels/dispatch.h:45; matvec_f32_ref) and MatvecF16Fn (:98; matvec_f16_ref):
 * dense row-major weights, double accumulation. */
int tqb200_matvec_f32(const float *w, const float *x, float *y, int out_dim, int in_dim);
int tqb200_matvec_f16(const uint16_t *w, const float *x, float *y, int out_dim, int in_dim);

/* -------------------------------------------------- whole-step decode engine
 * Replaces the GPU decode registry entry (GpuDecodeCreateFn / StepFn / ResetFn /
 * DestroyFn / LogitsFn, kernels/dispatch.h:353-378; the reference's engine is
 * kernels/cuda/gpu_engine.cu).  create() takes a tqb200_model_desc instead of a
 * ModelFile; the adapter builds one from the ModelFile's tensor table.  The
 * engine owns device copies of every weight, the KV arena and activations; a
 * step runs one CUDA graph and returns the greedy next token
 * (QwenModel::forward_token, runtime/qwen_forward_token.cpp:83-742). */
typedef struct tqb200_engine tqb200_engine;

typedef struct tqb200_engine_opts {
    int max_seq_len;   /* KV positions (<= desc->max_seq_len when that is > 0) */
    int kv_fp16;       /* 0 = fp32 KV (reference default), 1 = fp16 KV (RNE store, --kv-f16) */
    int use_graph;     /* capture the step once and replay it (default 1) */
    int pdl;           /* programmatic dependent launch between kernels (default 1) */
    int device;        /* CUDA device ordinal; -1 = current */
    /* Column-parallel sharding over tp_size GPUs, one process per GPU (new in this build;
     * the reference is single-device).  Dense models: every projection's output rows, the
     * attention heads and lm_head's vocabulary rows are split, and the activations are
     * all-gathered at each layer boundary (NCCL, or the peer exchange below).  MoE models:
     * expert parallelism (each rank holds tp_size-th of the experts; the attention runs
     * whole on every rank; the chosen experts' outputs are exchanged once per layer) with
     * lm_head split by vocabulary.  All ranks call create/step/generate/prefill in
     * lockstep. */
    int tp_size;       /* 1 = single GPU */
    int tp_rank;
    unsigned char nccl_id[128];  /* from tqb200_nccl_unique_id() on one rank, shared to all */
    int reserved[8];
} tqb200_engine_opts;

/* An NCCL unique id for tqb200_engine_opts.nccl_id (TQB200_ERR_UNSUPPORTED when the
 * library was built without NCCL). */
int tqb200_nccl_unique_id(unsigned char id[128]);

/* Peer exchange (no reference counterpart; the reference is single-device).  Every rank
 * exports its activation arena (a CUDA IPC handle, 64 bytes) after tqb200_engine_create,
 * the ranks share the handles (rank r's at handles + 64 r), and every rank then opens the
 * others' arenas.  From the next step on, each layer's all-gathers run inside the kernels
 * that produce the rows: attention, o_proj, gate/up and down (a MoE layer's expert down)
 * store their rows into every rank's buffer over NVLink and release a per-exchange counter
 * there; the consuming kernel waits for it (bounded: 20 s, then status
 * TQB200_ERR_TIMEOUT) instead of an NCCL launch.  Results are bit-identical to the NCCL
 * path.  i4 models only (VQ2 models keep NCCL); at most 8 ranks; all ranks must open
 * before any steps. */
int tqb200_engine_exchange_handle(tqb200_engine *e, unsigned char handle[64]);
int tqb200_engine_open_exchange(tqb200_engine *e, const unsigned char *handles, int n_ranks);

void tqb200_engine_default_opts(tqb200_engine_opts *opts);
/* GpuDecodeCreateFn (kernels/dispatch.h:356). */
int tqb200_engine_create(const tqb200_model_desc *desc, const tqb200_engine_opts *opts,
                         tqb200_engine **out);
/* GpuDecodeStepFn (kernels/dispatch.h:358): feeds token_id at the current position. */
int tqb200_engine_step(tqb200_engine *e, int token_id, int *next_token);
/* QwenModel::forward_prefill (runtime/qwen_model.h:169, runtime/qwen_forward_prefill.cpp:74):
 * feeds the n prompt tokens at positions pos .. pos+n-1 as one batch (projections and
 * experts on the tensor-core matmul, causal attention over the cache), leaves their K/V
 * in the cache and the last token's logits in the engine, and returns the greedy next
 * token.  Under expert parallelism (MoE, tp_size > 1) each rank's grouped GEMM covers its
 * own experts and the expert rows are summed across the ranks.  Falls back to n decode
 * steps where the batched path does not apply (dense models with tp_size > 1, VQ2
 * projections, head_dim other than 64/128), as the reference falls back to
 * forward_token. */
int tqb200_engine_prefill(tqb200_engine *e, const int *tokens, int n, int *next_token);
/* tqb200_engine_prefill launched kernel by kernel with a CUDA event after each launch:
 * ms_by_kind[k] sums the times of kind k (the kinds of tqb200_engine_profile_step, then
 * rmsnorm, x_pack, moe_plan, swiglu).  Batched prefill only (TQB200_ERR_INVALID_ARG
 * otherwise). */
int tqb200_engine_profile_prefill(tqb200_engine *e, const int *tokens, int n, float *ms_by_kind,
                                  int n_kinds, int *next_token);
/* Greedy-decodes n_steps tokens with the produced token fed back on the device (no
 * host round trip per token; main.cpp's decode loop, runtime/main.cpp:1038-1041, moved
 * onto the GPU): step i feeds the token of step i-1, the first feeds token_id.
 * out_tokens[n_steps] receives the produced ids; *device_ms (optional) the CUDA-event
 * time of the n graph launches. */
int tqb200_engine_generate(tqb200_engine *e, int token_id, int n_steps, int *out_tokens,
                           float *device_ms);
/* One step launched kernel by kernel (no graph, no PDL) with a CUDA event after every
 * launch; ms_by_kind[k] sums the kernel time per kind: 0 embed, 1 qkv, 2 qk-norm/rope/
 * kv-append, 3 attention, 4 o_proj, 5 gate/up, 6 down, 7 lm_head(+argmax). */
int tqb200_engine_profile_step(tqb200_engine *e, int token_id, float *ms_by_kind, int n_kinds,
                               int *next_token);
/* GpuDecodeResetFn (kernels/dispatch.h:359): rewinds the position to 0. */
int tqb200_engine_reset(tqb200_engine *e);
/* GpuDecodeDestroyFn (kernels/dispatch.h:360). */
int tqb200_engine_destroy(tqb200_engine *e);
/* GpuDecodeLogitsFn (kernels/dispatch.h:361): DEVICE pointer to [vocab] logits. */
const float *tqb200_engine_logits(const tqb200_engine *e);
int tqb200_engine_copy_logits(const tqb200_engine *e, float *host, int n);
int tqb200_engine_position(const tqb200_engine *e);
/* Sets the position of the next step (positions below it must already hold KV). */
int tqb200_engine_set_position(tqb200_engine *e, int pos);
/* The engine's CUDA stream and KV arena ([K|V][L][KVH][max_seq][hd]), for harnesses. */
int tqb200_engine_stream(const tqb200_engine *e, void **stream);
int tqb200_engine_kv_cache(const tqb200_engine *e, void **kv, size_t *bytes);
int tqb200_engine_weight_bytes(const tqb200_engine *e, size_t *bytes);
/* Device bytes the batched prefill holds in addition to the weights (no reference
 * counterpart): repacked copies of the matrices its tensor-core matmul cannot read in
 * place (those with in_dim / group_size not a multiple of 4); 0 before the first prefill
 * and when every matrix is read in place through a tensor map. */
int tqb200_engine_prefill_copy_bytes(const tqb200_engine *e, size_t *bytes);

/* In-graph timeline of tqb200_engine_generate (no reference counterpart; the reference
 * profiles a step op by op on the host, runtime/main.cpp --profile-out).  With a timeline
 * set, the generate graph is captured again with every projection, attention, router and
 * combine launch in a stamped form: each CTA's last thread records the global timer when
 * it enters, when it gets past its dependency wait and when it exits (plain stores at its
 * exit), for each of the first max_steps steps of every generate() call; max_steps = 0
 * turns it off and restores the unstamped kernels.  Needs use_graph. */
int tqb200_engine_set_timeline(tqb200_engine *e, int max_steps);
/* The last generate() call's timeline, averaged over its recorded steps: per kernel kind
 * (the kinds of tqb200_engine_profile_step) excl_ms[k] sums, per step, the launches'
 * in-step times, each from the launch's first CTA past its dependency wait to the next
 * stamped launch's (the step's last one: to its last CTA out), so they do not overlap
 * and the kernels that are not stamped (embed, token feed, NCCL) count with the launch
 * before them; incl_ms[k] the times from the first CTA in to the last out (overlapping
 * the previous kernel under programmatic dependent launch); launches[k] = launches of
 * kind k per step; *span_ms = first stamped CTA in to the last out. */
int tqb200_engine_timeline(const tqb200_engine *e, int n_kinds, double *excl_ms, double *incl_ms,
                           int *launches, int *steps, double *span_ms);
/* One recorded step of that timeline launch by launch: kinds[i] and, in us[6 i .. 6 i + 5],
 * the first and last CTA's entry, wait and exit of launch i in microseconds from the
 * step's first stamp (-1 where no CTA stamped).  *n_launches = launches reported. */
int tqb200_engine_timeline_launches(const tqb200_engine *e, int step, int max_launches,
                                    int *kinds, double *us, int *n_launches);

#ifdef __cplusplus
}
#endif
#endif /* TQB200_H */
