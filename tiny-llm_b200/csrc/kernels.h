// kernels.h — internal (C++) launch API shared by capi.cu and engine.cu.
// All launchers are stream-ordered, take device pointers, and return a
// TQB200_* status (errors recorded through set_error).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace tqb200 {

// ------------------------------------------------------------------ i4
// One matrix of a fused i4 matvec launch.  All jobs share x, in_dim and group.
struct I4Job {
    const uint8_t *w;     // interleaved i4 rows
    float *y;             // [rows]
    const float *bias;    // optional [rows], added after the dot (fp32)
    const float *resid;   // optional [rows]: y = resid + dot (residual fused into the store)
    int rows;
};

// y_j = W_j x (+bias_j) for up to 3 jobs in one launch (q/k/v, gate/up, ...).
int launch_i4_matvec(const I4Job *jobs, int n_jobs, const float *x, int in_dim, int group_size,
                     cudaStream_t stream);
// Symmetric W4A8 ("sdot5") semantics.
int launch_i4_matvec_sym(const uint8_t *w, const float *x, float *y, int rows, int in_dim,
                         int group_size, cudaStream_t stream);
// Bit-exact dequant of `rows` rows to fp32.
int launch_i4_dequant(const uint8_t *w, int rows, int dim, int group_size, float *out,
                      cudaStream_t stream);
// One dequantised row (embedding lookup, dequant_i4_row) selected on device by *token.
int launch_i4_embed_row(const uint8_t *w, const int *token, int dim, int group_size, float *out,
                        cudaStream_t stream);

int num_sms();

}  // namespace tqb200
