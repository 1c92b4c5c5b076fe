// capi.cu — the extern "C" boundary of libtqb200.so (declared in include/tqb200.h).
//
// Host-pointer entry points mirror the reference's dispatch signatures
// (kernels/dispatch.h) and are synchronous, like the reference's CPU
// variants: upload, launch, download, synchronise.  Device-pointer twins
// (tqb200_dev_*) are stream-ordered and never synchronise.
#include <cmath>
#include <cstdarg>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace tqb200 {

namespace {
thread_local char g_err[1024] = "";
}

int set_error(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return status;
}

// ------------------------------------------------------------------ device context
namespace {

struct DevBuf {
    void *p = nullptr;
    size_t cap = 0;
};

struct HostCtx {
    int device = -1;
    cudaStream_t stream = nullptr;
    std::vector<DevBuf> scratch;                            // per-call argument slots
    std::unordered_map<std::string, DevBuf> resident;       // (host ptr, bytes) -> device copy
    bool resident_on = false;
};

std::mutex g_mu;
HostCtx g_ctx;

int ensure_device() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return set_error(TQB200_ERR_NO_DEVICE, "no CUDA device visible");
    }
    int dev = 0;
    TQ_CUDA_TRY(cudaGetDevice(&dev));
    if (g_ctx.device != dev) {
        if (g_ctx.stream) cudaStreamDestroy(g_ctx.stream);
        for (auto &b : g_ctx.scratch)
            if (b.p) cudaFree(b.p);
        for (auto &kv : g_ctx.resident)
            if (kv.second.p) cudaFree(kv.second.p);
        g_ctx.scratch.clear();
        g_ctx.resident.clear();
        g_ctx.stream = nullptr;
        g_ctx.device = dev;
        TQ_CUDA_TRY(cudaStreamCreateWithFlags(&g_ctx.stream, cudaStreamNonBlocking));
    }
    return TQB200_OK;
}

// Growable device slot; contents undefined.  Allocations are 256-byte aligned.
int scratch(int slot, size_t bytes, void **out) {
    if ((int)g_ctx.scratch.size() <= slot) g_ctx.scratch.resize(slot + 1);
    DevBuf &b = g_ctx.scratch[slot];
    if (b.cap < bytes) {
        if (b.p) cudaFree(b.p);
        b.p = nullptr;
        b.cap = 0;
        const size_t cap = ((bytes + 255) / 256) * 256 + 256;
        TQ_CUDA_TRY(cudaMalloc(&b.p, cap));
        b.cap = cap;
    }
    *out = b.p;
    return TQB200_OK;
}

int upload(int slot, const void *host, size_t bytes, void **dev) {
    int st = scratch(slot, bytes ? bytes : 1, dev);
    if (st) return st;
    if (bytes) TQ_CUDA_TRY(cudaMemcpyAsync(*dev, host, bytes, cudaMemcpyHostToDevice, g_ctx.stream));
    return TQB200_OK;
}

// Weight upload: resident cache keyed by (host pointer, size) when enabled.
int upload_weight(int slot, const void *host, size_t bytes, void **dev) {
    if (!g_ctx.resident_on) return upload(slot, host, bytes, dev);
    char key[64];
    snprintf(key, sizeof key, "%p:%zu", host, bytes);
    auto it = g_ctx.resident.find(key);
    if (it != g_ctx.resident.end()) {
        *dev = it->second.p;
        return TQB200_OK;
    }
    DevBuf b;
    TQ_CUDA_TRY(cudaMalloc(&b.p, bytes + 256));
    b.cap = bytes + 256;
    TQ_CUDA_TRY(cudaMemcpy(b.p, host, bytes, cudaMemcpyHostToDevice));
    g_ctx.resident[key] = b;
    *dev = b.p;
    return TQB200_OK;
}

int download(void *host, const void *dev, size_t bytes) {
    if (bytes) TQ_CUDA_TRY(cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, g_ctx.stream));
    return TQB200_OK;
}

int finish() {
    TQ_CUDA_TRY(cudaStreamSynchronize(g_ctx.stream));
    return TQB200_OK;
}

#define TQ_TRY(expr)            \
    do {                        \
        int s_ = (expr);        \
        if (s_) return s_;      \
    } while (0)

size_t i4_bytes(int rows, int cols, int g) {
    const size_t ng = (size_t)(cols + g - 1) / g;
    return (size_t)rows * ng * (size_t)(4 + g / 2);
}

int check_i4(int rows, int cols, int g) {
    TQ_CHECK_ARG(rows >= 0 && cols > 0, "bad i4 shape %d x %d", rows, cols);
    TQ_CHECK_ARG(g > 0 && g % 2 == 0 && g <= 4096, "bad group_size %d", g);
    return TQB200_OK;
}

}  // namespace
}  // namespace tqb200

using namespace tqb200;

extern "C" {

int tqb200_version(void) { return 10000; }

const char *tqb200_last_error(void) { return g_err; }

const char *tqb200_status_string(int status) {
    switch (status) {
        case TQB200_OK: return "ok";
        case TQB200_ERR_INVALID_ARG: return "invalid argument";
        case TQB200_ERR_CUDA: return "CUDA error";
        case TQB200_ERR_UNSUPPORTED: return "unsupported";
        case TQB200_ERR_NO_DEVICE: return "no CUDA device";
        case TQB200_ERR_TIMEOUT: return "device wait timed out";
        default: return "unknown status";
    }
}

int tqb200_device_count(int *count) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    if (count) *count = n;
    return TQB200_OK;
}

int tqb200_set_resident_weights(int enabled) {
    std::lock_guard<std::mutex> lk(g_mu);
    g_ctx.resident_on = enabled != 0;
    return TQB200_OK;
}

int tqb200_clear_resident_weights(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto &kv : g_ctx.resident)
        if (kv.second.p) cudaFree(kv.second.p);
    g_ctx.resident.clear();
    return TQB200_OK;
}

// ------------------------------------------------------------------ i4 (host pointers)
int tqb200_matvec_i4(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                     int group_size) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_TRY(check_i4(out_dim, in_dim, group_size));
    TQ_CHECK_ARG(w && x && y, "null pointer");
    TQ_TRY(ensure_device());
    void *dw, *dx, *dy;
    TQ_TRY(upload_weight(0, w, i4_bytes(out_dim, in_dim, group_size), &dw));
    TQ_TRY(upload(3, x, (size_t)in_dim * 4, &dx));
    TQ_TRY(scratch(4, (size_t)out_dim * 4, &dy));
    I4Job j{(const uint8_t *)dw, (float *)dy, nullptr, nullptr, out_dim};
    TQ_TRY(launch_i4_matvec(&j, 1, (const float *)dx, in_dim, group_size, g_ctx.stream));
    TQ_TRY(download(y, dy, (size_t)out_dim * 4));
    return finish();
}

int tqb200_matvec_pair_i4(const uint8_t *w1, const uint8_t *w2, const float *x, float *y1,
                          float *y2, int out_dim, int in_dim, int group_size) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_TRY(check_i4(out_dim, in_dim, group_size));
    TQ_CHECK_ARG(w1 && w2 && x && y1 && y2, "null pointer");
    TQ_TRY(ensure_device());
    const size_t wb = i4_bytes(out_dim, in_dim, group_size);
    void *dw1, *dw2, *dx, *dy1, *dy2;
    TQ_TRY(upload_weight(0, w1, wb, &dw1));
    TQ_TRY(upload_weight(1, w2, wb, &dw2));
    TQ_TRY(upload(3, x, (size_t)in_dim * 4, &dx));
    TQ_TRY(scratch(4, (size_t)out_dim * 4, &dy1));
    TQ_TRY(scratch(5, (size_t)out_dim * 4, &dy2));
    I4Job j[2] = {{(const uint8_t *)dw1, (float *)dy1, nullptr, nullptr, out_dim},
                  {(const uint8_t *)dw2, (float *)dy2, nullptr, nullptr, out_dim}};
    TQ_TRY(launch_i4_matvec(j, 2, (const float *)dx, in_dim, group_size, g_ctx.stream));
    TQ_TRY(download(y1, dy1, (size_t)out_dim * 4));
    TQ_TRY(download(y2, dy2, (size_t)out_dim * 4));
    return finish();
}

int tqb200_matvec_qkv_i4(const uint8_t *wq, const uint8_t *wk, const uint8_t *wv,
                         const float *x, float *yq, float *yk, float *yv, int q_dim, int kv_dim,
                         int in_dim, int group_size) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_TRY(check_i4(q_dim, in_dim, group_size));
    TQ_TRY(check_i4(kv_dim, in_dim, group_size));
    TQ_CHECK_ARG(wq && wk && wv && x && yq && yk && yv, "null pointer");
    TQ_TRY(ensure_device());
    void *dq, *dk, *dv, *dx, *oq, *ok, *ov;
    TQ_TRY(upload_weight(0, wq, i4_bytes(q_dim, in_dim, group_size), &dq));
    TQ_TRY(upload_weight(1, wk, i4_bytes(kv_dim, in_dim, group_size), &dk));
    TQ_TRY(upload_weight(2, wv, i4_bytes(kv_dim, in_dim, group_size), &dv));
    TQ_TRY(upload(3, x, (size_t)in_dim * 4, &dx));
    TQ_TRY(scratch(4, (size_t)q_dim * 4, &oq));
    TQ_TRY(scratch(5, (size_t)kv_dim * 4, &ok));
    TQ_TRY(scratch(6, (size_t)kv_dim * 4, &ov));
    I4Job j[3] = {{(const uint8_t *)dq, (float *)oq, nullptr, nullptr, q_dim},
                  {(const uint8_t *)dk, (float *)ok, nullptr, nullptr, kv_dim},
                  {(const uint8_t *)dv, (float *)ov, nullptr, nullptr, kv_dim}};
    TQ_TRY(launch_i4_matvec(j, 3, (const float *)dx, in_dim, group_size, g_ctx.stream));
    TQ_TRY(download(yq, oq, (size_t)q_dim * 4));
    TQ_TRY(download(yk, ok, (size_t)kv_dim * 4));
    TQ_TRY(download(yv, ov, (size_t)kv_dim * 4));
    return finish();
}

int tqb200_matvec_i4_sym(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                         int group_size) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_TRY(check_i4(out_dim, in_dim, group_size));
    TQ_CHECK_ARG(w && x && y, "null pointer");
    TQ_TRY(ensure_device());
    void *dw, *dx, *dy;
    TQ_TRY(upload_weight(0, w, i4_bytes(out_dim, in_dim, group_size), &dw));
    TQ_TRY(upload(3, x, (size_t)in_dim * 4, &dx));
    TQ_TRY(scratch(4, (size_t)out_dim * 4, &dy));
    TQ_TRY(launch_i4_matvec_sym((const uint8_t *)dw, (const float *)dx, (float *)dy, out_dim,
                                in_dim, group_size, g_ctx.stream));
    TQ_TRY(download(y, dy, (size_t)out_dim * 4));
    return finish();
}

int tqb200_dequant_i4(const uint8_t *w, int rows, int dim, int group_size, float *out) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_TRY(check_i4(rows, dim, group_size));
    TQ_CHECK_ARG(w && out, "null pointer");
    TQ_TRY(ensure_device());
    void *dw, *dout;
    TQ_TRY(upload_weight(0, w, i4_bytes(rows, dim, group_size), &dw));
    TQ_TRY(scratch(4, (size_t)rows * dim * 4, &dout));
    TQ_TRY(launch_i4_dequant((const uint8_t *)dw, rows, dim, group_size, (float *)dout,
                             g_ctx.stream));
    TQ_TRY(download(out, dout, (size_t)rows * dim * 4));
    return finish();
}

// ------------------------------------------------------------------ i4 (device pointers)
int tqb200_dev_matvec_i4(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                         int group_size, void *stream) {
    TQ_TRY(check_i4(out_dim, in_dim, group_size));
    TQ_CHECK_ARG(w && x && y, "null pointer");
    I4Job j{w, y, nullptr, nullptr, out_dim};
    return launch_i4_matvec(&j, 1, x, in_dim, group_size, (cudaStream_t)stream);
}

int tqb200_dev_matvec_i4_pdl(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                             int group_size, void *stream) {
    TQ_TRY(check_i4(out_dim, in_dim, group_size));
    TQ_CHECK_ARG(w && x && y, "null pointer");
    I4Job j{w, y, nullptr, nullptr, out_dim};
    I4LaunchOpts o;
    o.x.mode = X_PLAIN;
    o.x.src = x;
    o.pdl = true;  // W may be read before the preceding kernel completes; x only after
    return launch_i4_matvec_ex(&j, 1, in_dim, group_size, o, (cudaStream_t)stream);
}

int tqb200_dev_matvec_i4_sym(const uint8_t *w, const float *x, float *y, int out_dim,
                             int in_dim, int group_size, void *stream) {
    TQ_TRY(check_i4(out_dim, in_dim, group_size));
    TQ_CHECK_ARG(w && x && y, "null pointer");
    return launch_i4_matvec_sym(w, x, y, out_dim, in_dim, group_size, (cudaStream_t)stream);
}

int tqb200_dev_dequant_i4(const uint8_t *w, int rows, int dim, int group_size, float *out,
                          void *stream) {
    TQ_TRY(check_i4(rows, dim, group_size));
    TQ_CHECK_ARG(w && out, "null pointer");
    return launch_i4_dequant(w, rows, dim, group_size, out, (cudaStream_t)stream);
}

// ------------------------------------------------------------------ i4 matmul
static int check_mm(int M, int K, int N, int G) {
    TQ_TRY(check_i4(M, K, G));
    TQ_CHECK_ARG(N >= 0, "matmul_i4: bad column count %d", N);
    TQ_CHECK_ARG(mm_group_supported(G), "matmul_i4: group_size %d is not 32, 64 or 128", G);
    return TQB200_OK;
}

int tqb200_matmul_i4(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim, int n,
                     int group_size) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_TRY(check_mm(out_dim, in_dim, n, group_size));
    TQ_CHECK_ARG(w && x && y, "null pointer");
    if (out_dim == 0 || n == 0) return TQB200_OK;
    TQ_TRY(ensure_device());
    void *dw, *dx, *dy, *ds, *dst;
    TQ_TRY(upload_weight(0, w, i4_bytes(out_dim, in_dim, group_size), &dw));
    TQ_TRY(upload(3, x, (size_t)in_dim * n * 4, &dx));
    TQ_TRY(scratch(4, (size_t)out_dim * n * 4, &dy));
    TQ_TRY(scratch(9, mm_scratch_bytes(out_dim, in_dim, n, group_size), &ds));
    TQ_TRY(scratch(10, 16, &dst));
    TQ_CUDA_TRY(cudaMemsetAsync(dst, 0, 4, g_ctx.stream));
    TQ_TRY(launch_matmul_i4((const uint8_t *)dw, (const float *)dx, (float *)dy, out_dim, in_dim,
                            n, group_size, ds, (int *)dst, g_ctx.stream));
    TQ_TRY(download(y, dy, (size_t)out_dim * n * 4));
    int hst = 0;
    TQ_TRY(download(&hst, dst, 4));
    TQ_TRY(finish());
    if (hst != 0) return set_error(TQB200_ERR_TIMEOUT, "matmul_i4: device status %d", hst);
    return TQB200_OK;
}

size_t tqb200_matmul_i4_scratch_bytes(int out_dim, int in_dim, int n, int group_size) {
    if (out_dim < 0 || in_dim <= 0 || n < 0) return 0;
    return mm_scratch_bytes(out_dim, in_dim, n, group_size);
}

int tqb200_dev_matmul_i4(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                         int n, int group_size, void *scratch, void *stream) {
    TQ_TRY(check_mm(out_dim, in_dim, n, group_size));
    TQ_CHECK_ARG(w && x && y && scratch, "null pointer");
    TQ_CHECK_ARG(((uintptr_t)scratch & 15) == 0, "matmul_i4: scratch not 16-byte aligned");
    return launch_matmul_i4(w, x, y, out_dim, in_dim, n, group_size, scratch, nullptr,
                            (cudaStream_t)stream);
}

// ------------------------------------------------------------------ VQ2 + BiIP
static int vq2_host(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                    const float *scale, const float *sign, int bs) {
    TQ_CHECK_ARG(w && x && y && out_dim >= 0 && in_dim > 0 && in_dim % 4 == 0,
                 "vq2: bad arguments (%d x %d)", out_dim, in_dim);
    TQ_TRY(ensure_device());
    void *dw, *dx, *dy, *dsg = nullptr, *dsc = nullptr;
    TQ_TRY(upload_weight(0, w, 2048 + (size_t)out_dim * (in_dim / 4), &dw));
    TQ_TRY(upload(3, x, (size_t)in_dim * 4, &dx));
    TQ_TRY(scratch(4, (size_t)out_dim * 4, &dy));
    if (sign) {
        TQ_TRY(upload(7, sign, (size_t)in_dim * 4, &dsg));
        if (scale) TQ_TRY(upload(8, scale, (size_t)in_dim * 4, &dsc));
    }
    VqLaunch a;
    a.job[0].w = (const uint8_t *)dw;
    a.job[0].y = (float *)dy;
    a.job[0].rows = out_dim;
    a.job[0].rot_sign = (const float *)dsg;
    a.job[0].rot_scale = (const float *)dsc;
    a.job[0].rot_bs = bs;
    a.K = in_dim;
    a.x.mode = X_PLAIN;
    a.x.src = (const float *)dx;
    TQ_TRY(launch_vq2_matvec(a, g_ctx.stream));
    TQ_TRY(download(y, dy, (size_t)out_dim * 4));
    return finish();
}

int tqb200_matvec_vq2(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim) {
    std::lock_guard<std::mutex> lk(g_mu);
    return vq2_host(w, x, y, out_dim, in_dim, nullptr, nullptr, 0);
}

int tqb200_matvec_vq2_rot(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                          const float *scale, const float *sign, int block_size) {
    std::lock_guard<std::mutex> lk(g_mu);
    return vq2_host(w, x, y, out_dim, in_dim, scale, sign, block_size);
}

int tqb200_dev_matvec_vq2_rot(const uint8_t *w, const float *x, float *y, int out_dim,
                              int in_dim, const float *scale, const float *sign, int block_size,
                              void *stream) {
    TQ_CHECK_ARG(w && x && y && in_dim % 4 == 0, "vq2: bad arguments");
    VqLaunch a;
    a.job[0].w = w;
    a.job[0].y = y;
    a.job[0].rows = out_dim;
    a.job[0].rot_sign = sign;
    a.job[0].rot_scale = scale;
    a.job[0].rot_bs = block_size;
    a.K = in_dim;
    a.x.mode = X_PLAIN;
    a.x.src = x;
    return launch_vq2_matvec(a, (cudaStream_t)stream);
}

int tqb200_biip_rotate(const float *x, float *y, int dim, const float *scale, const float *sign,
                       int block_size) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_CHECK_ARG(x && y && sign && dim > 0, "biip: bad arguments");
    TQ_TRY(ensure_device());
    void *dx, *dsg, *dsc = nullptr, *dy;
    TQ_TRY(upload(3, x, (size_t)dim * 4, &dx));
    TQ_TRY(upload(7, sign, (size_t)dim * 4, &dsg));
    if (scale) TQ_TRY(upload(8, scale, (size_t)dim * 4, &dsc));
    TQ_TRY(scratch(4, (size_t)dim * 4, &dy));
    TQ_TRY(launch_biip((const float *)dx, (float *)dy, dim, (const float *)dsc, (const float *)dsg,
                       block_size, g_ctx.stream));
    TQ_TRY(download(y, dy, (size_t)dim * 4));
    return finish();
}

// ------------------------------------------------------------------ decode ops (host pointers)
int tqb200_rmsnorm(const float *x, const float *weight, float *y, int n, float eps) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_CHECK_ARG(x && weight && y && n > 0, "rmsnorm: bad arguments");
    TQ_TRY(ensure_device());
    void *dx, *dw;
    TQ_TRY(upload(3, x, (size_t)n * 4, &dx));
    TQ_TRY(upload(7, weight, (size_t)n * 4, &dw));
    TQ_TRY(launch_rmsnorm((const float *)dx, (const float *)dw, (float *)dx, 1, n, eps,
                          g_ctx.stream));
    TQ_TRY(download(y, dx, (size_t)n * 4));
    return finish();
}

int tqb200_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim, int pos,
                float theta) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_CHECK_ARG(q && k && n_heads >= 0 && n_kv_heads >= 0 && head_dim > 0 && pos >= 0,
                 "rope: bad arguments");
    TQ_CHECK_ARG(head_dim % 2 == 0 && head_dim / 2 <= 256, "rope_ref: unsupported head_dim %d",
                 head_dim);
    TQ_TRY(ensure_device());
    void *dq, *dk, *dt;
    const size_t qb = (size_t)n_heads * head_dim * 4, kb = (size_t)n_kv_heads * head_dim * 4;
    std::vector<float> tab(head_dim);
    rope_row(theta, head_dim, pos, tab.data(), tab.data() + head_dim / 2);
    TQ_TRY(upload(3, q, qb, &dq));
    TQ_TRY(upload(7, k, kb, &dk));
    TQ_TRY(upload(8, tab.data(), (size_t)head_dim * 4, &dt));
    TQ_TRY(launch_rope((float *)dq, (float *)dk, n_heads, n_kv_heads, head_dim, (const float *)dt,
                       (const float *)dt + head_dim / 2, g_ctx.stream));
    TQ_TRY(download(q, dq, qb));
    TQ_TRY(download(k, dk, kb));
    return finish();
}

static int attention_host(const float *q, const void *kc, const void *vc, int elem, int seq_len,
                          int max_seq_len, int n_heads, int n_kv_heads, int head_dim,
                          float scale, float *out) {
    TQ_CHECK_ARG(q && kc && vc && out, "attention: null pointer");
    TQ_CHECK_ARG(seq_len >= 1 && seq_len <= max_seq_len && n_kv_heads > 0 &&
                     n_heads % n_kv_heads == 0 && head_dim > 0,
                 "attention: bad shape seq %d max %d heads %d/%d hd %d", seq_len, max_seq_len,
                 n_heads, n_kv_heads, head_dim);
    TQ_TRY(ensure_device());
    // only the first seq_len positions of every KV head travel: [KVH][seq_len][hd]
    const size_t row = (size_t)seq_len * head_dim * elem, pitch = (size_t)max_seq_len * head_dim * elem;
    void *dq, *dk, *dv, *dout, *dpart, *dtick;
    TQ_TRY(upload(3, q, (size_t)n_heads * head_dim * 4, &dq));
    TQ_TRY(scratch(8, row * n_kv_heads, &dk));
    TQ_TRY(scratch(9, row * n_kv_heads, &dv));
    TQ_CUDA_TRY(cudaMemcpy2DAsync(dk, row, kc, pitch, row, n_kv_heads, cudaMemcpyHostToDevice,
                                  g_ctx.stream));
    TQ_CUDA_TRY(cudaMemcpy2DAsync(dv, row, vc, pitch, row, n_kv_heads, cudaMemcpyHostToDevice,
                                  g_ctx.stream));
    AttnArgs a{};
    a.q = (const float *)dq;
    a.k = dk;
    a.v = dv;
    a.kv_fp16 = elem == 2;
    a.pos = nullptr;
    a.seq_len = seq_len;
    a.max_seq = seq_len;  // the device copy is packed to seq_len positions per head
    a.n_heads = n_heads;
    a.n_kv_heads = n_kv_heads;
    a.head_dim = head_dim;
    a.scale = scale;
    TQ_TRY(attn_plan(n_kv_heads, seq_len, &a.nsplit, &a.chunk_max));
    TQ_TRY(scratch(10, attn_partial_floats(n_heads, head_dim, a.nsplit) * 4, &dpart));
    if ((int)g_ctx.scratch.size() <= 11 || g_ctx.scratch[11].cap < (size_t)n_kv_heads * 4) {
        TQ_TRY(scratch(11, (size_t)n_kv_heads * 4, &dtick));
        TQ_CUDA_TRY(cudaMemsetAsync(dtick, 0, g_ctx.scratch[11].cap, g_ctx.stream));
    }
    dtick = g_ctx.scratch[11].p;
    TQ_TRY(scratch(4, (size_t)n_heads * head_dim * 4, &dout));
    a.partial = (float *)dpart;
    a.tickets = (unsigned int *)dtick;
    a.out = (float *)dout;
    TQ_TRY(launch_attention(a, g_ctx.stream));
    TQ_TRY(download(out, dout, (size_t)n_heads * head_dim * 4));
    return finish();
}

int tqb200_attention_decode(const float *q, const float *k_cache, const float *v_cache,
                            int seq_len, int max_seq_len, int n_heads, int n_kv_heads,
                            int head_dim, float scale, float *out) {
    std::lock_guard<std::mutex> lk(g_mu);
    return attention_host(q, k_cache, v_cache, 4, seq_len, max_seq_len, n_heads, n_kv_heads,
                          head_dim, scale, out);
}

int tqb200_attention_decode_f16kv(const float *q, const uint16_t *k_cache,
                                  const uint16_t *v_cache, int seq_len, int max_seq_len,
                                  int n_heads, int n_kv_heads, int head_dim, float scale,
                                  float *out) {
    std::lock_guard<std::mutex> lk(g_mu);
    return attention_host(q, k_cache, v_cache, 2, seq_len, max_seq_len, n_heads, n_kv_heads,
                          head_dim, scale, out);
}

int tqb200_swiglu(float *gate, const float *up, int n) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_CHECK_ARG(gate && up && n >= 0, "swiglu: bad arguments");
    if (n == 0) return TQB200_OK;
    TQ_TRY(ensure_device());
    void *dg, *du;
    TQ_TRY(upload(3, gate, (size_t)n * 4, &dg));
    TQ_TRY(upload(7, up, (size_t)n * 4, &du));
    TQ_TRY(launch_swiglu((float *)dg, (const float *)du, n, g_ctx.stream));
    TQ_TRY(download(gate, dg, (size_t)n * 4));
    return finish();
}

int tqb200_argmax(const float *logits, int n, int *index) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_CHECK_ARG(logits && index && n > 0, "argmax: bad arguments");
    TQ_TRY(ensure_device());
    void *dl, *pv, *pi, *dt, *dout;
    TQ_TRY(upload(3, logits, (size_t)n * 4, &dl));
    const int nb = argmax_blocks(n);
    TQ_TRY(scratch(12, (size_t)nb * 4, &pv));
    TQ_TRY(scratch(13, (size_t)nb * 4, &pi));
    if ((int)g_ctx.scratch.size() <= 14 || g_ctx.scratch[14].p == nullptr) {
        TQ_TRY(scratch(14, 64, &dt));
        TQ_CUDA_TRY(cudaMemsetAsync(dt, 0, 64, g_ctx.stream));
    }
    dt = g_ctx.scratch[14].p;
    dout = (char *)dt + 16;
    TQ_TRY(launch_argmax((const float *)dl, n, (float *)pv, (int *)pi, (unsigned int *)dt,
                         (int *)dout, g_ctx.stream));
    TQ_TRY(download(index, dout, 4));
    return finish();
}

int tqb200_topk_softmax(const float *gate_logits, int n, int k, int *indices, float *weights) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_CHECK_ARG(gate_logits && indices && weights, "topk_softmax: null pointer");
    if (k <= 0 || n <= 0) return TQB200_OK;  // the reference returns without writing
    TQ_CHECK_ARG(n <= 1024 && k <= 64, "topk_softmax: n %d k %d beyond 1024/64", n, k);
    TQ_TRY(ensure_device());
    void *dl, *di, *dw;
    TQ_TRY(upload(3, gate_logits, (size_t)n * 4, &dl));
    TQ_TRY(scratch(4, (size_t)k * 4, &di));
    TQ_TRY(scratch(5, (size_t)k * 4, &dw));
    TQ_TRY(launch_topk_softmax((const float *)dl, n, k, (int *)di, (float *)dw, g_ctx.stream));
    TQ_TRY(download(indices, di, (size_t)k * 4));
    TQ_TRY(download(weights, dw, (size_t)k * 4));
    return finish();
}

// ------------------------------------------------------------------ GDN ops, partial RoPE
int tqb200_l2norm_inplace(float *x, int n, float eps) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_CHECK_ARG(x && n > 0, "l2norm_inplace: bad arguments");
    TQ_TRY(ensure_device());
    void *dx;
    TQ_TRY(upload(3, x, (size_t)n * 4, &dx));
    TQ_TRY(launch_l2norm((float *)dx, 1, n, eps, g_ctx.stream));
    TQ_TRY(download(x, dx, (size_t)n * 4));
    return finish();
}

int tqb200_causal_conv1d_update(const float *x, float *conv_state, const float *weight, float *out,
                                int dim, int kernel_size) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_CHECK_ARG(x && conv_state && weight && out && dim > 0,
                 "causal_conv1d_update: bad arguments");
    TQ_CHECK_ARG(kernel_size >= 2, "causal_conv1d_update_ref: kernel_size %d < 2", kernel_size);
    TQ_TRY(ensure_device());
    const size_t sb = (size_t)dim * (kernel_size - 1) * 4;
    void *dx, *ds, *dw, *dout;
    TQ_TRY(upload(3, x, (size_t)dim * 4, &dx));
    TQ_TRY(upload(7, conv_state, sb, &ds));
    TQ_TRY(upload_weight(8, weight, (size_t)dim * kernel_size * 4, &dw));
    TQ_TRY(scratch(4, (size_t)dim * 4, &dout));
    TQ_TRY(launch_causal_conv1d((const float *)dx, (float *)ds, (const float *)dw, (float *)dout,
                                dim, kernel_size, g_ctx.stream));
    TQ_TRY(download(out, dout, (size_t)dim * 4));
    TQ_TRY(download(conv_state, ds, sb));
    return finish();
}

int tqb200_gdn_step(float *S, const float *q, const float *k, const float *v, float g, float beta,
                    float *o, int qk_dim, int v_dim) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_CHECK_ARG(S && q && k && v && o && qk_dim > 0, "gdn_step: bad arguments");
    TQ_CHECK_ARG(v_dim > 0 && v_dim <= 512, "gdn_step_ref: unsupported v_dim %d", v_dim);
    TQ_TRY(ensure_device());
    // decay = exp(g) with the host's libm, as gdn_step_ref computes it (std::exp(float))
    const float dc[2] = {std::exp(g), beta};
    const size_t sb = (size_t)qk_dim * v_dim * 4;
    void *dS, *dq, *dk, *dv, *dp, *dout;
    TQ_TRY(upload(3, S, sb, &dS));
    TQ_TRY(upload(7, q, (size_t)qk_dim * 4, &dq));
    TQ_TRY(upload(8, k, (size_t)qk_dim * 4, &dk));
    TQ_TRY(upload(9, v, (size_t)v_dim * 4, &dv));
    TQ_TRY(upload(10, dc, sizeof dc, &dp));
    TQ_TRY(scratch(4, (size_t)v_dim * 4, &dout));
    TQ_TRY(launch_gdn_step((float *)dS, (const float *)dq, (const float *)dk, (const float *)dv,
                           (const float *)dp, (const float *)dp + 1, (float *)dout, 1, qk_dim,
                           v_dim, g_ctx.stream));
    TQ_TRY(download(o, dout, (size_t)v_dim * 4));
    TQ_TRY(download(S, dS, sb));
    return finish();
}

int tqb200_dev_gdn_step(float *S, const float *q, const float *k, const float *v,
                        const float *decay, const float *beta, float *o, int n_heads, int qk_dim,
                        int v_dim, void *stream) {
    TQ_CHECK_ARG(S && q && k && v && decay && beta && o, "gdn_step: null pointer");
    return launch_gdn_step(S, q, k, v, decay, beta, o, n_heads, qk_dim, v_dim,
                           (cudaStream_t)stream);
}

int tqb200_rmsnorm_gated(const float *x, const float *gate, const float *weight, float *y, int n,
                         float eps) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_CHECK_ARG(x && gate && weight && y && n > 0, "rmsnorm_gated: bad arguments");
    TQ_TRY(ensure_device());
    void *dx, *dg, *dw, *dy;
    TQ_TRY(upload(3, x, (size_t)n * 4, &dx));
    TQ_TRY(upload(7, gate, (size_t)n * 4, &dg));
    TQ_TRY(upload(8, weight, (size_t)n * 4, &dw));
    TQ_TRY(scratch(4, (size_t)n * 4, &dy));
    TQ_TRY(launch_rmsnorm_gated((const float *)dx, (const float *)dg, (const float *)dw, (float *)dy,
                                1, n, eps, g_ctx.stream));
    TQ_TRY(download(y, dy, (size_t)n * 4));
    return finish();
}

int tqb200_partial_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim,
                        int rotary_dim, int pos, float theta) {
    std::lock_guard<std::mutex> lk(g_mu);
    TQ_CHECK_ARG(q && k && n_heads >= 0 && n_kv_heads >= 0 && head_dim > 0 && pos >= 0,
                 "partial_rope: bad arguments");
    TQ_CHECK_ARG(rotary_dim > 0 && rotary_dim <= head_dim && rotary_dim % 2 == 0,
                 "partial_rope_ref: bad rotary_dim %d (head_dim %d)", rotary_dim, head_dim);
    TQ_CHECK_ARG(rotary_dim / 2 <= 256, "partial_rope_ref: rotary_dim %d too large", rotary_dim);
    TQ_TRY(ensure_device());
    // the position's cos/sin with the host libm, the reference's expression with the
    // rotary width in place of head_dim (kernels/gdn/gdn_ops_ref.cpp:246-254)
    std::vector<float> tab(rotary_dim);
    rope_row(theta, rotary_dim, pos, tab.data(), tab.data() + rotary_dim / 2);
    const size_t qb = (size_t)n_heads * head_dim * 4, kb = (size_t)n_kv_heads * head_dim * 4;
    void *dq, *dk, *dt;
    TQ_TRY(upload(3, q, qb, &dq));
    TQ_TRY(upload(7, k, kb, &dk));
    TQ_TRY(upload(8, tab.data(), (size_t)rotary_dim * 4, &dt));
    TQ_TRY(launch_partial_rope((float *)dq, (float *)dk, n_heads, n_kv_heads, head_dim, rotary_dim,
                               (const float *)dt, (const float *)dt + rotary_dim / 2,
                               g_ctx.stream));
    TQ_TRY(download(q, dq, qb));
    TQ_TRY(download(k, dk, kb));
    return finish();
}

// ------------------------------------------------------------------ GPTQ, dense matvec
static int gptq_host(const uint8_t *w, const float *x, float *y, int out, int in, int n, int G) {
    TQ_CHECK_ARG(w && x && y && out > 0 && in > 0 && n > 0, "gptq: bad arguments");
    TQ_CHECK_ARG(G > 0 && in % G == 0 && G % 8 == 0 && in % 8 == 0,
                 "gptq: in_dim %d / group_size %d (in %% G == 0, G %% 8 == 0)", in, G);
    TQ_TRY(ensure_device());
    uint32_t flags = 0;
    std::memcpy(&flags, w + 4, 4);
    const bool gidx = (flags & 1u) != 0;
    void *dw, *dx, *dy;
    TQ_TRY(upload_weight(2, w, gptq_bytes(out, in, G, gidx), &dw));
    TQ_TRY(upload(3, x, (size_t)in * n * 4, &dx));
    TQ_TRY(scratch(4, (size_t)out * n * 4, &dy));
    TQ_TRY(launch_gptq_matmul((const uint8_t *)dw, gidx, (const float *)dx, (float *)dy, out, in, n,
                              G, g_ctx.stream));
    TQ_TRY(download(y, dy, (size_t)out * n * 4));
    return finish();
}

int tqb200_matvec_gptq(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim,
                       int group_size) {
    std::lock_guard<std::mutex> lk(g_mu);
    return gptq_host(w, x, y, out_dim, in_dim, 1, group_size);
}

int tqb200_matmul_gptq(const uint8_t *w, const float *x, float *y, int out_dim, int in_dim, int n,
                       int group_size) {
    std::lock_guard<std::mutex> lk(g_mu);
    return gptq_host(w, x, y, out_dim, in_dim, n, group_size);
}

int tqb200_dev_matvec_gptq(const uint8_t *w, int has_g_idx, const float *x, float *y, int out_dim,
                           int in_dim, int group_size, void *stream) {
    TQ_CHECK_ARG(w && x && y, "gptq: null pointer");
    return launch_gptq_matmul(w, has_g_idx != 0, x, y, out_dim, in_dim, 1, group_size,
                              (cudaStream_t)stream);
}

static int dense_host(const void *w, bool f16, const float *x, float *y, int out, int in) {
    TQ_CHECK_ARG(w && x && y && out >= 0 && in > 0, "matvec: bad arguments");
    if (out == 0) return TQB200_OK;
    TQ_TRY(ensure_device());
    void *dw, *dx, *dy;
    TQ_TRY(upload_weight(2, w, (size_t)out * in * (f16 ? 2 : 4), &dw));
    TQ_TRY(upload(3, x, (size_t)in * 4, &dx));
    TQ_TRY(scratch(4, (size_t)out * 4, &dy));
    TQ_TRY(launch_dense_matvec(dw, f16, (const float *)dx, (float *)dy, out, in, g_ctx.stream));
    TQ_TRY(download(y, dy, (size_t)out * 4));
    return finish();
}

int tqb200_matvec_f32(const float *w, const float *x, float *y, int out_dim, int in_dim) {
    std::lock_guard<std::mutex> lk(g_mu);
    return dense_host(w, false, x, y, out_dim, in_dim);
}

int tqb200_matvec_f16(const uint16_t *w, const float *x, float *y, int out_dim, int in_dim) {
    std::lock_guard<std::mutex> lk(g_mu);
    return dense_host(w, true, x, y, out_dim, in_dim);
}

}  // extern "C"
