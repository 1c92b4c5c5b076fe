// noalloc.cu — decode attention that allocates nothing.
//
// tqb200_dev_attention_decode_noalloc() runs the split-K attention kernel, whose
// per-split partial results and per-KV-head completion tickets normally live in
// memory from cudaMalloc, with that scratch in file-scope device arrays of fixed
// size instead.  It is meant for callers that cannot allocate device memory on the
// call path: hosts whose allocator forbids allocations it does not track, embedders
// that reserve every device byte up front, and latency-critical loops that cannot
// afford an allocation call (or the device-wide synchronisation of the free that
// would follow it).  The arrays exist once per device that loads the library and
// stay allocated until the process exits.
//
// Host code cannot use the arrays' names as device addresses (in host code a
// __device__ symbol names a host-side stand-in); the device address comes from
// cudaGetSymbolAddress, looked up once per device, with that device current, by the
// first call made on it.  Make that first call outside any stream capture.  With CUDA's
// default lazy module loading, that first call is also when the driver loads this
// library's device code and places the arrays in device memory; a caller that reserves
// the rest of the device up front makes the first call before reserving it, or sets
// CUDA_MODULE_LOADING=EAGER so the arrays are placed when the library loads.
//
// Every call shares the same arrays and leaves its contents in them.  The tickets
// must start at zero, so each call clears them on its stream first.  Calls that can
// overlap on the GPU (different streams, or several host threads) race on the
// arrays and must be serialised by the caller.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace tqb200 {

// Maximum scratch: 1 Mi floats (4 MiB) of split-K partials and 256 KV-head tickets.
constexpr size_t kNoAllocPartialFloats = size_t(1) << 20;
constexpr int kNoAllocTickets = 256;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_partial[kNoAllocPartialFloats];
static __device__ __align__(256) unsigned int g_noalloc_tickets[kNoAllocTickets];

namespace {

struct NoAllocScratch {
    float *partial = nullptr;
    unsigned int *tickets = nullptr;
};

std::mutex g_noalloc_mu;
NoAllocScratch g_noalloc_dev[kNoAllocMaxDevices];

// Device addresses of the arrays on the current device (looked up on first use).
int noalloc_scratch(NoAllocScratch *out) {
    int dev = 0;
    TQ_CUDA_TRY(cudaGetDevice(&dev));
    TQ_CHECK_ARG(dev >= 0 && dev < kNoAllocMaxDevices, "device ordinal %d above %d", dev,
                 kNoAllocMaxDevices);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocScratch &s = g_noalloc_dev[dev];
    if (!s.partial) {
        void *p = nullptr, *t = nullptr;
        TQ_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_partial));
        TQ_CUDA_TRY(cudaGetSymbolAddress(&t, g_noalloc_tickets));
        s.partial = static_cast<float *>(p);
        s.tickets = static_cast<unsigned int *>(t);
    }
    *out = s;
    return TQB200_OK;
}

}  // namespace
}  // namespace tqb200

using namespace tqb200;

extern "C" int tqb200_dev_attention_decode_noalloc(const float *q, const float *k_cache,
                                                   const float *v_cache, int seq_len,
                                                   int max_seq_len, int n_heads, int n_kv_heads,
                                                   int head_dim, float scale, float *out,
                                                   void *stream) {
    TQ_CHECK_ARG(q && k_cache && v_cache && out, "attention (no-alloc): null pointer");
    TQ_CHECK_ARG(seq_len >= 1 && seq_len <= max_seq_len && n_kv_heads > 0 &&
                     n_heads % n_kv_heads == 0 && head_dim > 0,
                 "attention (no-alloc): bad shape seq %d max %d heads %d/%d hd %d", seq_len,
                 max_seq_len, n_heads, n_kv_heads, head_dim);
    TQ_CHECK_ARG(n_kv_heads <= kNoAllocTickets,
                 "attention (no-alloc): %d KV heads exceed the fixed maximum of %d", n_kv_heads,
                 kNoAllocTickets);
    const size_t per_split = attn_partial_floats(n_heads, head_dim, 1);
    TQ_CHECK_ARG(per_split <= kNoAllocPartialFloats,
                 "attention (no-alloc): %d heads x head_dim %d need %zu scratch floats per "
                 "split, above the fixed maximum of %zu",
                 n_heads, head_dim, per_split, kNoAllocPartialFloats);
    TQ_CHECK_ARG((((uintptr_t)k_cache | (uintptr_t)v_cache) & 15u) == 0,
                 "attention (no-alloc): k_cache and v_cache must be 16-byte aligned");
    NoAllocScratch s;
    const int st = noalloc_scratch(&s);
    if (st) return st;
    AttnArgs a{};
    a.q = q;
    a.k = k_cache;
    a.v = v_cache;
    a.kv_fp16 = 0;
    a.pos = nullptr;
    a.seq_len = seq_len;
    a.max_seq = max_seq_len;
    a.n_heads = n_heads;
    a.n_kv_heads = n_kv_heads;
    a.head_dim = head_dim;
    a.scale = scale;
    int nsplit = 1, chunk = max_seq_len;
    const int pst = attn_plan(n_kv_heads, max_seq_len, &nsplit, &chunk);
    if (pst) return pst;
    // fewer splits when the partials of the planned split count would not fit
    const int max_split = (int)(kNoAllocPartialFloats / per_split);
    if (nsplit > max_split) nsplit = max_split;
    a.nsplit = nsplit;
    a.chunk_max = (max_seq_len + nsplit - 1) / nsplit;
    a.partial = s.partial;
    a.tickets = s.tickets;
    a.out = out;
    cudaStream_t strm = (cudaStream_t)stream;
    TQ_CUDA_TRY(cudaMemsetAsync(s.tickets, 0, sizeof(unsigned int) * n_kv_heads, strm));
    return launch_attention_split(a, strm);
}
