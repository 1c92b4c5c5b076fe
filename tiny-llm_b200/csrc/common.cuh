// common.cuh — shared device helpers for the tqb200 sm_100a kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdio>

#include "../../include/tqb200.h"

namespace tqb200 {

// ---------------------------------------------------------------- errors
// Sets the thread-local error message and returns the status (capi.cu).
int set_error(int status, const char *fmt, ...);

#define TQ_CUDA_TRY(expr)                                                                  \
    do {                                                                                   \
        cudaError_t e_ = (expr);                                                           \
        if (e_ != cudaSuccess) {                                                           \
            cudaGetLastError(); /* a non-sticky error must not surface at a later check */ \
            return ::tqb200::set_error(TQB200_ERR_CUDA, "%s:%d %s: %s", __FILE__, __LINE__, \
                                       #expr, cudaGetErrorString(e_));                     \
        }                                                                                  \
    } while (0)

#define TQ_CHECK_ARG(cond, ...)                                                            \
    do {                                                                                   \
        if (!(cond)) return ::tqb200::set_error(TQB200_ERR_INVALID_ARG, __VA_ARGS__);      \
    } while (0)

// Largest dynamic shared memory a block may opt into on the current device.
inline int max_dyn_smem() {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) {
        cudaGetLastError();
        return 227 * 1024 - 1024;
    }
    return v;
}

// Per-kernel record of the devices whose dynamic shared-memory limit has been raised,
// with the limit itself, so later launches skip the attribute queries.
struct KernelSmem {
    std::atomic<unsigned long long> mask{0};
    std::atomic<int> limit[64] = {};
};

// Raises kernel k's dynamic shared-memory limit to the most it can use on the current
// device (the opt-in limit minus its static shared memory), once per device.  *limit
// receives that most.
template <typename Kern>
inline cudaError_t smem_limit_once(Kern k, KernelSmem &ks, int *limit) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (ks.mask.load() & bit) {
        *limit = ks.limit[dev & 63].load();
        return cudaSuccess;
    }
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, k);
    if (e != cudaSuccess) return e;
    const int lim = max_dyn_smem() - (int)fa.sharedSizeBytes;
    *limit = lim;
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    if (e == cudaSuccess) {
        ks.limit[dev & 63].store(lim);
        ks.mask.fetch_or(bit);
    }
    return e;
}

// ---------------------------------------------------------------- fp16
// Exact binary16 -> binary32 (hardware cvt; identical values to the reference's
// half_to_float, kernels/ref_ops.h:51-74).
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// binary32 -> binary16 with the reference's exact rules (kernels/ref_ops.h:78-105):
// round-to-nearest-even, NaN -> sign|0x7E00, |f| < 2^-24 -> signed zero.  The
// last rule differs from IEEE (which rounds (2^-25, 2^-24) up to 2^-24), so the
// hardware conversion cannot be used where the KV cache must match bit for bit.
__device__ __forceinline__ uint16_t f2h_ref(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t a = x & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return (uint16_t)(sign | 0x7E00u);
    if (a >= 0x47800000u) return (uint16_t)(sign | 0x7C00u);
    if (a >= 0x38800000u) {
        uint32_t base = (a >> 13) - (112u << 10);
        const uint32_t rem = a & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (base & 1u))) base += 1u;
        return (uint16_t)(sign | base);
    }
    if (a < 0x33800000u) return (uint16_t)sign;
    const int e = (int)(a >> 23) - 127;
    const uint32_t mant = (a & 0x7FFFFFu) | 0x800000u;
    const int sh = -1 - e;
    uint32_t q = mant >> sh;
    const uint32_t rem = mant & ((1u << sh) - 1u);
    const uint32_t halfway = 1u << (sh - 1);
    if (rem > halfway || (rem == halfway && (q & 1u))) q += 1u;
    return (uint16_t)(sign | q);
}

// ---------------------------------------------------------------- loads
__device__ __forceinline__ uint32_t ldg_u32(const void *p) {
    uint32_t v;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 ldg_u128_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// ---------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------- mbarrier / bulk copy
// Thin wrappers over the sm_90+/sm_100 PTX for 1-D TMA bulk copies into shared
// memory completed on an mbarrier.  Waits are bounded (see mbar_wait).
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// Returns true once the phase with the given parity has completed, false when
// `max_cycles` SM clock cycles pass first (the caller records an error and stops).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, long long max_cycles) {
    const uint32_t a = smem_u32(bar);
    const long long t0 = clock64();
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
        if (clock64() - t0 > max_cycles) return false;
    }
}

// As mbar_wait, but each probe may suspend the thread for up to `hint_ns` until the phase
// completes (mbarrier.try_wait's suspend-time hint), so waiting warps leave the issue
// slots of their scheduler to the warps that are working.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, long long max_cycles,
                                                uint32_t hint_ns = 10000u) {
    const uint32_t a = smem_u32(bar);
    const long long t0 = clock64();
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(parity), "r"(hint_ns)
            : "memory");
        if (done) return true;
        if (clock64() - t0 > max_cycles) return false;
    }
}

// ~1 s at B200 clocks: no legitimate wait on a bulk copy comes near it.
constexpr long long kWaitCycles = 2000000000LL;

// Programmatic dependent launch (sm_90+): no-ops when launched without the attribute.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ uint32_t lds_u32(const uint8_t *p) {
    return *reinterpret_cast<const uint32_t *>(p);
}

__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Device error codes written to an int status word by kernels with bounded waits.
enum : int {
    kDevOk = 0,
    kDevTimeoutTma = 1,   // a TMA bulk copy did not complete within the wait bound
    kDevBadStage = 2,     // a pass did not fit its shared-memory stage (host planning bug)
    kDevBadToken = 3,     // token id outside [0, vocab)
    kDevBadPosition = 4,  // position outside [0, max_seq)
    kDevBadExpert = 5,    // expert index outside [0, n_experts)
    kDevTimeoutPeer = 6,  // a peer rank's exchanged rows did not arrive within the bound
};

}  // namespace tqb200
