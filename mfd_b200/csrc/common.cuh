// common.cuh -- shared device helpers for the MFD verify-step kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mfd_b200.h"

#define MFD_FULL_MASK 0xffffffffu

namespace mfd {

// Records a human-readable message for mfd_last_error(); defined in capi.cu.
void set_error(const char* fmt, ...);

// ------------------------------------------------------------------ orderable keys
// A float mapped to a uint32 whose unsigned order equals the float order (-inf < ... < +inf < NaN);
// NaN is canonicalised to the positive quiet NaN first, so every NaN sorts above +inf as torch.topk has it,
// and -0.0 to +0.0, which compare equal as values (ties between them fall to the index).
__device__ __forceinline__ uint32_t ord_f32(float v) {
    uint32_t b = __float_as_uint(v);
    if ((b & 0x7fffffffu) > 0x7f800000u) b = 0x7fc00000u;
    if (b == 0x80000000u) b = 0u;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unord_f32(uint32_t o) {
    uint32_t b = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
    return __uint_as_float(b);
}
// Top-k key: larger value first, equal values by lower index first.
__device__ __forceinline__ uint64_t topk_key(float v, uint32_t idx) {
    return ((uint64_t)ord_f32(v) << 32) | (uint64_t)(~idx);
}
__device__ __forceinline__ float key_value(uint64_t k) { return unord_f32((uint32_t)(k >> 32)); }
__device__ __forceinline__ uint32_t key_index(uint64_t k) { return ~(uint32_t)k; }

// double -> uint64 with the same order (finite and infinite values)
__device__ __forceinline__ uint64_t ord_f64(double v) {
    uint64_t b = (uint64_t)__double_as_longlong(v);
    return (b & 0x8000000000000000ull) ? ~b : (b | 0x8000000000000000ull);
}

// ------------------------------------------------------------------ loads
__device__ __forceinline__ float4 ldg_stream_f4(const void* p) {
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float bf16_at(const uint16_t* p) { return __uint_as_float((uint32_t)(*p) << 16); }

// hardware base-2 exponential (MUFU); relative error about 2^-22
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr float kLog2e = 1.4426950408889634f;

// Packed float32 pairs (Blackwell f32x2 arithmetic): every lane of add / sub / mul / fma .rn.f32x2 is the IEEE
// round-to-nearest result of the scalar operation on that lane, with one instruction for both.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t dup2(float a) { return pk2(a, a); }
// three-input maximum (one instruction; the maximum is exact, so any grouping gives the same value)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
// the maximum over the 32 lanes of a full warp in one reduction
__device__ __forceinline__ float warp_max_f32(float v) {
    float d;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(d) : "f"(v));
    return d;
}

// ------------------------------------------------------------------ warp helpers
__device__ __forceinline__ uint64_t shfl_u64(uint64_t v, int src) {
    uint32_t lo = __shfl_sync(MFD_FULL_MASK, (uint32_t)v, src);
    uint32_t hi = __shfl_sync(MFD_FULL_MASK, (uint32_t)(v >> 32), src);
    return ((uint64_t)hi << 32) | lo;
}
__device__ __forceinline__ uint64_t shfl_xor_u64(uint64_t v, int m) {
    uint32_t lo = __shfl_xor_sync(MFD_FULL_MASK, (uint32_t)v, m);
    uint32_t hi = __shfl_xor_sync(MFD_FULL_MASK, (uint32_t)(v >> 32), m);
    return ((uint64_t)hi << 32) | lo;
}
__device__ __forceinline__ double shfl_f64(double v, int src) {
    return __longlong_as_double((long long)shfl_u64((uint64_t)__double_as_longlong(v), src));
}

// Warp min of a 64-bit key (all lanes receive it).
__device__ __forceinline__ uint64_t warp_min_u64(uint64_t v) {
    uint32_t hi = __reduce_min_sync(MFD_FULL_MASK, (uint32_t)(v >> 32));
    uint32_t lo = __reduce_min_sync(MFD_FULL_MASK, ((uint32_t)(v >> 32) == hi) ? (uint32_t)v : 0xffffffffu);
    return ((uint64_t)hi << 32) | lo;
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
    uint32_t hi = __reduce_max_sync(MFD_FULL_MASK, (uint32_t)(v >> 32));
    uint32_t lo = __reduce_max_sync(MFD_FULL_MASK, ((uint32_t)(v >> 32) == hi) ? (uint32_t)v : 0u);
    return ((uint64_t)hi << 32) | lo;
}

// ------------------------------------------------------------------ mbarrier + bulk async copy (no multicast)
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
// global -> this CTA's shared memory, completion counted on `bar`; src, dst 16-byte aligned, bytes % 16 == 0
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}
// order this thread's earlier generic-proxy shared-memory accesses before later async-proxy (bulk copy) ones
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Wait for phase `parity` of `bar` to complete, at most `max_tries` polls; false on timeout (the caller records
// an error status and stops instead of spinning forever).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t max_tries = (1u << 26)) {
    const uint32_t a = smem_addr(bar);
    for (uint32_t i = 0; i < max_tries; ++i) {
        uint32_t done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// SMs of the current device (host).
inline int current_sm_count() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

// online (max, sum of exp(x - max)) pair merge; -inf maxima carry a zero sum
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
    float mn = fmaxf(m, m2);
    if (mn == -INFINITY) { m = mn; s = 0.f; return; }
    s = s * fast_exp2((m - mn) * kLog2e) + s2 * fast_exp2((m2 - mn) * kLog2e);
    m = mn;
}

}  // namespace mfd

#define MFD_CHECK_LAUNCH(name)                                                  \
    do {                                                                        \
        cudaError_t _e = cudaGetLastError();                                    \
        if (_e != cudaSuccess) {                                                \
            mfd::set_error("%s: launch failed: %s", name, cudaGetErrorString(_e)); \
            return MFD_ERR_CUDA;                                                \
        }                                                                       \
    } while (0)
