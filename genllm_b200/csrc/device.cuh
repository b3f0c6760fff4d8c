// device.cuh — sm_100a device helpers: mbarriers, TMA tensor loads, L2
// policies, bounded waits and the number-format conversions the path needs.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace gkv {

// Device error word bits (gkv_check_device_errors).
constexpr uint32_t kErrBadPage = 1u;
constexpr uint32_t kErrTimeout = 2u;

// A wait on an asynchronous copy gives up after this long (ns), records
// kErrTimeout and lets the kernel finish instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's generic-proxy shared-memory accesses before later
// async-proxy (TMA) accesses of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait for phase `parity` of `bar`, for at most kWaitLimitNs. Returns false
// on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// L2 policy for data read exactly once per step (the KV pages).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// L2 policy for data written now and read back soon by another CTA or
// kernel (split partials) while other traffic streams through L2.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void st_f32_hint(float* p, float v, uint64_t policy) {
    asm volatile("st.global.L2::cache_hint.f32 [%0], %1, %2;" ::"l"(p), "f"(v), "l"(policy) : "memory");
}

// Drop a 128-byte L2 line without writing it back (data read for the last
// time, e.g. split partials once merged).
__device__ __forceinline__ void l2_discard_line(const void* p) {
    asm volatile("discard.global.L2 [%0], 128;" ::"l"(p) : "memory");
}

// 3-D tiled TMA load (no multicast) completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2),
        "l"(policy)
        : "memory");
}

// 3-D tiled TMA prefetch of a box into L2 (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int32_t c0, int32_t c1, int32_t c2) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}

__device__ __forceinline__ float exp2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// bf16 pair (packed in a u32, low half first in memory) -> two floats.
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// fp32 -> bf16 bits with the reference's rounding (include/utils/bfloat16.hpp:
// 18-41): round to nearest even, exponent-0 inputs to signed zero, NaN keeps a
// single mantissa bit, overflow to infinity.
__device__ __forceinline__ uint16_t bf16_bits_ref(float f) {
    const uint32_t u = __float_as_uint(f);
    const uint32_t e = (u >> 23) & 0xFFu;
    const uint32_t sign = (u >> 16) & 0x8000u;
    if (e == 0xFFu) return static_cast<uint16_t>(sign | 0x7F80u | ((u & 0x7FFFFFu) ? 1u : 0u));
    if (e == 0) return static_cast<uint16_t>(sign);
    return static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// The same bits as bf16_bits_ref with fewer instructions: for normal fp32
// values the reference's rounding is round-to-nearest-even, which is the
// hardware conversion; zero exponents (flushed to a signed zero) and
// infinities / NaNs take the reference's path.
__device__ __forceinline__ uint16_t bf16_bits_ref_fast(float f) {
    const uint32_t u = __float_as_uint(f);
    const uint32_t e = u & 0x7F800000u;
    if (e == 0u || e == 0x7F800000u) return bf16_bits_ref(f);
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Store one fp32 output element in the requested dtype (reference codes).
__device__ __forceinline__ void store_out(void* out, size_t idx, float v, int dtype) {
    if (dtype == 0) {
        static_cast<float*>(out)[idx] = v;
    } else if (dtype == 30) {
        static_cast<uint16_t*>(out)[idx] = bf16_bits_ref(v);
    } else {
        static_cast<__half*>(out)[idx] = __float2half_rn(v);
    }
}

}  // namespace gkv
