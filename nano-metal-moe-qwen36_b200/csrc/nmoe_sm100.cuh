// nmoe_sm100.cuh -- sm_100a primitives used by the single-launch decode kernel:
// bulk async copies (TMA engine, non-tensor form) completing on mbarriers,
// release/acquire counters, bounded waits, bf16 tensor-core MMA.
#pragma once
#include <stdint.h>

#include "nmoe_common.cuh"

namespace nmoe {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint (ns): the thread sleeps in hardware until the phase
// completes or the hint expires, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Every wait loop is capped by an iteration count as well as by the deadline, so
// termination never depends on %globaltimer advancing.
constexpr uint32_t kMaxSpins = 1u << 22;

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t deadline) {
    for (uint32_t it = 0; !mbar_try_wait(bar, parity); ++it) {
        if (it >= kMaxSpins || globaltimer_ns() > deadline) return false;
        if (it > 32) __nanosleep(32);
    }
    return true;
}
// Sleeping wait for the grouped GEMM's role warps: each try suspends up to 20 us.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, uint64_t deadline) {
    for (uint32_t it = 0; !mbar_try_wait_sleep(bar, parity, 20000u); ++it)
        if (it >= (1u << 16) || globaltimer_ns() > deadline) return false;
    return true;
}
// Warp-uniform: all 32 lanes must call; all get the same answer.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity, uint64_t deadline) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, deadline));
}

__device__ __forceinline__ uint64_t policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Global -> shared bulk copy (no tensor map, no multicast). 16-byte aligned, size % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add_u32(uint32_t *p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ bool spin_until_geq(const uint32_t *p, uint32_t target, uint64_t deadline) {
    for (uint32_t it = 0; ld_acquire_u32(p) < target; ++it) {
        if (it >= kMaxSpins || globaltimer_ns() > deadline) return false;
        __nanosleep(32);
    }
    return true;
}

__device__ __forceinline__ uint4 lds128(const void *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ float4 lds128f(const float *p) { return *reinterpret_cast<const float4 *>(p); }

// D += A(16x16 bf16) * B(16x8 bf16), fp32 accumulate.
__device__ __forceinline__ void mma_bf16(float *d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two packed quantised values (v_i in the low half-word's field, v_{i+vpw/2} in the high
// one) as a bf16x2 pair of exact integers: OR the field into the mantissa of 128.0
// (0x4300), then subtract 128.
template <int kBits>
__device__ __forceinline__ uint32_t q_pair_bf16x2(uint32_t w, int i) {
    constexpr uint32_t mask = kBits == 4 ? 0x000F000Fu : 0x00030003u;
    const uint32_t v = ((w >> (kBits * i)) & mask) | 0x43004300u;
    uint32_t r;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(0x43004300u));
    return r;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float bf16_round(float v) { return __uint_as_float(pack_bf16x2(v, 0.f) << 16); }

__device__ __forceinline__ float bf16_dot8(const uint4 w, const float *xr) {
    float a = 0.f, b = 0.f;
    a = fmaf(bf16_lo(w.x), xr[0], a);
    b = fmaf(bf16_hi(w.x), xr[1], b);
    a = fmaf(bf16_lo(w.y), xr[2], a);
    b = fmaf(bf16_hi(w.y), xr[3], b);
    a = fmaf(bf16_lo(w.z), xr[4], a);
    b = fmaf(bf16_hi(w.z), xr[5], b);
    a = fmaf(bf16_lo(w.w), xr[6], a);
    b = fmaf(bf16_hi(w.w), xr[7], b);
    return a + b;
}

}  // namespace nmoe
