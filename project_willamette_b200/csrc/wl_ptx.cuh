// wl_ptx.cuh -- inline-PTX helpers for sm_100a: mbarriers, 1-D bulk async
// copies (TMA engine, global -> this CTA's shared memory), programmatic
// dependent launch, and bounded waits.
//
// Every wait in this library is bounded by g_wait_limit_ns of %globaltimer
// (2 s unless wl_set_wait_limit_ns changed it on this device); a wait that
// runs out returns false and the caller records WL_DEV_ERR_TIMEOUT in the
// library's device status word instead of hanging.
#pragma once

#include <cstdint>

namespace wl {

constexpr uint64_t WL_WAIT_LIMIT_DEFAULT_NS = 2000000000ull;  // 2 s
constexpr uint32_t WL_DEV_ERR_TIMEOUT = 1u;

// The limit of every bounded wait, one copy per device (set from the host by
// wl_set_wait_limit_ns).  Read once when a wait starts to spin.
__device__ uint64_t g_wait_limit_ns = WL_WAIT_LIMIT_DEFAULT_NS;
__device__ __forceinline__ uint64_t wait_limit_ns() {
    return *reinterpret_cast<volatile const uint64_t *>(&g_wait_limit_ns);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

// Wait for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns(), limit = wait_limit_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > limit) return false;
    }
    return true;
}

// 1-D bulk copy of `bytes` (multiple of 16) from global memory into this
// CTA's shared memory; both addresses 16-byte aligned.  Completion is
// counted as transaction bytes on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same, with an L2 eviction-priority hint (weights streamed once).
__device__ __forceinline__ void bulk_g2s_evict_first(void *dst_smem, const void *src_gmem,
                                                     uint32_t bytes, uint64_t *bar,
                                                     uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch: let the next kernel in the stream start
// its prologue now / wait until the previous kernel's writes are visible.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint4 lds128(const void *p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}

// t[0] + t[1] + ... + t[n-1] added in that order from +0, one rounding per
// add (the reference's sequential loops, bit for bit).  A plain loop unrolled
// 128 times: the compiler then issues the loads far enough ahead of the
// dependent adds that the loop runs at about 4.25 cycles per element on
// sm_100a (a hand-written 32-element prefetch of float4 loads ran at 6.5).
__device__ __forceinline__ float seq_sum(const float *t, uint32_t n) {
    float s = 0.0f;
#pragma unroll 128
    for (uint32_t i = 0; i < n; ++i) s = __fadd_rn(s, t[i]);
    return s;
}

// Sum of x[i] * x[i] for i = 0, 1, ..., n - 1 in that order, one rounding per
// product and per add (the reference's sequential RMSNorm loop, bit for bit),
// by one thread.  A CTA that can spare the threads squares the elements in
// parallel first and calls seq_sum (a multiply in the dependent loop costs
// about twice the add's latency per element).  x 16-byte aligned.
__device__ __forceinline__ float seq_sum_sq(const float *x, uint32_t n) {
    float t = 0.0f;
    const uint32_t n4 = (n & ~31u) / 4u;  // float4s in whole groups of 32 elements
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    if (n4) {
        float4 nxt[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) nxt[j] = x4[j];
        for (uint32_t i = 0; i < n4; i += 8) {
            float4 cur[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
            if (i + 8 < n4) {
#pragma unroll
                for (int j = 0; j < 8; ++j) nxt[j] = x4[i + 8 + j];
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                t = __fadd_rn(t, __fmul_rn(cur[j].x, cur[j].x));
                t = __fadd_rn(t, __fmul_rn(cur[j].y, cur[j].y));
                t = __fadd_rn(t, __fmul_rn(cur[j].z, cur[j].z));
                t = __fadd_rn(t, __fmul_rn(cur[j].w, cur[j].w));
            }
        }
    }
    for (uint32_t i = n4 * 4u; i < n; ++i) t = __fadd_rn(t, __fmul_rn(x[i], x[i]));
    return t;
}

// Activation quantiser rounding: round(v) half away from zero, clamped to
// [-127, 127], NaN -> 0 -- Rust's f32::round, then the clamp and saturating
// `as i8` of the reference's absmax quantiser.  Exact, and without the slow
// round/convert instructions: for a = min(|v|, 127), b = a + 0.5 rounded
// toward zero has floor(b) = floor(a + 0.5) (every integer below 128 is a
// float, so truncation cannot step over one), and b + 2^23 rounded toward
// zero lies in [2^23, 2^23 + 128), where floats are the integers, so its
// low bits are floor(b).
__device__ __forceinline__ int quant_round_i8(float v) {
    const float a = fminf(fabsf(v), 127.0f);
    const int qa =
        (int)(__float_as_uint(__fadd_rz(__fadd_rz(a, 0.5f), 8388608.0f)) - 0x4B000000u);
    return v > 0.0f ? qa : (v < 0.0f ? -qa : 0);  // NaN fails both tests -> 0
}

// Four quantised values (low bytes of q0..q3) packed into one word, q0 lowest.
__device__ __forceinline__ uint32_t pack_i8x4(int q0, int q1, int q2, int q3) {
    return __byte_perm(__byte_perm((uint32_t)q0, (uint32_t)q1, 0x0040u),
                       __byte_perm((uint32_t)q2, (uint32_t)q3, 0x0040u), 0x5410u);
}

// Packed f32 pairs (sm_100a): one instruction, each lane rounded to nearest
// as the scalar mul.rn / add.rn.  A packed multiply whose result feeds a
// packed add can still be fused into one FMA by the assembler (one rounding
// instead of two), so code that must keep two roundings uses these only where
// no add consumes a product, and keeps scalar mul.rn / add.rn there.
__device__ __forceinline__ float2 f2_mul_rn(float2 a, float2 b) {
    float2 d;
    asm("{.reg .b64 a, b, d;\n\t"
        "mov.b64 a, {%2, %3};\n\t"
        "mov.b64 b, {%4, %5};\n\t"
        "mul.rn.f32x2 d, a, b;\n\t"
        "mov.b64 {%0, %1}, d;}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 f2_fma_rn(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{.reg .b64 a, b, c, d;\n\t"
        "mov.b64 a, {%2, %3};\n\t"
        "mov.b64 b, {%4, %5};\n\t"
        "mov.b64 c, {%6, %7};\n\t"
        "fma.rn.f32x2 d, a, b, c;\n\t"
        "mov.b64 {%0, %1}, d;}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 f2_add_rn(float2 a, float2 b) {
    float2 d;
    asm("{.reg .b64 a, b, d;\n\t"
        "mov.b64 a, {%2, %3};\n\t"
        "mov.b64 b, {%4, %5};\n\t"
        "add.rn.f32x2 d, a, b;\n\t"
        "mov.b64 {%0, %1}, d;}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

}  // namespace wl
