// i2s_f32act.cuh -- the reference's f32-activation I2_S matvec kernels.
//
// On x86-64 hosts with SSSE3 the reference's dispatch (bitlinear.rs:67-142,
// dispatch.rs:159-184) runs the int8-activation kernel (i2s_matvec.cuh).
// Three other kernels keep the activations in f32, with their own summation
// orders, and give different bits:
//   WL_I2S_KERNEL_SCALAR     bitlinear_i2s_matvec_f32_scalar (bitlinear.rs:146-242):
//       the fallback when no SIMD kernel is selected;
//   WL_I2S_KERNEL_SSE2_F32   bitlinear_i2s_matvec_f32_sse2 (bitlinear_sse2.rs:89-124,
//       block_accumulate :206-235, hsum_ps :249-255): the x86 kernel of a
//       build with --cfg willamette_sse2_f32 (bitlinear.rs:125-126);
//   WL_I2S_KERNEL_SCALAR_LUT bitlinear_i2s_matvec_f32_lut_scalar (bitlinear_lut.rs:59-131):
//       x86 hosts with SSE2 but not SSSE3.
// Each output row is one thread running that kernel's f32 chains in that
// kernel's order with IEEE round-to-nearest adds (no reassociation, no FMA),
// so every output is the reference's bits.  These arms exist so that a
// caller whose dispatch picks one of them gets its numbers, not the int8
// kernel's; they are correctness arms (the int8 kernel is the x86 default
// and the one tuned for bandwidth).
//
// Element order inside a 128-value block: byte gp holds the codes of elements
// gp, gp + 32, gp + 64, gp + 96 in bits 7:6, 5:4, 3:2, 1:0; code 0 -> -1,
// 1 -> 0, 2 -> +1, 3 -> 0.
#pragma once

#include <cstdint>

namespace wl {

constexpr uint32_t I2S_KERNEL_SCALAR = 0u;      // WL_I2S_KERNEL_SCALAR: Kernel::Scalar
constexpr uint32_t I2S_KERNEL_SCALAR_LUT = 3u;  // WL_I2S_KERNEL_SCALAR_LUT: Kernel::X86Sse2ScalarLut
constexpr uint32_t I2S_KERNEL_SSE2_F32 = 4u;    // WL_I2S_KERNEL_SSE2_F32: X86Sse2, --cfg willamette_sse2_f32
constexpr int I2S_F32ACT_THREADS = 64;

template <uint32_t MODE>
__global__ void __launch_bounds__(I2S_F32ACT_THREADS)
    i2s_f32act_kernel(const uint8_t *__restrict__ packed, float w_scale, uint32_t K, uint32_t N,
                      const float *__restrict__ x, float *__restrict__ y) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= N) return;
    const uint8_t *rp = packed + (size_t)row * (K / 4u);
    const uint32_t blocks = K / 128u;
    if constexpr (MODE == I2S_KERNEL_SCALAR) {
        // pos / neg: one chain each, elements in (block, byte, code) order
        float pos = 0.0f, neg = 0.0f;
        for (uint32_t bk = 0; bk < blocks; ++bk) {
            const float *xb = x + bk * 128u;
#pragma unroll 2
            for (uint32_t h = 0; h < 2; ++h) {
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(rp + bk * 32u + h * 16u));
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int gq = 0; gq < 16; ++gq) {
                    const uint32_t b = (w[gq >> 2] >> (8 * (gq & 3))) & 0xFFu;
                    const uint32_t gp = h * 16u + (uint32_t)gq;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t code = (b >> (6 - 2 * j)) & 3u;
                        const float xv = __ldg(xb + gp + 32u * (uint32_t)j);
                        if (code == 0u) neg = __fadd_rn(neg, xv);
                        else if (code == 2u) pos = __fadd_rn(pos, xv);
                    }
                }
            }
        }
        y[row] = __fmul_rn(w_scale, __fsub_rn(pos, neg));
    } else if constexpr (MODE == I2S_KERNEL_SSE2_F32) {
        // four lanes k of a pos and a neg vector: lane k takes the elements
        // 4c + k of each block, c = 0..31 in order (masked adds: +0 where the
        // code does not match, which leaves a chain that starts at +0 as is)
        float pos[4] = {0.0f, 0.0f, 0.0f, 0.0f}, neg[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (uint32_t bk = 0; bk < blocks; ++bk) {
            const float *xb = x + bk * 128u;
            const uint4 v0 = __ldg(reinterpret_cast<const uint4 *>(rp + bk * 32u));
            const uint4 v1 = __ldg(reinterpret_cast<const uint4 *>(rp + bk * 32u + 16u));
            const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const int j = c >> 3;  // element 4c + k = 32 j + gp, gp = 4 (c % 8) + k
                const float4 xv = __ldg(reinterpret_cast<const float4 *>(xb + 4 * c));
                const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
                const uint32_t word = w[c & 7];  // bytes gp = 4 (c % 8) .. +3
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t code = (word >> (8 * k + 6 - 2 * j)) & 3u;
                    if (code == 2u) pos[k] = __fadd_rn(pos[k], xs[k]);
                    else if (code == 0u) neg[k] = __fadd_rn(neg[k], xs[k]);
                }
            }
        }
        // hsum_ps: (v0 + v3) + (v2 + v1)
        const float hp = __fadd_rn(__fadd_rn(pos[0], pos[3]), __fadd_rn(pos[2], pos[1]));
        const float hn = __fadd_rn(__fadd_rn(neg[0], neg[3]), __fadd_rn(neg[2], neg[1]));
        y[row] = __fmul_rn(w_scale, __fsub_rn(hp, hn));
    } else {
        // LUT: per byte the table value ((t0 + t1) + t2) + t3 with t_j = -x, 0,
        // x, 0 for codes 0..3 of element gp + 32 j, added to y in byte order;
        // y * scale at the end
        float acc = 0.0f;
        for (uint32_t bk = 0; bk < blocks; ++bk) {
            const float *xb = x + bk * 128u;
#pragma unroll 2
            for (uint32_t h = 0; h < 2; ++h) {
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(rp + bk * 32u + h * 16u));
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int gq = 0; gq < 16; ++gq) {
                    const uint32_t b = (w[gq >> 2] >> (8 * (gq & 3))) & 0xFFu;
                    const uint32_t gp = h * 16u + (uint32_t)gq;
                    float t[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t code = (b >> (6 - 2 * j)) & 3u;
                        const float xv = __ldg(xb + gp + 32u * (uint32_t)j);
                        t[j] = code == 0u ? -xv : (code == 2u ? xv : 0.0f);
                    }
                    acc = __fadd_rn(acc, __fadd_rn(__fadd_rn(__fadd_rn(t[0], t[1]), t[2]), t[3]));
                }
            }
        }
        y[row] = __fmul_rn(acc, w_scale);
    }
}

}  // namespace wl
