// q8_0.cuh -- Q8_0 matvec / lm-head rows for sm_100a, bit-exact.
//
// Reference: q8_0_matvec_f32 (src/model/linear.rs:171-224) and the lm-head
// arm of compute_logits (src/model/lm_head.rs:103), both through
// q8_0::dot_row (src/model/q8_0.rs:50-70) -> dot_row_avx2
// (src/model/q8_0_simd.rs:72-104) on x86 hosts with AVX2.
//
// Per 32-value block the AVX2 kernel keeps 8 lanes,
//     s_j = (((0 + q_j x_j) + q_{8+j} x_{8+j}) + q_{16+j} x_{16+j}) + q_{24+j} x_{24+j},
// folds the halves h_i = s_i + s_{4+i}, reduces (h_0 + h_2) + (h_1 + h_3)
// (hsum_sse, q8_0_simd.rs:145-157) and adds d * that to a row total, blocks
// in order.  One thread computes one block's d * hsum with the same IEEE
// operations; one thread per row then adds the block terms in block order.
//
// Device layout (one-time repack): row = [q: K int8][d: K/32 f16][pad to 16 B].
#pragma once

#include <cstdint>

#include "q6k_lmhead.cuh"  // f16_bits_to_f32
#include "wl_ptx.cuh"

namespace wl {

constexpr int Q8_THREADS = 256;

__host__ __device__ constexpr uint32_t q8_row_stride(uint32_t K) {
    return K + (((K / 32u) * 2u + 15u) & ~15u);
}

__device__ __forceinline__ uint32_t q8_xpad(uint32_t i) { return i + (i >> 5) * 4u; }

__global__ void q8_0_repack_kernel(const uint8_t *__restrict__ raw, uint32_t K, uint32_t N,
                                   uint8_t *__restrict__ out) {
    const uint32_t nb = K / 32u, stride = q8_row_stride(K);
    const size_t total = (size_t)N * nb;
    for (size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (size_t)gridDim.x * blockDim.x) {
        const uint32_t row = (uint32_t)(t / nb), b = (uint32_t)(t % nb);
        const uint8_t *src = raw + ((size_t)row * nb + b) * 34u;
        uint8_t *dst = out + (size_t)row * stride;
        for (int i = 0; i < 32; ++i) dst[b * 32u + i] = src[2 + i];
        dst[K + 2u * b] = src[0];
        dst[K + 2u * b + 1] = src[1];
        if (b == 0)
            for (uint32_t i = K + 2u * nb; i < stride; ++i) dst[i] = 0;
    }
}

// y[N] = rows(packed) . x[K]; smem: padded x + block terms of one row tile.
__global__ void __launch_bounds__(Q8_THREADS)
    q8_0_matvec_kernel(const uint8_t *__restrict__ packed, uint32_t K, uint32_t N,
                       const float *__restrict__ x, float *__restrict__ y) {
    extern __shared__ __align__(16) float q8smem[];
    const uint32_t nb = K / 32u, stride = q8_row_stride(K);
    const uint32_t R = nb >= Q8_THREADS ? 1u : Q8_THREADS / nb;  // rows per tile
    float *xs = q8smem;
    float *terms = q8smem + K + K / 8u;

    pdl_launch_dependents();
    pdl_wait();
    for (uint32_t i = threadIdx.x; i < K; i += Q8_THREADS) xs[q8_xpad(i)] = x[i];
    __syncthreads();

    for (uint32_t r = blockIdx.x * R; r < N; r += gridDim.x * R) {
        for (uint32_t t = threadIdx.x; t < R * nb; t += Q8_THREADS) {
            const uint32_t row = r + t / nb, b = t % nb;
            if (row >= N) continue;
            const uint8_t *rp = packed + (size_t)row * stride;
            const uint4 v0 = __ldg(reinterpret_cast<const uint4 *>(rp + 32u * b));
            const uint4 v1 = __ldg(reinterpret_cast<const uint4 *>(rp + 32u * b + 16u));
            const uint32_t words[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
            const float *xb = xs + q8_xpad(32u * b);  // 32 contiguous floats
            float s[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) s[j] = 0.0f;
#pragma unroll
            for (int off = 0; off < 32; off += 8) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int e = off + j;
                    const int qv = (int)(int8_t)((words[e >> 2] >> (8 * (e & 3))) & 0xFFu);
                    s[j] = __fadd_rn(s[j], __fmul_rn((float)qv, xb[e]));
                }
            }
            float h[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) h[i] = __fadd_rn(s[i], s[4 + i]);
            const float hs = __fadd_rn(__fadd_rn(h[0], h[2]), __fadd_rn(h[1], h[3]));
            const uint32_t dbits = (uint32_t)rp[K + 2u * b] | ((uint32_t)rp[K + 2u * b + 1] << 8);
            terms[t] = __fmul_rn(f16_bits_to_f32(dbits), hs);
        }
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < R; i += Q8_THREADS) {
            const uint32_t row = r + i;
            if (row >= N) continue;
            float total = 0.0f;
            for (uint32_t b = 0; b < nb; ++b) total = __fadd_rn(total, terms[i * nb + b]);
            y[row] = total;
        }
        __syncthreads();
    }
}

}  // namespace wl
