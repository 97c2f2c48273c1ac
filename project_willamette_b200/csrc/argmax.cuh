// argmax.cuh -- greedy argmax over a device logit vector.
//
// Reference: argmax (src/model/lm_head.rs:161-174): a strict '>' scan from
// index 0, so ties keep the lowest index and NaN never replaces the running
// best (a NaN at index 0 therefore wins).  Encoded as the maximum of
// (orderable(v) << 32) | (0xFFFFFFFF - i), see f32_order_key.
#pragma once

#include <cstdint>

#include "q6k_lmhead.cuh"  // f32_order_key
#include "wl_ptx.cuh"

namespace wl {

constexpr int ARGMAX_THREADS = 512;

__global__ void __launch_bounds__(ARGMAX_THREADS)
    argmax_kernel(const float *__restrict__ logits, uint32_t n,
                  unsigned long long *__restrict__ slot, uint32_t *__restrict__ counter,
                  uint32_t *__restrict__ out_id) {
    __shared__ unsigned long long cta_best;
    __shared__ uint32_t s_last;
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) cta_best = 0ull;
    __syncthreads();
    unsigned long long best = 0ull;
    for (uint32_t i = blockIdx.x * ARGMAX_THREADS + threadIdx.x; i < n;
         i += gridDim.x * ARGMAX_THREADS) {
        const unsigned long long key = ((unsigned long long)f32_order_key(logits[i], i) << 32) |
                                       (unsigned long long)(0xFFFFFFFFu - i);
        best = best > key ? best : key;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
        best = best > o ? best : o;
    }
    if ((threadIdx.x & 31) == 0) atomicMax(&cta_best, best);
    __syncthreads();
    if (threadIdx.x == 0) {
        atomicMax(slot, cta_best);
        __threadfence();
        s_last = atomicAdd(counter, 1u) == gridDim.x - 1 ? 1u : 0u;
        if (s_last) {
            __threadfence();
            const unsigned long long k = atomicExch(slot, 0ull);
            *out_id = 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
            *counter = 0u;
        }
    }
}

}  // namespace wl
