// exact_sum.cuh -- the reference's sequential f32 sum of non-negative values,
// bit for bit, by a whole CTA.
//
// The reference adds in index order: s = 0; for i: s = RN(s + a[i]) (the
// RMSNorm sum of squares, primitives.rs:227-254; the softmax denominator,
// attention.rs:45-73).  One thread doing that is bound by the add's latency
// (about 4.3 cycles per element on sm_100a: 15 us for a 6912-element FFN
// sub-norm).  For a[i] >= 0 the partial sums never decrease, and while s
// stays in one binade [2^e, 2^(e+1)) every add rounds to the same grid of
// step u = 2^(e-23): RN(s + a) = s + u * round(a / u) exactly, unless
// a / u sits exactly half-way (then the tie goes to the even result, which
// depends on s) or the sum leaves the binade.  The increments round(a / u)
// are integers that do not depend on s, so their sums can be formed in
// parallel and added to s's bit pattern in one step.
//
// The CTA splits the values into one contiguous chunk per thread (at most
// 32 values, held in registers) and
//   1. guesses each chunk's binade from a prefix sum of the chunk totals (a
//      guess only: nothing below relies on it being right);
//   2. for a chunk whose guessed binade holds over the whole chunk (with a
//      margin), sums its increments D; a chunk with a tie, a value of the
//      binade or above, a negative / inf / NaN value, or no usable guess is
//      marked sequential;
//   3. merges, within each warp, consecutive chunks with the same binade
//      into runs (a segmented scan of D) and lists the runs in order;
//   4. one thread walks the list.  A run is applied in one integer add when
//      the running sum s really is in the run's binade and mantissa(s) + D
//      stays below 2^23: every partial sum of the run then lies in
//      [s, s + D u] inside the binade, so every add rounded to step u and
//      the result is exactly s + D u.  Otherwise (a wrong guess, a marked
//      chunk, s = 0 at the start) the run's values are added one by one
//      with IEEE adds.  Either way the result is the sequential sum's.
#pragma once

#include <cstdint>

#include "wl_ptx.cuh"

namespace wl {

constexpr uint32_t EXACT_SUM_MAX_CHUNK = 32;  // values per thread held in registers
// Below this many values one thread adding them in order is faster: the walk
// costs about 100-200 cycles per run (a dependent chain of loads, compares
// and branches), about 30 runs for a sum of squares of 2560 normal values
// (measured on sm_100a with 256 threads: 10,900 cycles either way at 2560,
// 15,600 against 29,400 at 6912).
constexpr uint32_t EXACT_SUM_PAR_MIN = 4096;

// Shared scratch: warp totals (float [32]), warp run counts (uint32 [32]),
// the run list (uint2 [nt]).
__host__ __device__ constexpr uint32_t exact_sum_scratch_bytes(uint32_t nt) {
    return 256u + 8u * nt;
}

// s + a[0] + ... + a[n-1], one IEEE add at a time, by one thread; the loads
// of the next block of 8 are in flight while a block is added (a block is
// padded with +0, which leaves any s unchanged: s starts at +0 and an IEEE
// round-to-nearest sum is -0 only when both operands are -0).
__device__ __forceinline__ float seq_sum_from(float s, const float *a, uint32_t n) {
    float nx[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) nx[k] = (uint32_t)k < n ? a[k] : 0.0f;
    for (uint32_t i = 0; i < n; i += 8u) {
        float cur[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) cur[k] = nx[k];
        if (i + 8u < n) {
#pragma unroll
            for (int k = 0; k < 8; ++k) nx[k] = i + 8u + k < n ? a[i + 8u + k] : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) s = __fadd_rn(s, cur[k]);
    }
    return s;
}

// The sequential sum of a[0..n) (shared memory), returned to every thread
// of the CTA.  Every thread must call it; blockDim.x a multiple of 32, at
// most 1024; scratch: exact_sum_scratch_bytes(blockDim.x) bytes of shared
// memory, 8-byte aligned, not overlapping a.  Exact for any input; fast
// when the values are non-negative and finite.  n < EXACT_SUM_PAR_MIN or
// n > 32 * blockDim.x: one thread adds them all.
__device__ __forceinline__ float cta_exact_sum_nonneg(const float *a, uint32_t n, uint8_t *scratch) {
    const uint32_t tid = threadIdx.x, nt = blockDim.x, lane = tid & 31u, w = tid >> 5;
    float *wtot = reinterpret_cast<float *>(scratch);
    uint32_t *wcnt = reinterpret_cast<uint32_t *>(scratch + 128);
    uint2 *runs = reinterpret_cast<uint2 *>(scratch + 256);
    if (n == 0u) return 0.0f;
    if (n < EXACT_SUM_PAR_MIN || n > EXACT_SUM_MAX_CHUNK * nt) {
        if (tid == 0) wtot[0] = seq_sum(a, n);
        __syncthreads();
        const float r = wtot[0];
        __syncthreads();
        return r;
    }
    const uint32_t L = (n + nt - 1u) / nt, nch = (n + L - 1u) / L;  // chunks >= nch are empty
    const uint32_t c0 = min(n, tid * L), len = min(n, c0 + L) - c0;

    // 1. the chunk in registers, its total (for the guess) and the values
    //    the integer path does not take: sign bit set, inf, NaN
    float v[EXACT_SUM_MAX_CHUNK];
    float cs = 0.0f;
    bool seq = false;
#pragma unroll
    for (uint32_t k = 0; k < EXACT_SUM_MAX_CHUNK; ++k) {
        if (k >= L) break;
        v[k] = k < len ? a[c0 + k] : 0.0f;
    }
#pragma unroll
    for (uint32_t k = 0; k < EXACT_SUM_MAX_CHUNK; ++k) {
        if (k >= L) break;
        seq |= (__float_as_uint(v[k]) >> 23) >= 0xFFu;
        cs += v[k];
    }
    float inc = cs;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= (uint32_t)off) inc += y;
    }
    if (lane == 31u) wtot[w] = inc;
    __syncthreads();
    float p0 = inc - cs;
    for (uint32_t k = 0; k < w; ++k) p0 += wtot[k];

    // 2. the binade guess and the chunk's increments in its units
    uint32_t es = 0, D = 0;
    if (!seq && len > 0u && p0 > 0.0f) {
        const uint32_t ea = __float_as_uint(p0 * (1.0f - 0x1p-10f)) >> 23;
        const uint32_t eb = __float_as_uint((p0 + cs) * (1.0f + 0x1p-10f)) >> 23;
        seq = ea != eb || ea < 1u || ea > 254u;
        es = ea;
#pragma unroll
        for (uint32_t k = 0; k < EXACT_SUM_MAX_CHUNK; ++k) {
            if (k >= L) break;
            const uint32_t b = __float_as_uint(v[k]), e = b >> 23;
            const uint32_t m = e ? ((b & 0x7FFFFFu) | 0x800000u) : b;  // v = m * 2^(max(e,1) - 150)
            const int32_t sh = (int32_t)es - (int32_t)(e ? e : 1u);   // v / u = m / 2^sh
            if (sh < 1) {
                seq = seq || k < len;  // a value of s's binade or above leaves the binade
            } else if (sh < 32) {
                const uint32_t half = 1u << (sh - 1), r = m & ((half << 1) - 1u);
                seq = seq || r == half;  // a tie: the rounding depends on s
                D += (m >> sh) + (r > half ? 1u : 0u);
            }
        }
        seq = seq || D >= 0x800000u;
    } else {
        seq = true;
    }
    if (seq) es = 0;

    // 3. runs: consecutive chunks of one warp with the same binade (a
    //    sequential chunk is a run of its own), listed in order; record =
    //    (last chunk | binade << 16, total increment)
    const uint32_t prev = __shfl_up_sync(0xffffffffu, es, 1);
    const bool head = lane == 0u || es == 0u || prev == 0u || prev != es;
    const uint32_t heads = __ballot_sync(0xffffffffu, head);
    const uint32_t seg = 31u - __clz(heads & (0xFFFFFFFFu >> (31u - lane)));
    uint32_t run = D;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, run, off);
        if (lane >= seg + (uint32_t)off) run += y;
    }
    const bool tail = tid < nch && (lane == 31u || tid + 1u == nch || ((heads >> (lane + 1u)) & 1u));
    const uint32_t tails = __ballot_sync(0xffffffffu, tail);
    if (lane == 0u) wcnt[w] = __popc(tails);
    __syncthreads();
    if (tail) {
        uint32_t idx = __popc(tails & ((1u << lane) - 1u));
        for (uint32_t k = 0; k < w; ++k) idx += wcnt[k];
        runs[idx] = make_uint2(tid | (es << 16), run);
    }
    __syncthreads();

    // 4. one thread applies the runs in order
    if (tid == 0) {
        uint32_t nruns = 0;
        for (uint32_t k = 0; k < nt / 32u; ++k) nruns += wcnt[k];
        float s = 0.0f;
        uint32_t start = 0;
        uint2 nx = runs[0];
        for (uint32_t r = 0; r < nruns; ++r) {
            const uint2 cur = nx;
            if (r + 1u < nruns) nx = runs[r + 1u];
            const uint32_t last = cur.x & 0xFFFFu, e = cur.x >> 16, sb = __float_as_uint(s);
            if (e != 0u && (sb >> 23) == e && (sb & 0x7FFFFFu) + cur.y < 0x800000u) {
                s = __uint_as_float(sb + cur.y);
            } else {
                const uint32_t i0 = start * L;
                s = seq_sum_from(s, a + i0, min(n, (last + 1u) * L) - i0);
            }
            start = last + 1u;
        }
        wtot[0] = s;
    }
    __syncthreads();
    const float r = wtot[0];
    __syncthreads();  // the scratch may be reused after the return
    return r;
}

// The same, as a called function: a kernel whose main loop needs its
// registers calls this instead of inlining the sum.
__device__ __noinline__ float cta_exact_sum_nonneg_call(const float *a, uint32_t n, uint8_t *scratch) {
    return cta_exact_sum_nonneg(a, n, scratch);
}

}  // namespace wl
