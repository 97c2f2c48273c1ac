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
//      marked sequential.  a / u = a * 2^(150-e) is a power-of-two scaling
//      (exact, or below 2^-100 where it underflows), so round(a / u) is one
//      rint and a tie is |t - rint(t)| = 0.5;
//   3. merges, within each warp, consecutive chunks with the same binade
//      into runs (a segmented scan of D) and lists the runs in order;
//   4. one thread walks the runs.  A run is applied in one integer add when
//      the running sum s really is in the run's binade and mantissa(s) + D
//      stays below 2^23: every partial sum of the run then lies in
//      [s, s + D u] inside the binade, so every add rounded to step u and
//      the result is exactly s + D u.  Otherwise (a wrong guess, a marked
//      chunk, s = 0 at the start) the run's values are added one by one
//      with IEEE adds.  Either way the result is the sequential sum's.
// What stays serial is one chunk of IEEE adds per binade the sum crosses and
// about one integer add per warp.
#pragma once

#include <cstdint>

#include "wl_ptx.cuh"

namespace wl {

constexpr uint32_t EXACT_SUM_MAX_CHUNK = 32;  // values per thread held in registers
// Below this many values one thread adding them in order is faster: the
// phases cost about 3,000 cycles and the walk about 40 cycles per integer
// run and 100-250 per sequential chunk, about 30 runs for a sum of squares
// of normal values (measured on sm_100a with 256 threads: 6,300 against
// 4,500 cycles at 1024 values, 7,600 against 11,000 at 2560, 9,300 against
// 29,400 at 6912).
constexpr uint32_t EXACT_SUM_PAR_MIN = 2048;

// Shared scratch: warp totals (float [32]), warp run counts (uint32 [32]),
// the run list (uint2 [nt]).
__host__ __device__ constexpr uint32_t exact_sum_scratch_bytes(uint32_t nt) {
    return 256u + 8u * nt;
}

// s + a[0] + ... + a[c-1] for c <= W, one IEEE add at a time, by one
// thread: all W loads issued first, then W adds, the values past c read as
// +0 (which leaves any s unchanged: s starts at +0 and an IEEE
// round-to-nearest sum is -0 only when both operands are -0).
template <uint32_t W>
__device__ __forceinline__ float seq_sum_w(float s, const float *a, uint32_t c) {
    float v[W];
#pragma unroll
    for (uint32_t k = 0; k < W; ++k) v[k] = k < c ? a[k] : 0.0f;
#pragma unroll
    for (uint32_t k = 0; k < W; ++k) s = __fadd_rn(s, v[k]);
    return s;
}

// The same for c <= 32, at the narrowest of 8 / 16 / 32 adds.
__device__ __forceinline__ float seq_sum_small(float s, const float *a, uint32_t c) {
    if (c <= 8u) return seq_sum_w<8>(s, a, c);
    if (c <= 16u) return seq_sum_w<16>(s, a, c);
    return seq_sum_w<32>(s, a, c);
}

// s + a[0] + ... + a[n-1] in order, any n.
__device__ __forceinline__ float seq_sum_from(float s, const float *a, uint32_t n) {
    for (uint32_t i = 0; i < n; i += 32u) s = seq_sum_small(s, a + i, min(32u, n - i));
    return s;
}

// s + a[0] + ... + a[c-1] for c <= W, c a multiple of 4, a 16-byte aligned:
// c / 4 vector loads, then W adds (+0 past c; none when c = W).  One thread issues about one
// instruction every 2-3 cycles here, so the walk below is bound by its
// instruction count: a scalar load, its guard and its add per value cost
// about 20 cycles per value, this about 5.
template <uint32_t W>
__device__ __forceinline__ float seq_sum_v4(float s, const float *a, uint32_t c) {
    float v[W];
#pragma unroll
    for (uint32_t j = 0; j < W / 4u; ++j) {
        const float4 q = 4u * j < c ? *reinterpret_cast<const float4 *>(a + 4u * j)
                                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        v[4u * j] = q.x;
        v[4u * j + 1u] = q.y;
        v[4u * j + 2u] = q.z;
        v[4u * j + 3u] = q.w;
    }
#pragma unroll
    for (uint32_t k = 0; k < W; ++k) s = __fadd_rn(s, v[k]);
    return s;
}

// Step 4 below: one thread applies the run list in order.  Chunks are LC
// values (a multiple of 4, at most 32) starting at multiples of LC; a
// sequential record of one whole chunk is LC / 4 vector loads and LC adds.
template <uint32_t LC>
__device__ __forceinline__ float exact_sum_walk(const float *a, uint32_t n, const uint2 *runs,
                                                uint32_t nruns) {
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
            const uint32_t i0 = start * LC, cnt = min(n, (last + 1u) * LC) - i0;
            s = cnt == LC ? seq_sum_v4<LC>(s, a + i0, LC) : seq_sum_from(s, a + i0, cnt);
        }
        start = last + 1u;
    }
    return s;
}

// Exclusive prefix over warps of one value per warp (v[0..nw), shared
// memory), for warp w, by a shuffle scan in every warp; *total = the sum.
template <typename T>
__device__ __forceinline__ T warp_prefix_of(const T *v, uint32_t nw, uint32_t w, uint32_t lane, T *total) {
    const T x = lane < nw ? v[lane] : T(0);
    T inc = x;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const T y = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= (uint32_t)off) inc += y;
    }
    *total = __shfl_sync(0xffffffffu, inc, 31);
    return __shfl_sync(0xffffffffu, inc - x, w);
}

// The sequential sum of a[0..n) (shared memory), returned to every thread
// of the CTA.  Every thread must call it; blockDim.x a multiple of 32, at
// most 1024; scratch: exact_sum_scratch_bytes(blockDim.x) bytes of shared
// memory, 8-byte aligned, not overlapping a.  Exact for any input; fast
// when the values are non-negative and finite.  n < EXACT_SUM_PAR_MIN,
// n > 32 * blockDim.x or a not 16-byte aligned: one thread adds them all.
__device__ __forceinline__ float cta_exact_sum_nonneg(const float *a, uint32_t n, uint8_t *scratch) {
    const uint32_t tid = threadIdx.x, nt = blockDim.x, lane = tid & 31u, w = tid >> 5;
    float *wtot = reinterpret_cast<float *>(scratch);
    uint32_t *wcnt = reinterpret_cast<uint32_t *>(scratch + 128);
    uint2 *runs = reinterpret_cast<uint2 *>(scratch + 256);
    if (n == 0u) return 0.0f;
    // chunks of L values, L a multiple of 4: a whole chunk is L / 4 vectors
    const uint32_t L = ((n + nt - 1u) / nt + 3u) & ~3u;
    if (n < EXACT_SUM_PAR_MIN || L > EXACT_SUM_MAX_CHUNK || (reinterpret_cast<uintptr_t>(a) & 15u)) {
        if (tid == 0) wtot[0] = seq_sum(a, n);
        __syncthreads();
        const float r = wtot[0];
        __syncthreads();
        return r;
    }
    const uint32_t nch = (n + L - 1u) / L;  // chunks >= nch are empty
    const uint32_t c0 = min(n, tid * L), len = min(n, c0 + L) - c0;

    // 1. the chunk in registers, its total (for the guess) and the values
    //    the integer path does not take: sign bit set, inf, NaN
    float v[EXACT_SUM_MAX_CHUNK];
    float cs = 0.0f;
    bool seq = false;
    if (len == L) {
#pragma unroll
        for (uint32_t j = 0; j < EXACT_SUM_MAX_CHUNK / 4u; ++j) {
            if (4u * j >= L) break;
            const float4 q = *reinterpret_cast<const float4 *>(a + c0 + 4u * j);
            v[4u * j] = q.x;
            v[4u * j + 1u] = q.y;
            v[4u * j + 2u] = q.z;
            v[4u * j + 3u] = q.w;
        }
    } else {
#pragma unroll
        for (uint32_t k = 0; k < EXACT_SUM_MAX_CHUNK; ++k) {
            if (k >= L) break;
            v[k] = k < len ? a[c0 + k] : 0.0f;
        }
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
    float ftot;
    const float p0 = (inc - cs) + warp_prefix_of(wtot, nt / 32u, w, lane, &ftot);

    // 2. the binade guess and the chunk's increments in its units
    uint32_t es = 0, D = 0;
    if (!seq && len > 0u && p0 > 0.0f) {
        const uint32_t ea = __float_as_uint(p0 * (1.0f - 0x1p-10f)) >> 23;
        const uint32_t eb = __float_as_uint((p0 + cs) * (1.0f + 0x1p-10f)) >> 23;
        // ea >= 23 keeps the scale 2^(150-ea) a normal float
        seq = ea != eb || ea < 23u || ea > 254u;
        es = ea;
        const float scale = __uint_as_float((277u - min(max(ea, 23u), 254u)) << 23);
        float Df = 0.0f, tmax = 0.0f;
        bool tie = false;
#pragma unroll
        for (uint32_t k = 0; k < EXACT_SUM_MAX_CHUNK; ++k) {
            if (k >= L) break;
            const float t = __fmul_rn(v[k], scale);  // a / u (values past len are +0)
            const float r = rintf(t);
            tie = tie || fabsf(__fsub_rn(t, r)) == 0.5f;
            Df = __fadd_rn(Df, r);  // integers below 2^24 add exactly
            tmax = fmaxf(tmax, t);
        }
        // a value of s's binade or above (t >= 2^23) leaves the binade
        seq = seq || tie || tmax >= 0x1p23f || Df >= 0x1p23f;
        D = seq ? 0u : (uint32_t)Df;
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
    uint32_t nruns;
    const uint32_t base = warp_prefix_of(wcnt, nt / 32u, w, lane, &nruns);
    if (tail) runs[base + __popc(tails & ((1u << lane) - 1u))] = make_uint2(tid | (es << 16), run);
    __syncthreads();

    // 4. one thread applies the runs in order
    if (tid == 0) {
        float s;
        switch (L >> 2) {
        case 1: s = exact_sum_walk<4>(a, n, runs, nruns); break;
        case 2: s = exact_sum_walk<8>(a, n, runs, nruns); break;
        case 3: s = exact_sum_walk<12>(a, n, runs, nruns); break;
        case 4: s = exact_sum_walk<16>(a, n, runs, nruns); break;
        case 5: s = exact_sum_walk<20>(a, n, runs, nruns); break;
        case 6: s = exact_sum_walk<24>(a, n, runs, nruns); break;
        case 7: s = exact_sum_walk<28>(a, n, runs, nruns); break;
        default: s = exact_sum_walk<32>(a, n, runs, nruns); break;
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
