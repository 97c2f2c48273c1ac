// exact_sum.cuh -- the reference's sequential f32 sum of non-negative terms,
// bit for bit, computed by a whole CTA instead of one thread.
//
// The reference adds the terms of its RMSNorm sum of squares
// (rms_norm_f32, primitives.rs:245-248) and of its softmax denominator
// (softmax_inplace, attention.rs:61-65) one after another:
//     s_0 = +0,  s_{i+1} = fl(s_i + t_i)      (round to nearest even)
// A dependent add costs about 4 cycles, so one thread needs ~28k cycles for
// a 6912-term sum.  For t_i >= 0 the running sum never decreases, which
// makes the rounding predictable:
//  * While s_i and s_{i+1} lie in one binade [2^E, 2^(E+1)) (or both below
//    2^-126, where the spacing is 2^-149), every float there is a multiple of
//    the spacing u, so fl(s_i + t_i) = s_i + u * round(t_i / u) -- an exact
//    integer step that does not depend on s_i, unless t_i / u is exactly
//    half-way between two integers (then the tie goes to the even result,
//    which does depend on s_i).
//  * Prefix sums P_i = t_0 + ... + t_{i-1}, computed here in f32 by a block
//    scan (relative error below 2^-17 for the sizes accepted), bound the
//    running sum: every add errs by at most half a spacing of its result, at
//    most 2^-24 s_i + 2^-150, and s never decreases, so |s_i - P_i| <
//    (i + 1)(2^-23 P_i + 2^-148).  With 2^-16 P_i more for the scan's own
//    error: when that interval around P_i and the one around P_{i+1} lie in
//    one binade, step i is such an integer step ("certain").
// So the CTA classifies every step in parallel, sums the integer steps of
// each run of certain steps in one binade with a block scan, turns every run
// into one addend (its steps times the spacing: exact) and every remaining
// step (binade crossings, ties, the first non-zero term) into its term, and
// one thread adds that short list in order -- the reference's additions at
// the remaining steps, exact additions for the runs.  The result is the
// sequential sum's bits.  Any negative or non-finite term, a total near the
// f32 range limit, or more list entries than the list holds, send the whole
// sum to one thread's sequential loop instead.
#pragma once

#include <cstdint>

#include "wl_ptx.cuh"

namespace wl {

constexpr int EXS_MAX_ENTRIES = 256;   // runs + single steps the walk can take
constexpr int EXS_MAX_PER_THREAD = 64; // terms per thread (n <= 64 * blockDim.x)
constexpr int EXS_U = -1000;           // entry kind: one step added as the reference does

struct ExactSumSmem {
    float wf[32];           // per-warp partial sums (block scans)
    long long wr[32];
    int wc[32];
    int last_key[512];      // last step's key of every thread (blockDim.x <= 512)
    int bad;
    float result;
    int e_idx[EXS_MAX_ENTRIES + 1];
    int e_key[EXS_MAX_ENTRIES + 1];
    long long e_c[EXS_MAX_ENTRIES + 1];  // sum of the integer steps before the entry
    __align__(16) float addend[EXS_MAX_ENTRIES];
};

// Binade exponent of v, or -127 for v < 2^-126 (the subnormal spacing).
__device__ __forceinline__ int exs_region(float v) {
    return v < 1.17549435e-38f ? -127 : (int)((__float_as_uint(v) >> 23) & 0xFFu) - 127;
}

// Step i in units of the spacing 2^ue of its binade: *r = round(t / 2^ue),
// or EXS_U when t / 2^ue is a tie (the even result depends on s_i) or too
// large to stay in a binade.  t >= +0, finite.
__device__ __forceinline__ int exs_step(float t, int ue, int *r) {
    const uint32_t tb = __float_as_uint(t);
    const uint32_t be = tb >> 23;
    const uint32_t m = be ? ((tb & 0x7FFFFFu) | 0x800000u) : tb;
    const int et = be ? (int)be - 127 : -126;
    const int d = ue - et + 23;  // t / 2^ue = m * 2^-d
    if (d <= 0) {
        if (m == 0) { *r = 0; return ue; }
        if (-d > 7) return EXS_U;  // a step of 2^31 spacings cannot stay in a binade
        *r = (int)(m << (-d));
        return ue;
    }
    if (d > 30) { *r = 0; return ue; }  // below half a spacing (m < 2^24 <= 2^(d-1))
    const uint32_t half = 1u << (d - 1), rem = m & ((half << 1) - 1u);
    if (rem == half) return EXS_U;
    *r = (int)((m >> d) + (rem > half ? 1u : 0u));
    return ue;
}

// The binade of every s in [lo, hi] when lo and hi share one, as the
// spacing exponent; EXS_U otherwise.  P0 <= P1 are prefix sums around which
// the running sum can deviate by the margin of the step index i (its bound,
// plus 2^-16 P for the prefix sums' own rounding).
__device__ __forceinline__ int exs_binade(float P0, float P1, uint32_t i) {
    const float fi = (float)i;
    const float lo = P0 - ((fi + 1.0f) * 1.1920929e-7f + 1.52587891e-5f) * P0 - (fi + 1.0f) * 3.5e-45f;
    const float hi = P1 + ((fi + 2.0f) * 1.1920929e-7f + 1.52587891e-5f) * P1 + (fi + 2.0f) * 3.5e-45f;
    const int E = exs_region(lo);
    if (E != exs_region(hi)) return EXS_U;
    return E == -127 ? -149 : E - 23;
}

// Step classification: key = spacing exponent (-149 .. 104) of a certain
// step's binade, EXS_U for a step the walk adds itself; r = the step in units
// of the spacing (certain steps).  P, Pn: prefix sums before and after t.
__device__ __forceinline__ int exs_classify(float P, float Pn, float t, uint32_t i, int *r) {
    const int ue = exs_binade(P, Pn, i);
    if (ue == EXS_U) return EXS_U;  // may cross a binade boundary
    return exs_step(t, ue, r);
}

// Inclusive block scans (blockDim.x a multiple of 32, <= 512).
__device__ __forceinline__ float exs_scan_f(float v, ExactSumSmem &sh, float *total) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= (uint32_t)o) v = __fadd_rn(v, u);
    }
    if (lane == 31) sh.wf[warp] = v;
    __syncthreads();
    float off = 0.0f, tot = 0.0f;
    for (uint32_t w = 0; w < nw; ++w) {
        const float x = sh.wf[w];
        if (w < warp) off = __fadd_rn(off, x);
        tot = __fadd_rn(tot, x);
    }
    __syncthreads();
    *total = tot;
    return __fadd_rn(v, off);
}

__device__ __forceinline__ void exs_scan_rc(long long r, int c, ExactSumSmem &sh, long long *r_ex,
                                            int *c_ex, long long *r_tot, int *c_tot) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    long long rv = r;
    int cv = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const long long ur = __shfl_up_sync(0xffffffffu, rv, o);
        const int uc = __shfl_up_sync(0xffffffffu, cv, o);
        if (lane >= (uint32_t)o) {
            rv += ur;
            cv += uc;
        }
    }
    if (lane == 31) {
        sh.wr[warp] = rv;
        sh.wc[warp] = cv;
    }
    __syncthreads();
    long long ro = 0, rt = 0;
    int co = 0, ct = 0;
    for (uint32_t w = 0; w < nw; ++w) {
        const long long xr = sh.wr[w];
        const int xc = sh.wc[w];
        if (w < warp) {
            ro += xr;
            co += xc;
        }
        rt += xr;
        ct += xc;
    }
    __syncthreads();
    *r_ex = ro + rv - r;
    *c_ex = co + cv - c;
    *r_tot = rt;
    *c_tot = ct;
}

// The sequential sum of t[0..n) (16-byte aligned; every term expected >= +0),
// returned to every thread of the CTA.  All threads must call it; blockDim.x
// a multiple of 32 and <= 512.
__device__ __forceinline__ float block_exact_sum_nonneg(const float *t, uint32_t n, ExactSumSmem &sh) {
    const uint32_t tid = threadIdx.x, nthr = blockDim.x;
    const uint32_t ept = (n + nthr - 1) / nthr;
    const uint32_t i0 = min(n, tid * ept), i1 = min(n, i0 + ept);
    if (tid == 0) sh.bad = (n < 64u || ept > (uint32_t)EXS_MAX_PER_THREAD) ? 1 : 0;
    // pass 1: this thread's terms; a negative (sign bit), NaN or infinite
    // term sends the sum to the sequential loop
    float loc = 0.0f;
    bool bad = false;
    for (uint32_t i = i0; i < i1; ++i) {
        const float v = t[i];
        bad |= (__float_as_uint(v) >> 31) != 0u || !isfinite(v);
        loc = __fadd_rn(loc, v);
    }
    __syncthreads();
    if (bad) sh.bad = 1;
    float total;
    const float incl = exs_scan_f(loc, sh, &total);  // (syncs)
    const float Pex = __fsub_rn(incl, loc) < 0.0f ? 0.0f : __fsub_rn(incl, loc);
    if (!(total < 1.0e37f)) sh.bad = 1;  // keep away from the f32 range limit
    __syncthreads();
    if (sh.bad) {
        if (tid == 0) sh.result = seq_sum(t, n);
        __syncthreads();
        return sh.result;
    }
    // pass 2: classify this thread's steps; count list entries, sum steps.
    // Usually the thread's whole range stays in one binade (same margin,
    // taken at its last index): every step is then an integer step of that
    // binade, computed independently of the others; else step by step.
    const float Pend = __fadd_rn(Pex, loc);
    const int seg_ue = i0 < i1 ? exs_binade(Pex, Pend, i1 - 1u) : EXS_U;
    float P = Pex;
    int first_key = EXS_U, prev = EXS_U;
    int cnt = 0;
    long long rs = 0;
    for (uint32_t i = i0; i < i1; ++i) {
        const float v = t[i];
        int r = 0, key;
        if (seg_ue != EXS_U) {
            key = exs_step(v, seg_ue, &r);
        } else {
            const float Pn = __fadd_rn(P, v);
            key = exs_classify(P, Pn, v, i, &r);
            P = Pn;
        }
        if (i == i0) first_key = key;
        else if (key == EXS_U || key != prev) ++cnt;
        if (key != EXS_U) rs += r;
        prev = key;
    }
    if (i0 < i1) sh.last_key[tid] = prev;
    __syncthreads();
    // the first step starts an entry unless it continues the previous
    // thread's run (same binade, both certain)
    bool first_new = false;
    if (i0 < i1) {
        first_new = tid == 0 || first_key == EXS_U || sh.last_key[tid - 1] == EXS_U ||
                    sh.last_key[tid - 1] != first_key;
        if (first_new) ++cnt;
    }
    long long r_ex, r_tot;
    int c_ex, c_tot;
    exs_scan_rc(rs, cnt, sh, &r_ex, &c_ex, &r_tot, &c_tot);
    if (c_tot > EXS_MAX_ENTRIES) {  // too many crossings or ties: sequential loop
        if (tid == 0) sh.result = seq_sum(t, n);
        __syncthreads();
        return sh.result;
    }
    // pass 3: write this thread's entries (the same classification as pass 2)
    if (cnt > 0) {
        P = Pex;
        int e = c_ex;
        long long c = r_ex;
        prev = EXS_U;
        for (uint32_t i = i0; i < i1; ++i) {
            const float v = t[i];
            int r = 0, key;
            if (seg_ue != EXS_U) {
                key = exs_step(v, seg_ue, &r);
            } else {
                const float Pn = __fadd_rn(P, v);
                key = exs_classify(P, Pn, v, i, &r);
                P = Pn;
            }
            const bool start = i == i0 ? first_new : (key == EXS_U || key != prev);
            if (start) {
                sh.e_idx[e] = (int)i;
                sh.e_key[e] = key;
                sh.e_c[e] = c;
                ++e;
            }
            if (key != EXS_U) c += r;
            prev = key;
        }
    }
    if (tid == 0) sh.e_c[c_tot] = r_tot;
    __syncthreads();
    // each entry's addend: a run's steps times its spacing (exact, < 2^24
    // spacings within a binade), or a single step's own term
    for (int k = (int)tid; k < c_tot; k += (int)nthr) {
        const int key = sh.e_key[k];
        float a;
        if (key == EXS_U) {
            a = t[sh.e_idx[k]];
        } else {
            const float unit = __uint_as_float(key >= -126 ? (uint32_t)(key + 127) << 23
                                                           : 1u << (key + 149));
            a = __fmul_rn((float)(sh.e_c[k + 1] - sh.e_c[k]), unit);
        }
        sh.addend[k] = a;
    }
    __syncthreads();
    // the walk: the addends in order, each one rounding (exact for the runs)
    if (tid == 0) sh.result = seq_sum(sh.addend, (uint32_t)c_tot);
    __syncthreads();
    return sh.result;
}

}  // namespace wl
