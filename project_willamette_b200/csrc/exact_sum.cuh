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
//  * The exact prefix sums P_i = t_0 + ... + t_{i-1} (computed here in
//    double) bound the running sum: every add errs by at most half a spacing
//    of its result, at most 2^-24 s_i + 2^-150, and s never decreases, so
//    |s_i - P_i| <= i (2^-24 s_i + 2^-150) < (i + 1)(2^-23 P_i + 2^-148).
//    When that interval around P_i and the one around P_{i+1} lie in one
//    binade, step i is such an integer step ("certain").
// So the CTA classifies every step in parallel, sums the integer steps of
// each run of certain steps in one binade with a block scan, and one thread
// then walks the short list of runs and remaining steps (binade crossings,
// ties, the first non-zero term), adding each run with one exact add and
// each remaining term with the reference's own add.  The result is the
// sequential sum's bits.  Any negative or non-finite term, a total near the
// f32 range limit, or more remaining steps than the list holds, send the
// whole sum to one thread's sequential loop instead.
#pragma once

#include <cstdint>

#include "wl_ptx.cuh"

namespace wl {

constexpr int EXS_MAX_ENTRIES = 256;   // runs + single steps the walk can take
constexpr int EXS_MAX_PER_THREAD = 64; // terms per thread (n <= 64 * blockDim.x)
constexpr int EXS_U = -1000;           // entry kind: one step added as the reference does

struct ExactSumSmem {
    double wd[32];          // per-warp partial sums (block scans)
    long long wr[32];
    int wc[32];
    int last_key[512];      // last step's key of every thread (blockDim.x <= 512)
    int n_entries;
    int bad;
    float result;
    int e_idx[EXS_MAX_ENTRIES + 1];
    int e_key[EXS_MAX_ENTRIES + 1];
    long long e_c[EXS_MAX_ENTRIES + 1];  // sum of the integer steps before the entry
};

// Step classification: key = spacing exponent (-149 .. 104) of a certain
// step's binade, EXS_U for a step the walk adds itself; r = the step in units
// of the spacing (certain steps).
__device__ __forceinline__ int exs_region(double v) {
    // binade exponent of v, or -127 for v < 2^-126 (the subnormal spacing)
    if (v < 1.1754943508222875e-38) return -127;
    return (int)((__double2hiint(v) >> 20) & 0x7FF) - 1023;
}

__device__ __forceinline__ int exs_classify(double P, double Pn, float t, uint32_t i, int *r) {
    const double d0 = (double)(i + 1u) * (P * 1.1920928955078125e-07 + 2.8025969286496341e-45);
    const double d1 = (double)(i + 2u) * (Pn * 1.1920928955078125e-07 + 2.8025969286496341e-45);
    const int E = exs_region(P - d0);
    if (E != exs_region(Pn + d1)) return EXS_U;  // may cross a binade boundary
    const int ue = E == -127 ? -149 : E - 23;    // spacing exponent of the binade
    const uint32_t tb = __float_as_uint(t);
    const uint32_t be = tb >> 23;                // t >= +0, finite (checked by the caller)
    const uint32_t m = be ? ((tb & 0x7FFFFFu) | 0x800000u) : tb;
    const int et = be ? (int)be - 127 : -126;
    // t / u = m * 2^(et - 23 - ue)
    const int d = ue - et + 23;
    if (d <= 0) {
        if (m == 0) { *r = 0; return ue; }
        if (-d > 7) return EXS_U;  // a step of 2^31 spacings cannot stay in a binade
        *r = (int)(m << (-d));
        return ue;
    }
    if (d > 30) { *r = 0; return ue; }  // below half a spacing (m < 2^24 <= 2^(d-1))
    const uint32_t half = 1u << (d - 1), rem = m & ((half << 1) - 1u);
    if (rem == half) return EXS_U;      // a tie: the even result depends on s_i
    *r = (int)((m >> d) + (rem > half ? 1u : 0u));
    return ue;
}

// Inclusive block scan helpers (blockDim.x a multiple of 32, <= 1024).
__device__ __forceinline__ double exs_scan_d(double v, ExactSumSmem &sh, double *total) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= (uint32_t)o) v += u;
    }
    if (lane == 31) sh.wd[warp] = v;
    __syncthreads();
    double off = 0.0, tot = 0.0;
    for (uint32_t w = 0; w < nw; ++w) {
        const double x = sh.wd[w];
        if (w < warp) off += x;
        tot += x;
    }
    __syncthreads();
    *total = tot;
    return v + off;
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
        if (w < warp) {
            ro += sh.wr[w];
            co += sh.wc[w];
        }
        rt += sh.wr[w];
        ct += sh.wc[w];
    }
    __syncthreads();
    *r_ex = ro + rv - r;
    *c_ex = co + cv - c;
    *r_tot = rt;
    *c_tot = ct;
}

// The sequential sum of t[0..n) (shared or global memory, 16-byte aligned;
// every term expected >= +0), returned to every thread of the CTA.  All
// threads must call it; blockDim.x a multiple of 32 and <= 512.
__device__ __noinline__ float block_exact_sum_nonneg(const float *t, uint32_t n, ExactSumSmem &sh) {
    const uint32_t tid = threadIdx.x, nthr = blockDim.x;
    const uint32_t ept = (n + nthr - 1) / nthr;
    const uint32_t i0 = min(n, tid * ept), i1 = min(n, i0 + ept);
    if (tid == 0) sh.bad = (n < 64u || ept > (uint32_t)EXS_MAX_PER_THREAD) ? 1 : 0;
    // pass 1: this thread's terms in double; any term that is negative (sign
    // bit), NaN or infinite sends the sum to the sequential loop
    double loc = 0.0;
    bool bad = false;
    for (uint32_t i = i0; i < i1; ++i) {
        const float v = t[i];
        bad |= (__float_as_uint(v) >> 31) != 0u || !isfinite(v);
        loc += (double)v;
    }
    __syncthreads();
    if (bad) sh.bad = 1;
    double total;
    const double Pex = exs_scan_d(loc, sh, &total) - loc;  // exclusive prefix (syncs)
    if (total >= 1.0e38) sh.bad = 1;  // keep away from the f32 range limit
    __syncthreads();
    if (sh.bad) {
        if (tid == 0) sh.result = seq_sum(t, n);
        __syncthreads();
        return sh.result;
    }
    // pass 2: classify this thread's steps; count list entries and sum steps
    double P = Pex;
    int first_key = EXS_U, prev = EXS_U;
    int cnt = 0;
    long long rs = 0;
    for (uint32_t i = i0; i < i1; ++i) {
        const float v = t[i];
        const double Pn = P + (double)v;
        int r = 0;
        const int key = exs_classify(P, Pn, v, i, &r);
        if (i == i0) first_key = key;
        else if (key == EXS_U || key != prev) ++cnt;
        if (key != EXS_U) rs += r;
        prev = key;
        P = Pn;
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
    // pass 3: write this thread's entries (same classification as pass 2)
    P = Pex;
    int e = c_ex;
    long long c = r_ex;
    prev = EXS_U;
    for (uint32_t i = i0; i < i1; ++i) {
        const float v = t[i];
        const double Pn = P + (double)v;
        int r = 0;
        const int key = exs_classify(P, Pn, v, i, &r);
        const bool start = i == i0 ? first_new : (key == EXS_U || key != prev);
        if (start) {
            sh.e_idx[e] = (int)i;
            sh.e_key[e] = key;
            sh.e_c[e] = c;
            ++e;
        }
        if (key != EXS_U) c += r;
        prev = key;
        P = Pn;
    }
    if (tid == 0) {
        sh.e_idx[c_tot] = (int)n;
        sh.e_key[c_tot] = EXS_U;
        sh.e_c[c_tot] = r_tot;
        sh.n_entries = c_tot;
    }
    __syncthreads();
    // the walk: each run adds (sum of its steps) * spacing, exactly; each
    // single step is the reference's add
    if (tid == 0) {
        float s = 0.0f;
        for (int k = 0; k < c_tot; ++k) {
            const int key = sh.e_key[k];
            if (key == EXS_U) {
                s = __fadd_rn(s, t[sh.e_idx[k]]);
            } else {
                const long long steps = sh.e_c[k + 1] - sh.e_c[k];  // < 2^24 within a binade
                const float unit = __uint_as_float(key >= -126 ? (uint32_t)(key + 127) << 23
                                                               : 1u << (key + 149));
                s = __fadd_rn(s, __fmul_rn((float)steps, unit));
            }
        }
        sh.result = s;
    }
    __syncthreads();
    return sh.result;
}

}  // namespace wl
