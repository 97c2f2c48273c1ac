// i2s_matvec.cuh -- I2_S BitLinear decode path for sm_100a.
//
// Reference: bitlinear_i2s_matvec_f32_sse2_i8 (src/model/bitlinear_sse2.rs:313-342),
// quantize_input_absmax_i8 (:285-304), dot_i8_ternary (:353-386), code map
// (src/model/bitlinear.rs:43-50), packed layout (src/gguf/tensor.rs:86-105).
//
// Two kernels chained with programmatic dependent launch (PDL):
//   1. quantize_absmax_kernel: per-row absmax int8 quantisation of x.
//   2. i2s_matvec_kernel: each CTA owns a contiguous range of weight rows.
//      Before waiting on kernel 1 it starts 1-D bulk copies (TMA engine) of
//      its rows into a ring of shared-memory stages, so weight streaming
//      overlaps the previous kernel.  Then it loads the quantised activations
//      it needs into registers and computes the exact int32 ternary dots.
//
// Data layout (HBM): the reference's own I2_S layout, untouched.  A row is
// in_dim/4 bytes; byte gp of 32-byte block b holds the 2-bit codes of
// elements b*128 + gp + {0, 32, 64, 96} in bits {7:6, 5:4, 3:2, 1:0}.  So a
// 32-bit word at byte offset 16*(p&1) + 4j of block p/2 yields, for each
// shift s in {6, 4, 2, 0}, four codes that line up with four consecutive
// int8 activations -- one dp4a per shift, no repack.
//
// Arithmetic: codes c in {0,1,2,3} map to t = c - 1 except code 3 -> 0.
// acc = sum_c dp4a(c, a) - sum(a) - 2 * sum_{c==3}(a), all int32 and exact,
// so the result is bit-identical to the reference's int32 dot whatever the
// summation order.  The output is (w_scale * act_scale) * (float)acc with
// IEEE round-to-nearest multiplies, as the reference computes it.
#pragma once

#include <cstdint>

#include "wl_ptx.cuh"

namespace wl {

constexpr int I2S_THREADS = 256;
constexpr int I2S_WARPS = I2S_THREADS / 32;
constexpr int I2S_MAX_STAGES = 8;
constexpr uint32_t I2S_STAGE_BUDGET = 96u * 1024u;  // bytes of weight stages per CTA
constexpr int QUANT_THREADS = 512;

struct I2sJob {
    const uint8_t *w;    // out_dim x (K/4) bytes, 16-byte aligned
    float w_scale;
    uint32_t out_dim;
    uint32_t row_begin;  // first row of this job in the concatenated row space
    float *y;
    int32_t *acc;        // may be null
};

struct I2sMatvecParams {
    I2sJob jobs[4];
    int njobs;
    uint32_t K;             // in_dim, multiple of 128
    uint32_t total_rows;
    uint32_t rows_per_cta;
    uint32_t nstages;
    uint32_t use_pdl;
    const int8_t *q;        // quantised activations, K bytes, 16-byte aligned
    const float *act_scale; // 1 f32
    uint32_t *status;
};

// ---------------------------------------------------------------------------
// Kernel 1: per-row absmax quantisation (bitlinear_sse2.rs:285-304).
// max over |x| ignores NaN (the reference's strict '>' never takes a NaN);
// inv = 127/max (IEEE division); q = roundf(x*inv) (half away from zero, as
// Rust's f32::round) clamped to +-127, NaN -> 0 (Rust's saturating `as i8`);
// scale = max/127, or 1.0 and all-zero q for an all-zero row.
__global__ void __launch_bounds__(QUANT_THREADS)
    quantize_absmax_kernel(const float *__restrict__ x, uint32_t n, int8_t *__restrict__ q,
                           float *__restrict__ act_scale) {
    pdl_launch_dependents();
    pdl_wait();
    const float *xr = x + (size_t)blockIdx.x * n;
    int8_t *qr = q + (size_t)blockIdx.x * n;
    __shared__ float red[QUANT_THREADS / 32];

    float m = 0.0f;
    for (uint32_t i = threadIdx.x * 4; i < n; i += QUANT_THREADS * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(xr + i);
        m = fmaxf(m, fabsf(v.x));
        m = fmaxf(m, fabsf(v.y));
        m = fmaxf(m, fabsf(v.z));
        m = fmaxf(m, fabsf(v.w));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    float max_abs = red[0];
#pragma unroll
    for (int w = 1; w < QUANT_THREADS / 32; ++w) max_abs = fmaxf(max_abs, red[w]);

    if (max_abs == 0.0f) {
        for (uint32_t i = threadIdx.x * 4; i < n; i += QUANT_THREADS * 4)
            *reinterpret_cast<uint32_t *>(qr + i) = 0u;
        if (threadIdx.x == 0) act_scale[blockIdx.x] = 1.0f;
        return;
    }
    const float inv = __fdiv_rn(127.0f, max_abs);
    for (uint32_t i = threadIdx.x * 4; i < n; i += QUANT_THREADS * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(xr + i);
        const float e[4] = {v.x, v.y, v.z, v.w};
        uint32_t packed = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float r = roundf(__fmul_rn(e[k], inv));
            int qi = 0;
            if (!isnan(r)) qi = (int)fminf(fmaxf(r, -127.0f), 127.0f);
            packed |= (uint32_t)(qi & 0xFF) << (8 * k);
        }
        *reinterpret_cast<uint32_t *>(qr + i) = packed;
    }
    if (threadIdx.x == 0) act_scale[blockIdx.x] = __fdiv_rn(max_abs, 127.0f);
}

// ---------------------------------------------------------------------------
// Kernel 2 helpers.

// Issue chunk `c` of this CTA's row range [r0, r1) into `stage`.  A chunk
// may span two fused weights; each contiguous segment is one bulk copy.
__device__ __forceinline__ void i2s_issue_chunk(const I2sMatvecParams &p, uint32_t c,
                                                uint32_t r0, uint32_t r1, uint32_t rpi,
                                                uint32_t row_bytes, uint8_t *stage,
                                                uint64_t *bar, uint64_t policy) {
    uint32_t a = r0 + c * rpi;
    const uint32_t b = min(a + rpi, r1);
    mbar_arrive_expect_tx(bar, (b - a) * row_bytes);
    uint32_t off = 0;
    for (int j = 0; j < p.njobs && a < b; ++j) {
        const uint32_t jb = p.jobs[j].row_begin, je = jb + p.jobs[j].out_dim;
        if (a >= je) continue;
        const uint32_t e = min(b, je);
        const uint32_t bytes = (e - a) * row_bytes;
        bulk_g2s_evict_first(stage + off, p.jobs[j].w + (size_t)(a - jb) * row_bytes, bytes, bar,
                             policy);
        off += bytes;
        a = e;
    }
}

// One 32-bit weight word (16 codes) against the four activation words it
// lines up with.  Accumulates sum(c*a) and ORs the code-3 detector.
__device__ __forceinline__ int32_t i2s_word(uint32_t w, uint32_t a0, uint32_t a1, uint32_t a2,
                                            uint32_t a3, int32_t acc, uint32_t &c3) {
    acc = __dp4a((int)((w >> 6) & 0x03030303u), (int)a0, acc);
    acc = __dp4a((int)((w >> 4) & 0x03030303u), (int)a1, acc);
    acc = __dp4a((int)((w >> 2) & 0x03030303u), (int)a2, acc);
    acc = __dp4a((int)(w & 0x03030303u), (int)a3, acc);
    c3 |= w & (w >> 1);
    return acc;
}

// Sum over the code-3 positions of one word (rare path; the reference
// quantiser never emits code 3, but the reference maps it to 0).
__device__ __forceinline__ int32_t i2s_word_c3(uint32_t w, uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, int32_t acc) {
    const uint32_t m = w & (w >> 1) & 0x55555555u;
    acc = __dp4a((int)((m >> 6) & 0x01010101u), (int)a0, acc);
    acc = __dp4a((int)((m >> 4) & 0x01010101u), (int)a1, acc);
    acc = __dp4a((int)((m >> 2) & 0x01010101u), (int)a2, acc);
    acc = __dp4a((int)(m & 0x01010101u), (int)a3, acc);
    return acc;
}

__device__ __forceinline__ int32_t sum_bytes(uint4 v) {
    int32_t s = __dp4a((int)v.x, 0x01010101, 0);
    s = __dp4a((int)v.y, 0x01010101, s);
    s = __dp4a((int)v.z, 0x01010101, s);
    return __dp4a((int)v.w, 0x01010101, s);
}

// Kernel 2.  LPR lanes cooperate on one row (RPW = 32/LPR rows per warp),
// lane s of a row owns the 16-byte weight slots p = s + LPR*i.  NP > 0: the
// NP slots' activations (4 x 16 bytes each) live in registers for the whole
// kernel; NP == 0: activations are re-read from L1 per row (very large K).
template <int LPR, int NP>
__global__ void __launch_bounds__(I2S_THREADS, 1)
    i2s_matvec_kernel(const __grid_constant__ I2sMatvecParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[I2S_MAX_STAGES];
    constexpr int RPW = 32 / LPR;
    constexpr uint32_t RPI = I2S_WARPS * RPW;

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t row_bytes = p.K >> 2;
    const uint32_t P = p.K >> 6;
    const uint32_t stage_bytes = RPI * row_bytes;
    const uint32_t r0 = blockIdx.x * p.rows_per_cta;
    const uint32_t r1 = min(r0 + p.rows_per_cta, p.total_rows);
    if (r0 >= r1) {
        pdl_launch_dependents();
        return;
    }
    const uint32_t nchunks = (r1 - r0 + RPI - 1) / RPI;
    const uint32_t nst = p.nstages;
    const uint64_t policy = l2_policy_evict_first();

    if (tid == 0) {
        for (uint32_t s = 0; s < nst; ++s) mbar_init(&full_bar[s], 1);
        fence_mbar_init();
        const uint32_t pre = min(nchunks, nst);
        for (uint32_t c = 0; c < pre; ++c)
            i2s_issue_chunk(p, c, r0, r1, RPI, row_bytes, smem + c * stage_bytes, &full_bar[c],
                            policy);
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();  // the quantised activations come from the previous kernel

    const uint32_t s = lane % LPR;
    const uint32_t sub = lane / LPR;
    const float act_scale = *p.act_scale;

    uint4 act[NP > 0 ? NP : 1][4];
    int32_t asum = 0;
    if constexpr (NP > 0) {
#pragma unroll
        for (int i = 0; i < NP; ++i) {
            const uint32_t pp = s + LPR * i;
#pragma unroll
            for (int o = 0; o < 4; ++o) {
                if (pp < P) {
                    act[i][o] = __ldg(reinterpret_cast<const uint4 *>(
                        p.q + (pp >> 1) * 128 + (pp & 1) * 16 + 32 * o));
                    asum += sum_bytes(act[i][o]);
                } else {
                    act[i][o] = make_uint4(0, 0, 0, 0);
                }
            }
        }
    } else {
        for (uint32_t pp = s; pp < P; pp += LPR) {
#pragma unroll
            for (int o = 0; o < 4; ++o)
                asum += sum_bytes(__ldg(reinterpret_cast<const uint4 *>(
                    p.q + (pp >> 1) * 128 + (pp & 1) * 16 + 32 * o)));
        }
    }

    for (uint32_t c = 0; c < nchunks; ++c) {
        const uint32_t st = c % nst;
        const bool ok = mbar_wait(&full_bar[st], (c / nst) & 1u);
        if (!__syncthreads_and(ok)) {
            if (tid == 0) atomicOr(p.status, WL_DEV_ERR_TIMEOUT);
            // Give the copies already in flight a bounded chance to land
            // before this CTA's shared memory is released.
            for (uint32_t k = c; k < min(nchunks, c + nst); ++k)
                (void)mbar_wait(&full_bar[k % nst], (k / nst) & 1u);
            return;
        }
        const uint32_t row_local = warp * RPW + sub;
        const uint32_t row = r0 + c * RPI + row_local;
        const uint8_t *rp = smem + st * stage_bytes + row_local * row_bytes;
        int32_t dot = -asum;
        uint32_t c3 = 0;
        if (row < r1) {
            if constexpr (NP > 0) {
#pragma unroll
                for (int i = 0; i < NP; ++i) {
                    const uint32_t pp = s + LPR * i;
                    if (pp < P) {
                        const uint4 wv = *reinterpret_cast<const uint4 *>(rp + 16 * pp);
                        dot = i2s_word(wv.x, act[i][0].x, act[i][1].x, act[i][2].x, act[i][3].x,
                                       dot, c3);
                        dot = i2s_word(wv.y, act[i][0].y, act[i][1].y, act[i][2].y, act[i][3].y,
                                       dot, c3);
                        dot = i2s_word(wv.z, act[i][0].z, act[i][1].z, act[i][2].z, act[i][3].z,
                                       dot, c3);
                        dot = i2s_word(wv.w, act[i][0].w, act[i][1].w, act[i][2].w, act[i][3].w,
                                       dot, c3);
                    }
                }
            } else {
                for (uint32_t pp = s; pp < P; pp += LPR) {
                    const uint4 wv = *reinterpret_cast<const uint4 *>(rp + 16 * pp);
                    uint4 a[4];
#pragma unroll
                    for (int o = 0; o < 4; ++o)
                        a[o] = __ldg(reinterpret_cast<const uint4 *>(
                            p.q + (pp >> 1) * 128 + (pp & 1) * 16 + 32 * o));
                    dot = i2s_word(wv.x, a[0].x, a[1].x, a[2].x, a[3].x, dot, c3);
                    dot = i2s_word(wv.y, a[0].y, a[1].y, a[2].y, a[3].y, dot, c3);
                    dot = i2s_word(wv.z, a[0].z, a[1].z, a[2].z, a[3].z, dot, c3);
                    dot = i2s_word(wv.w, a[0].w, a[1].w, a[2].w, a[3].w, dot, c3);
                }
            }
        }
#pragma unroll
        for (int off = LPR / 2; off > 0; off >>= 1) {
            dot += __shfl_xor_sync(0xffffffffu, dot, off);
            c3 |= __shfl_xor_sync(0xffffffffu, c3, off);
        }
        if ((c3 & 0x55555555u) != 0u) {  // uniform across the LPR lanes of this row
            int32_t corr = 0;
            if (row < r1) {
                for (uint32_t pp = s; pp < P; pp += LPR) {
                    const uint4 wv = *reinterpret_cast<const uint4 *>(rp + 16 * pp);
                    uint4 a[4];
#pragma unroll
                    for (int o = 0; o < 4; ++o)
                        a[o] = __ldg(reinterpret_cast<const uint4 *>(
                            p.q + (pp >> 1) * 128 + (pp & 1) * 16 + 32 * o));
                    corr = i2s_word_c3(wv.x, a[0].x, a[1].x, a[2].x, a[3].x, corr);
                    corr = i2s_word_c3(wv.y, a[0].y, a[1].y, a[2].y, a[3].y, corr);
                    corr = i2s_word_c3(wv.z, a[0].z, a[1].z, a[2].z, a[3].z, corr);
                    corr = i2s_word_c3(wv.w, a[0].w, a[1].w, a[2].w, a[3].w, corr);
                }
            }
            // Only the lanes of rows that took this branch participate.
            const uint32_t grp = __match_any_sync(__activemask(), row_local);
#pragma unroll
            for (int off = LPR / 2; off > 0; off >>= 1)
                corr += __shfl_xor_sync(grp, corr, off);
            dot -= 2 * corr;
        }
        if (s == 0 && row < r1) {
            int j = 0;
            while (j + 1 < p.njobs && row >= p.jobs[j + 1].row_begin) ++j;
            const I2sJob &job = p.jobs[j];
            const uint32_t local = row - job.row_begin;
            const float combined = __fmul_rn(job.w_scale, act_scale);
            job.y[local] = __fmul_rn(combined, __int2float_rn(dot));
            if (job.acc) job.acc[local] = dot;
        }
        // Every thread is done with stage st: refill it with chunk c + nst.
        __syncthreads();
        if (tid == 0 && c + nst < nchunks)
            i2s_issue_chunk(p, c + nst, r0, r1, RPI, row_bytes, smem + st * stage_bytes,
                            &full_bar[st], policy);
    }
}

}  // namespace wl
