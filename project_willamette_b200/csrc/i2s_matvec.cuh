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

#include "exact_sum.cuh"
#include "tp.cuh"
#include "wl_ptx.cuh"

namespace wl {

constexpr int I2S_THREADS = 256;
constexpr int I2S_WARPS = I2S_THREADS / 32;
constexpr int I2S_MAX_STAGES = 8;
constexpr uint32_t I2S_STAGE_BUDGET = 64u * 1024u;  // weight stages per CTA (2 CTAs/SM)
constexpr uint32_t I2S_FUSE_Q_MAX_K = 8192;         // x (f32) + q (int8) staged in smem
constexpr int QUANT_THREADS = 512;

struct I2sJob {
    const uint8_t *w;    // out_dim x (K/4) bytes, 16-byte aligned
    float w_scale;
    uint32_t out_dim;
    uint32_t row_begin;  // first row of this job in the concatenated row space
    float *y;
    int32_t *acc;        // may be null
    uint32_t row_off;    // tensor parallel: first global row of this slice in y/acc
};

struct I2sMatvecParams {
    I2sJob jobs[4];
    int njobs;
    uint32_t K;             // in_dim, multiple of 128
    uint32_t total_rows;
    uint32_t rows_per_cta;
    uint32_t nstages;
    uint32_t use_pdl;
    const int8_t *q;        // quantised activations, K bytes, 16-byte aligned (!FUSE_Q)
    const float *act_scale; // 1 f32 (!FUSE_Q)
    const float *x;         // f32 input, K floats, 16-byte aligned (FUSE_Q)
    int8_t *q_out;          // FUSE_Q: optional copy of the quantised input (CTA 0)
    float *scale_out;       // FUSE_Q: optional activation scale (CTA 0)
    uint32_t *status;
    uint32_t *status_host;  // optional: host-mapped word set to 1 (plain store) with any status bit
    TpParams tp;            // world 0: single GPU
    // Decode-step fusions (FUSE_Q only): the CTA transforms its input before
    // quantising it, and the epilogue can add the output into y in place.
    uint32_t pre;           // I2S_PRE_NONE / I2S_PRE_RMSNORM / I2S_PRE_RELU2_RMSNORM
    const float *norm_w;    // RMSNorm weight, K floats
    const float *x2;        // I2S_PRE_RELU2_RMSNORM: the up projection, K floats
    float eps;
    uint32_t residual;      // y[r] = y[r] + out (reference residual add)
    uint32_t finite_flag;   // status bit set when a residual sum is not finite
    uint32_t exact_norm;    // sum of squares in the reference's sequential order
    // FUSE_Q shared-memory staging, set by the host when it fits: the up
    // vector of I2S_PRE_RELU2_RMSNORM (fast mode) and the residual rows this
    // CTA adds into, both copied asynchronously right after the dependency
    // wait so that their load latency overlaps the input transform.
    uint32_t stage_up;
    uint32_t stage_res;
};

constexpr uint32_t I2S_PRE_NONE = 0, I2S_PRE_RMSNORM = 1, I2S_PRE_RELU2_RMSNORM = 2;

// ---------------------------------------------------------------------------
// Kernel 1: per-row absmax quantisation (bitlinear_sse2.rs:285-304).
// max over |x| ignores NaN (the reference's strict '>' never takes a NaN);
// inv = 127/max (IEEE division); q = roundf(x*inv) (half away from zero, as
// Rust's f32::round) clamped to +-127, NaN -> 0 (Rust's saturating `as i8`);
// scale = max/127, or 1.0 and all-zero q for an all-zero row.
__global__ void __launch_bounds__(QUANT_THREADS)
    quantize_absmax_kernel(const float *__restrict__ x, uint32_t n, int8_t *__restrict__ q,
                           float *__restrict__ act_scale, int32_t *__restrict__ rowsum) {
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
        if (threadIdx.x == 0) {
            act_scale[blockIdx.x] = 1.0f;
            if (rowsum) rowsum[blockIdx.x] = 0;
        }
        return;
    }
    const float inv = __fdiv_rn(127.0f, max_abs);
    int32_t rsum = 0;
    for (uint32_t i = threadIdx.x * 4; i < n; i += QUANT_THREADS * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(xr + i);
        const float e[4] = {v.x, v.y, v.z, v.w};
        uint32_t packed = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int qi = quant_round_i8(__fmul_rn(e[k], inv));
            packed |= (uint32_t)(qi & 0xFF) << (8 * k);
        }
        *reinterpret_cast<uint32_t *>(qr + i) = packed;
        rsum = __dp4a((int)packed, 0x01010101, rsum);
    }
    if (threadIdx.x == 0) act_scale[blockIdx.x] = __fdiv_rn(max_abs, 127.0f);
    if (rowsum) {  // sum of the quantised row (the GEMM's code-offset term)
        __shared__ int32_t ired[QUANT_THREADS / 32];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) rsum += __shfl_xor_sync(0xffffffffu, rsum, off);
        if ((threadIdx.x & 31) == 0) ired[threadIdx.x >> 5] = rsum;
        __syncthreads();
        if (threadIdx.x == 0) {
            int32_t t = 0;
            for (int w = 0; w < QUANT_THREADS / 32; ++w) t += ired[w];
            rowsum[blockIdx.x] = t;
        }
    }
}

// ---------------------------------------------------------------------------
// Row-dot building blocks shared by the per-op and the streaming kernels.

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int32_t dp4a_us(uint32_t a, uint32_t b, int32_t c) {
    int32_t d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Four accumulators, one per code position in a byte.  Masking without
// shifting leaves the codes of bits 7:6 / 5:4 / 3:2 / 1:0 scaled by 64 / 16 /
// 4 / 1, so a6 = 64*sum(c*a) etc.; every term is an exact multiple, so the
// arithmetic right shifts in i2s_acc_total are exact.  |a6| <= 192*127*K/4
// stays below 2^31 for K <= 65536.
struct I2sAcc {
    int32_t a6, a4, a2, a0;
};

template <bool C3>
__device__ __forceinline__ void i2s_word(uint32_t w, uint32_t x0, uint32_t x1, uint32_t x2,
                                         uint32_t x3, I2sAcc &acc, uint32_t &c3) {
    acc.a6 = dp4a_us(w & 0xC0C0C0C0u, x0, acc.a6);
    acc.a4 = dp4a_us(w & 0x30303030u, x1, acc.a4);
    acc.a2 = dp4a_us(w & 0x0C0C0C0Cu, x2, acc.a2);
    acc.a0 = dp4a_us(w & 0x03030303u, x3, acc.a0);
    if constexpr (C3) c3 |= w & (w >> 1);
}

// One 16-byte weight slot (64 codes) against its four activation vectors.
template <bool C3>
__device__ __forceinline__ void i2s_slot(const uint4 &wv, const uint4 (&a)[4], I2sAcc &acc,
                                         uint32_t &c3) {
    i2s_word<C3>(wv.x, a[0].x, a[1].x, a[2].x, a[3].x, acc, c3);
    i2s_word<C3>(wv.y, a[0].y, a[1].y, a[2].y, a[3].y, acc, c3);
    i2s_word<C3>(wv.z, a[0].z, a[1].z, a[2].z, a[3].z, acc, c3);
    i2s_word<C3>(wv.w, a[0].w, a[1].w, a[2].w, a[3].w, acc, c3);
}

__device__ __forceinline__ int32_t i2s_acc_total(const I2sAcc &acc) {
    return (acc.a6 >> 6) + (acc.a4 >> 4) + (acc.a2 >> 2) + acc.a0;
}

// Sum of the activations at code-3 positions of one word (rare path; the
// reference quantiser never emits code 3, but the reference maps it to 0).
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

// Shared-memory layout of the quantised activations in the fused kernels
// (V = true): vector o (0..3) of weight slot pp -- the 16 activations that
// line up with code bits 7:6 / 5:4 / 3:2 / 1:0 of the slot -- sits at
// o * plane + pp * 16, plane = K/4 + 32 bytes.  The 8 lanes of a row read
// vector o of 8 consecutive slots: 128 contiguous bytes, one wavefront per
// quarter-warp.  (In the natural layout those 8 vectors lie at offsets
// 0, 16, 128, 144, ...: a 4-way bank conflict in every quarter-warp, 16
// wavefronts per 128-bit load, measured at about 1.3 us per matvec.)  The
// 32-byte pad puts the 4 planes on different banks for the quantiser's stores.
constexpr uint32_t I2S_QS_PAD = 128;  // bytes beyond K that the layout needs
__host__ __device__ __forceinline__ uint32_t qs_plane(uint32_t K) { return K / 4u + 32u; }
__device__ __forceinline__ uint32_t qs_index(uint32_t e, uint32_t plane) {
    const uint32_t r = e & 127u;  // element e = 128 b + 32 o + 16 h + j, slot 2 b + h
    return (r >> 5) * plane + ((e >> 7) * 2u + ((r >> 4) & 1u)) * 16u + (r & 15u);
}

// The four 16-byte activation vectors that line up with weight slot pp, from
// the natural layout (V = false: element order) or the fused kernels' layout.
template <bool V>
__device__ __forceinline__ void i2s_load_act(const int8_t *q, uint32_t pp, uint32_t plane,
                                             uint4 (&a)[4]) {
    if constexpr (V) {
#pragma unroll
        for (int o = 0; o < 4; ++o)
            a[o] = *reinterpret_cast<const uint4 *>(q + o * plane + pp * 16u);
    } else {
        const int8_t *base = q + (pp >> 1) * 128u + (pp & 1u) * 16u;
#pragma unroll
        for (int o = 0; o < 4; ++o) a[o] = *reinterpret_cast<const uint4 *>(base + 32 * o);
    }
}

// Correction for code-3 codes of one row (slots pp = s, s+stride, ... < P).
template <bool V>
__device__ __forceinline__ int32_t i2s_row_c3(const uint8_t *rp, const int8_t *q, uint32_t plane,
                                              uint32_t s, uint32_t stride, uint32_t P) {
    int32_t corr = 0;
    for (uint32_t pp = s; pp < P; pp += stride) {
        const uint4 wv = *reinterpret_cast<const uint4 *>(rp + 16 * pp);
        uint4 a[4];
        i2s_load_act<V>(q, pp, plane, a);
        corr = i2s_word_c3(wv.x, a[0].x, a[1].x, a[2].x, a[3].x, corr);
        corr = i2s_word_c3(wv.y, a[0].y, a[1].y, a[2].y, a[3].y, corr);
        corr = i2s_word_c3(wv.z, a[0].z, a[1].z, a[2].z, a[3].z, corr);
        corr = i2s_word_c3(wv.w, a[0].w, a[1].w, a[2].w, a[3].w, corr);
    }
    return corr;
}

// Warp-sum of a thread's share of the quantised activations, stored for the
// CTA total (read after the quantiser's final barrier: cta_qsum).
__device__ __forceinline__ void publish_qsum(int32_t qsum, int32_t *ared) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, off);
    if ((threadIdx.x & 31) == 0) ared[threadIdx.x >> 5] = qsum;
}
__device__ __forceinline__ int32_t cta_qsum(const int32_t *ared) {
    int32_t t = 0;
#pragma unroll
    for (int w = 0; w < I2S_WARPS; ++w) t += ared[w];
    return t;
}

// Decode-step input transform + absmax quantisation (same IEEE steps as
// quantize_absmax_kernel) by the whole CTA, the input held in registers:
// every global load of a thread is issued before any is used (one memory
// round trip per CTA instead of one per 1024-element pass), the RMSNorm
// weights were copied to `nw` (shared memory) before the dependency wait.
// Every CTA computes the same values in the same order:
//   I2S_PRE_RMSNORM:       rms_norm(x, w)              (primitives.rs:227-254)
//   I2S_PRE_RELU2_RMSNORM: rms_norm(relu(x)^2 * x2, w) (ffn.rs:37-65, then the
//                          ffn_sub_norm of cached_forward.rs:480-494)
// rms_norm: mean = sum(v*v) / K, rsqrt = 1 / sqrt(mean + eps), out = (v *
// rsqrt) * w.  The sum of squares is a tree (fast mode), or with EXACT the
// reference's sequential loop over the squares stored in `chain`.
constexpr int I2S_PRE_V = (int)(I2S_FUSE_Q_MAX_K / (I2S_THREADS * 4u));  // float4 per thread

template <bool EXACT>
__device__ __forceinline__ float cta_prepare_regs(const I2sMatvecParams &p, uint32_t K,
                                                  const float *nw, int8_t *qs, float *red,
                                                  int32_t *ared, const float *us,
                                                  float *chain = nullptr) {
    const uint32_t tid = threadIdx.x, nthr = blockDim.x;
    const bool relu2 = p.pre == I2S_PRE_RELU2_RMSNORM;
    // float4 slots this CTA's K needs: the unrolled loops leave at the first
    // unused one (a warp-uniform branch) instead of issuing predicated-off
    // work for every slot up to I2S_FUSE_Q_MAX_K.
    const int kmax = (int)((K + nthr * 4u - 1u) / (nthr * 4u));
    float4 v[I2S_PRE_V];
#pragma unroll
    for (int k = 0; k < I2S_PRE_V; ++k) {
        if (k >= kmax) break;
        const uint32_t i = tid * 4u + (uint32_t)k * nthr * 4u;
        if (i < K) v[k] = *reinterpret_cast<const float4 *>(p.x + i);
    }
    if (relu2 && us) {  // v = relu(x)^2 * up, up copied to this thread's slots of `us`
        asm volatile("cp.async.wait_group 1;" ::: "memory");
#pragma unroll
        for (int k = 0; k < I2S_PRE_V; ++k) {
            if (k >= kmax) break;
            const uint32_t i = tid * 4u + (uint32_t)k * nthr * 4u;
            if (i < K) {
                const float4 u = *reinterpret_cast<const float4 *>(us + i);
                float4 &x = v[k];
                const float r0 = x.x > 0.0f ? x.x : 0.0f, r1 = x.y > 0.0f ? x.y : 0.0f;
                const float r2 = x.z > 0.0f ? x.z : 0.0f, r3 = x.w > 0.0f ? x.w : 0.0f;
                x.x = __fmul_rn(__fmul_rn(r0, r0), u.x);
                x.y = __fmul_rn(__fmul_rn(r1, r1), u.y);
                x.z = __fmul_rn(__fmul_rn(r2, r2), u.z);
                x.w = __fmul_rn(__fmul_rn(r3, r3), u.w);
            }
        }
    } else if (relu2) {  // the up vector in two halves (bounded registers)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float4 u[I2S_PRE_V / 2];
#pragma unroll
            for (int k = 0; k < I2S_PRE_V / 2; ++k) {
                if (h * (I2S_PRE_V / 2) + k >= kmax) break;
                const uint32_t i = tid * 4u + (uint32_t)(h * (I2S_PRE_V / 2) + k) * nthr * 4u;
                if (i < K) u[k] = *reinterpret_cast<const float4 *>(p.x2 + i);
            }
#pragma unroll
            for (int k = 0; k < I2S_PRE_V / 2; ++k) {
                const int kk = h * (I2S_PRE_V / 2) + k;
                if (kk >= kmax) break;
                const uint32_t i = tid * 4u + (uint32_t)kk * nthr * 4u;
                if (i < K) {
                    float4 &x = v[kk];
                    const float r0 = x.x > 0.0f ? x.x : 0.0f, r1 = x.y > 0.0f ? x.y : 0.0f;
                    const float r2 = x.z > 0.0f ? x.z : 0.0f, r3 = x.w > 0.0f ? x.w : 0.0f;
                    x.x = __fmul_rn(__fmul_rn(r0, r0), u[k].x);
                    x.y = __fmul_rn(__fmul_rn(r1, r1), u[k].y);
                    x.z = __fmul_rn(__fmul_rn(r2, r2), u[k].z);
                    x.w = __fmul_rn(__fmul_rn(r3, r3), u[k].w);
                }
            }
        }
    }
    if (p.pre != I2S_PRE_NONE) {
        float sum_sq;
        if constexpr (EXACT) {
            // exact mode: the reference's loop sum_sq += x[i] * x[i], i = 0, 1,
            // ...: the squares (one rounding each) stored in parallel, then
            // their sequential sum (exact_sum.cuh)
#pragma unroll
            for (int k = 0; k < I2S_PRE_V; ++k) {
                if (k >= kmax) break;
                const uint32_t i = tid * 4u + (uint32_t)k * nthr * 4u;
                if (i < K)
                    *reinterpret_cast<float4 *>(chain + i) =
                        make_float4(__fmul_rn(v[k].x, v[k].x), __fmul_rn(v[k].y, v[k].y),
                                    __fmul_rn(v[k].z, v[k].z), __fmul_rn(v[k].w, v[k].w));
            }
            __syncthreads();
            if (K + I2S_QS_PAD >= exact_sum_scratch_bytes(I2S_THREADS)) {
                // the quantised-input buffer is free until the quantisation
                sum_sq = cta_exact_sum_nonneg_call(chain, K, reinterpret_cast<uint8_t *>(qs));
            } else {
                if (tid == 0) red[0] = seq_sum(chain, K);
                __syncthreads();
                sum_sq = red[0];
            }
        } else {
            float ss = 0.0f;
#pragma unroll
            for (int k = 0; k < I2S_PRE_V; ++k) {
                if (k >= kmax) break;
                const uint32_t i = tid * 4u + (uint32_t)k * nthr * 4u;
                if (i < K)
                    ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(__fmul_rn(v[k].x, v[k].x), __fmul_rn(v[k].y, v[k].y)),
                                                 __fadd_rn(__fmul_rn(v[k].z, v[k].z), __fmul_rn(v[k].w, v[k].w))));
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
            if ((tid & 31) == 0) red[tid >> 5] = ss;
            __syncthreads();
            sum_sq = red[0];
            for (uint32_t w = 1; w < nthr / 32; ++w) sum_sq = __fadd_rn(sum_sq, red[w]);
        }
        const float mean = __fdiv_rn(sum_sq, (float)K);
        const float rsqrt = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
#pragma unroll
        for (int k = 0; k < I2S_PRE_V; ++k) {
            if (k >= kmax) break;
            const uint32_t i = tid * 4u + (uint32_t)k * nthr * 4u;
            if (i < K) {
                const float4 w = *reinterpret_cast<const float4 *>(nw + i);
                v[k].x = __fmul_rn(__fmul_rn(v[k].x, rsqrt), w.x);
                v[k].y = __fmul_rn(__fmul_rn(v[k].y, rsqrt), w.y);
                v[k].z = __fmul_rn(__fmul_rn(v[k].z, rsqrt), w.z);
                v[k].w = __fmul_rn(__fmul_rn(v[k].w, rsqrt), w.w);
            }
        }
        __syncthreads();  // red is reused below
    }
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < I2S_PRE_V; ++k) {
        if (k >= kmax) break;
        const uint32_t i = tid * 4u + (uint32_t)k * nthr * 4u;
        if (i < K)
            m = fmaxf(fmaxf(fmaxf(m, fabsf(v[k].x)), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w)));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    float max_abs = red[0];
    for (uint32_t w = 1; w < nthr / 32; ++w) max_abs = fmaxf(max_abs, red[w]);
    const float inv = max_abs == 0.0f ? 0.0f : __fdiv_rn(127.0f, max_abs);
    int32_t qsum = 0;
#pragma unroll
    for (int k = 0; k < I2S_PRE_V; ++k) {
        if (k >= kmax) break;
        const uint32_t i = tid * 4u + (uint32_t)k * nthr * 4u;
        if (i < K) {
            const uint32_t packed =
                max_abs != 0.0f
                    ? pack_i8x4(quant_round_i8(__fmul_rn(v[k].x, inv)),
                                quant_round_i8(__fmul_rn(v[k].y, inv)),
                                quant_round_i8(__fmul_rn(v[k].z, inv)),
                                quant_round_i8(__fmul_rn(v[k].w, inv)))
                    : 0u;
            *reinterpret_cast<uint32_t *>(qs + qs_index(i, qs_plane(K))) = packed;
            qsum = __dp4a((int)packed, 0x01010101, qsum);
        }
    }
    publish_qsum(qsum, ared);
    __syncthreads();
    return max_abs == 0.0f ? 1.0f : __fdiv_rn(max_abs, 127.0f);
}

// A host-mapped copy of "some status bit is set", for the host-buffer call that
// reads its output straight from pinned host memory and so has no device
// copy to bring the status word back with (a plain store: device atomics on
// host memory are not available over every host link).
__device__ __forceinline__ void i2s_flag_host(const I2sMatvecParams &p) {
    if (p.status_host) *reinterpret_cast<volatile uint32_t *>(p.status_host) = 1u;
}

// ---------------------------------------------------------------------------
// Kernel 2: per-op matvec (one BitLinear, or several sharing one input).

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

// LPR lanes cooperate on one row (RPW = 32/LPR rows per warp); lane s owns
// the 16-byte weight slots pp = s + LPR*i.  NP > 0: those slots' activations
// (4 x 16 bytes each) live in registers for the whole kernel; NP == 0: they
// are re-read from L1 per row (very large K).  FUSE_Q: the CTA quantises the
// f32 input itself (no separate kernel, one dependency hop less).  C3: the
// weights may contain code 0b11 (checked per row; the fast path otherwise).
// At most 128 registers per thread, so the next op's CTA fits on the same SM.
// The programmatic-launch trigger comes after the row loop: the next op's
// CTAs then arrive while this op's last rows finish and start their weight
// copies there.  (Triggering at entry let them run their prologue beside this
// op's whole pre-phase and row loop on the same SMs, which slowed this op's
// slowest CTAs by 2-4 us: a BitNet decode token took 1631 instead of 1427 us.)
template <int LPR, int NP, bool FUSE_Q, bool C3, bool EXACT = false>
__global__ void __launch_bounds__(I2S_THREADS, 2)
    i2s_matvec_kernel(const __grid_constant__ I2sMatvecParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[I2S_MAX_STAGES];
    __shared__ float red[I2S_WARPS];
    __shared__ int32_t ared[I2S_WARPS];
    __shared__ uint32_t s_bad;  // a warp's weight wait timed out (resident-chunk loop)
    constexpr int RPW = 32 / LPR;
    constexpr uint32_t RPI = I2S_WARPS * RPW;

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t K = p.K;
    const uint32_t row_bytes = K >> 2;
    const uint32_t P = K >> 6;
    const uint32_t stage_bytes = RPI * row_bytes;
    const uint32_t r0 = blockIdx.x * p.rows_per_cta;
    const uint32_t r1 = min(r0 + p.rows_per_cta, p.total_rows);
    if (r0 >= r1) {
        pdl_launch_dependents();
        if (p.tp.world) {
            // the CTA-done counter is shared with the previous kernel, whose
            // last CTA re-arms it: count only once that kernel has finished
            pdl_wait();
            if (tid == 0) tp_arrive(p.tp);
        }
        return;
    }
    const uint32_t nchunks = (r1 - r0 + RPI - 1) / RPI;
    const uint32_t nst = p.nstages;
    const uint64_t policy = l2_policy_evict_first();

    if (tid == 0) {
        s_bad = 0;
        for (uint32_t s = 0; s < nst; ++s) mbar_init(&full_bar[s], 1);
        fence_mbar_init();
        const uint32_t pre = min(nchunks, nst);
        for (uint32_t c = 0; c < pre; ++c)
            i2s_issue_chunk(p, c, r0, r1, RPI, row_bytes, smem + c * stage_bytes, &full_bar[c],
                            policy);
    }
    // The RMSNorm weights do not depend on earlier kernels either.  Exact mode
    // (the reference's sequential sum of squares) keeps them after the
    // quantised input, so that xs holds the transformed input for that sum.
    const bool exact_pre = EXACT && FUSE_Q && p.pre != I2S_PRE_NONE;
    if constexpr (FUSE_Q) {
        if (!exact_pre && p.pre != I2S_PRE_NONE) {
            float *nw = reinterpret_cast<float *>(smem + nst * stage_bytes);
            for (uint32_t i = tid * 4u; i < K; i += I2S_THREADS * 4u)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(nw + i)),
                             "l"(p.norm_w + i)
                             : "memory");
            asm volatile("cp.async.commit_group;" ::: "memory");
        } else if (p.pre != I2S_PRE_NONE) {  // exact mode: after the quantised input
            float *nw = reinterpret_cast<float *>(smem + nst * stage_bytes + (size_t)K * 5u +
                                                  I2S_QS_PAD);
            for (uint32_t i = tid * 4u; i < K; i += I2S_THREADS * 4u)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(nw + i)),
                             "l"(p.norm_w + i)
                             : "memory");
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
    }
    __syncthreads();
    pdl_wait();  // the input comes from the previous kernel
    if (p.tp.world && p.tp.wait) {
        // the input is a vector all ranks gathered into this rank's block
        if (tid == 0 && !tp_wait(p.tp)) {
            atomicOr(p.status, WL_DEV_ERR_PEER_TIMEOUT);
            i2s_flag_host(p);
        }
        __syncthreads();
    }

    float act_scale;
    const int8_t *q;
    if constexpr (FUSE_Q) {
        float *xs = reinterpret_cast<float *>(smem + nst * stage_bytes);
        int8_t *qs = reinterpret_cast<int8_t *>(xs + K);
        float *us = reinterpret_cast<float *>(qs + K + I2S_QS_PAD);  // K floats (stage_up)
        // exact mode stages the RMSNorm weights where fast mode keeps up
        float *ysm = us + ((p.stage_up || exact_pre) ? K : 0u);       // this CTA's rows (stage_res)
        if (p.pre != I2S_PRE_NONE) {
            asm volatile("cp.async.wait_all;" ::: "memory");
            __syncthreads();
        }
        // Two copy groups, always both committed (possibly empty) so that
        // "wait_group 1" means the first one has landed.
        if (p.stage_up)
            for (uint32_t i = tid * 4u; i < K; i += I2S_THREADS * 4u)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(us + i)),
                             "l"(p.x2 + i)
                             : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
        if (p.stage_res)
            for (uint32_t j = tid; j < r1 - r0; j += I2S_THREADS) {
                const uint32_t row = r0 + j;
                int jb = 0;
                while (jb + 1 < p.njobs && row >= p.jobs[jb + 1].row_begin) ++jb;
                const I2sJob &job = p.jobs[jb];
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(ysm + j)),
                             "l"(job.y + job.row_off + (row - job.row_begin))
                             : "memory");
            }
        asm volatile("cp.async.commit_group;" ::: "memory");
        // exact mode: RMSNorm weights at `us`, the transformed input to xs
        // for the reference's sequential sum of squares
        if constexpr (EXACT)
            act_scale = exact_pre ? cta_prepare_regs<true>(p, K, us, qs, red, ared, nullptr, xs)
                                  : cta_prepare_regs<false>(p, K, xs, qs, red, ared, nullptr);
        else
            act_scale = cta_prepare_regs<false>(p, K, xs, qs, red, ared, p.stage_up ? us : nullptr);
        if (blockIdx.x == 0) {
            if (p.q_out)
                for (uint32_t i = tid * 16; i < K; i += I2S_THREADS * 16)
                    *reinterpret_cast<uint4 *>(p.q_out + i) =
                        *reinterpret_cast<const uint4 *>(qs + qs_index(i, qs_plane(K)));
            if (p.scale_out && tid == 0) *p.scale_out = act_scale;
        }
        q = qs;
    } else {
        act_scale = *p.act_scale;
        q = p.q;
    }

    const uint32_t s = lane % LPR;
    const uint32_t sub = lane / LPR;
    const uint32_t plane = qs_plane(K);  // FUSE_Q: layout of the quantised activations
    uint4 act[NP > 0 ? NP : 1][4];
    // Sum of the quantised activations (the code-offset term): with FUSE_Q
    // the quantiser produced the CTA total, subtracted once per row after the
    // lane reduction; otherwise each lane sums the slots it owns.
    int32_t asum = 0;
    if constexpr (FUSE_Q) asum = cta_qsum(ared);
    if constexpr (NP > 0) {
#pragma unroll
        for (int i = 0; i < NP; ++i) {
            const uint32_t pp = s + LPR * i;
            if (pp < P) {
                i2s_load_act<FUSE_Q>(q, pp, plane, act[i]);
                if constexpr (!FUSE_Q) {
#pragma unroll
                    for (int o = 0; o < 4; ++o) asum += sum_bytes(act[i][o]);
                }
            } else {
#pragma unroll
                for (int o = 0; o < 4; ++o) act[i][o] = make_uint4(0, 0, 0, 0);
            }
        }
    } else {
        if constexpr (!FUSE_Q) {
            for (uint32_t pp = s; pp < P; pp += LPR) {
                uint4 a[4];
                i2s_load_act<FUSE_Q>(q, pp, plane, a);
#pragma unroll
                for (int o = 0; o < 4; ++o) asum += sum_bytes(a[o]);
            }
        }
    }

    float *ysm = nullptr;  // staged residual rows (visible after the loop's first barrier)
    if constexpr (FUSE_Q) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        if (p.stage_res)
            ysm = reinterpret_cast<float *>(smem + nst * stage_bytes + (size_t)K * 5u + I2S_QS_PAD +
                                            ((p.stage_up || exact_pre) ? (size_t)K * 4u : 0u));
    }
    // Every chunk requested up front (no ring reuse): each warp waits for a
    // chunk's weights itself and the loop needs no CTA barrier.  Otherwise
    // the CTA waits together and refills a stage once all warps are done.
    const bool resident = nchunks <= nst;
    if (resident) __syncthreads();  // staged residual rows visible to every warp
    for (uint32_t c = 0; c < nchunks; ++c) {
        const uint32_t st = c % nst;
        if (resident) {
            if (!__all_sync(0xffffffffu, mbar_wait(&full_bar[st], 0u))) {
                if (lane == 0) atomicOr(&s_bad, 1u);
                break;
            }
        } else if (!__syncthreads_and(mbar_wait(&full_bar[st], (c / nst) & 1u))) {
            if (tid == 0) {
                atomicOr(p.status, WL_DEV_ERR_TIMEOUT);
                i2s_flag_host(p);
            }
            // Give the copies already in flight a bounded chance to land
            // before this CTA's shared memory is released.
            for (uint32_t k = c; k < min(nchunks, c + nst); ++k)
                (void)mbar_wait(&full_bar[k % nst], (k / nst) & 1u);
            if (p.tp.world && tid == 0) tp_arrive(p.tp);
            return;
        }
        const uint32_t row_local = warp * RPW + sub;
        const uint32_t row = r0 + c * RPI + row_local;
        const uint8_t *rp = smem + st * stage_bytes + row_local * row_bytes;
        I2sAcc acc = {0, 0, 0, 0};
        uint32_t c3 = 0;
        if (row < r1) {
            if constexpr (NP > 0) {
#pragma unroll
                for (int i = 0; i < NP; ++i) {
                    const uint32_t pp = s + LPR * i;
                    if (pp < P)
                        i2s_slot<C3>(*reinterpret_cast<const uint4 *>(rp + 16 * pp), act[i], acc,
                                     c3);
                }
            } else {
                for (uint32_t pp = s; pp < P; pp += LPR) {
                    uint4 a[4];
                    i2s_load_act<FUSE_Q>(q, pp, plane, a);
                    i2s_slot<C3>(*reinterpret_cast<const uint4 *>(rp + 16 * pp), a, acc, c3);
                }
            }
        }
        int32_t dot = i2s_acc_total(acc) - (FUSE_Q ? 0 : asum);
#pragma unroll
        for (int off = LPR / 2; off > 0; off >>= 1) {
            dot += __shfl_xor_sync(0xffffffffu, dot, off);
            if constexpr (C3) c3 |= __shfl_xor_sync(0xffffffffu, c3, off);
        }
        if constexpr (FUSE_Q) dot -= asum;
        if constexpr (C3) {
            if ((c3 & 0x55555555u) != 0u) {  // uniform across the LPR lanes of this row
                int32_t corr = row < r1 ? i2s_row_c3<FUSE_Q>(rp, q, plane, s, LPR, P) : 0;
                // Only the lanes of rows that took this branch participate.
                const uint32_t grp = __match_any_sync(__activemask(), row_local);
#pragma unroll
                for (int off = LPR / 2; off > 0; off >>= 1)
                    corr += __shfl_xor_sync(grp, corr, off);
                dot -= 2 * corr;
            }
        }
        if (s == 0 && row < r1) {
            int j = 0;
            while (j + 1 < p.njobs && row >= p.jobs[j + 1].row_begin) ++j;
            const I2sJob &job = p.jobs[j];
            const uint32_t local = row - job.row_begin;
            const float combined = __fmul_rn(job.w_scale, act_scale);
            const float yv = __fmul_rn(combined, __int2float_rn(dot));
            if (p.tp.world) {
                // gathered output: every rank's replica of y gets the row
                // (residual: this rank's replica + y, the same on every rank)
                float v = yv;
                if (p.residual) {
                    v = __fadd_rn(ysm ? ysm[row - r0] : job.y[job.row_off + local], yv);
                    if (p.finite_flag && !isfinite(v)) {
                        atomicOr(p.status, p.finite_flag);
                        i2s_flag_host(p);
                    }
                }
                tp_store_all(p.tp, job.y + job.row_off + local, v);
            } else if (p.residual) {
                float *dst = job.y + job.row_off + local;
                const float nv = __fadd_rn(ysm ? ysm[row - r0] : *dst, yv);
                *dst = nv;
                if (p.finite_flag && !isfinite(nv)) {
                    atomicOr(p.status, p.finite_flag);
                    i2s_flag_host(p);
                }
            } else {
                job.y[job.row_off + local] = yv;
            }
            if (job.acc) job.acc[job.row_off + local] = dot;
        }
        if (!resident) {
            // Every thread is done with stage st: refill it with chunk c + nst.
            __syncthreads();
            if (tid == 0 && c + nst < nchunks)
                i2s_issue_chunk(p, c + nst, r0, r1, RPI, row_bytes, smem + st * stage_bytes,
                                &full_bar[st], policy);
        }
    }
    if (resident) {
        __syncthreads();
        if (s_bad && tid == 0) {
            atomicOr(p.status, WL_DEV_ERR_TIMEOUT);
            i2s_flag_host(p);
            // bounded waits for the copies still in flight before the CTA's
            // shared memory is released
            for (uint32_t k = 0; k < nchunks; ++k) (void)mbar_wait(&full_bar[k], 0u);
        }
    }
    pdl_launch_dependents();
    if (p.tp.world && tid == 0) tp_arrive(p.tp);  // after the loop's final barrier
}

// One-time scan: does a packed I2_S tensor contain code 0b11 anywhere?
__global__ void i2s_scan_code3_kernel(const uint4 *__restrict__ w, size_t n16,
                                      uint32_t *__restrict__ found) {
    uint32_t any = 0;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16;
         i += (size_t)gridDim.x * blockDim.x) {
        const uint4 v = w[i];
        any |= (v.x & (v.x >> 1)) | (v.y & (v.y >> 1)) | (v.z & (v.z >> 1)) | (v.w & (v.w >> 1));
    }
    if (__any_sync(0xffffffffu, (any & 0x55555555u) != 0u) && (threadIdx.x & 31) == 0)
        atomicOr(found, 1u);
}

}  // namespace wl
