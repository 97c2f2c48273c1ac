// bitnet_decode.cuh -- the non-BitLinear kernels of the device-resident
// BitNet b1.58 decode step (embedding, attention with the i8 KV cache, final
// norm).  The BitLinears run through i2s_matvec_kernel, whose CTAs apply the
// RMSNorm (and relu^2 * up for the down projection) to their input before
// quantising it, and whose epilogue adds the residual in place.
//
// Reference step: forward_with_cache_progress_into / forward_one_layer /
// scaled_dot_product_attention_into / apply_ffn_block
// (src/model/cached_forward.rs:206-504); primitives: rms_norm_f32
// (primitives.rs:227-254), apply_rope_f32 NEOX (:283-345), softmax_inplace
// (attention.rs:45-73), KVCache append / read_into (kv_cache.rs:154-259).
//
// The step reads the token and the position from device memory, so a whole
// step (and greedy decode: lm-head -> token -> next step) is replayed from a
// CUDA graph without host round trips.
//
// Numerics: the per-element arithmetic is the reference's, IEEE
// round-to-nearest, no FMA contraction; RoPE cos/sin come from a table the
// host fills with the C library's powf/sinf/cosf exactly as the reference
// computes them.  Sums (RMSNorm, attention dot products, softmax, the V
// weighted sum) run as parallel trees instead of the reference's sequential
// loops (exp is glibc's expf restated, glibc_expf.cuh), so hidden states
// agree to rounding level, not bit for bit.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>
#include <type_traits>

#include "exact_sum.cuh"
#include "glibc_expf.cuh"
#include "q6k_lmhead.cuh"
#include "tp.cuh"
#include "wl_ptx.cuh"

namespace wl {

constexpr uint32_t WL_DEV_ERR_NONFINITE = 4u;  // non-finite hidden after a layer
constexpr uint32_t WL_DEV_ERR_POSITION = 8u;   // KV cache full
constexpr int ATTN_THREADS = 256;

// ---------------------------------------------------------------------------
// Block-wide reductions (deterministic: fixed shuffle tree, then warps in order).
__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = red[0];
    for (uint32_t w = 1; w < blockDim.x / 32; ++w) t = __fadd_rn(t, red[w]);
    return t;
}

__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = red[0];
    for (uint32_t w = 1; w < blockDim.x / 32; ++w) t = fmaxf(t, red[w]);
    return t;
}

// ---------------------------------------------------------------------------
// Embedding: the token's row of the tied Q6_K table (repacked lm-head
// layout, q6k_lmhead.cuh), dequantised w = (d * sc) * q (q6_k.rs:25-69).
// One CTA per 256-value super-block, one thread per value.  CTA 0 also
// appends the token to the generated-id list when `ids` is set.
struct EmbedParams {
    const uint8_t *packed;  // repacked Q6_K rows
    uint32_t nb, row_stride;
    const uint32_t *token;
    float *hidden;
    uint32_t *ids;          // optional: ids[*step] = token, ++*step
    uint32_t *step;
};

__global__ void __launch_bounds__(256) embed_q6k_kernel(const __grid_constant__ EmbedParams p) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t tok = *p.token;
    const uint32_t b = blockIdx.x, t = threadIdx.x;
    const uint8_t *row = p.packed + (size_t)tok * p.row_stride;
    const uint8_t *ql = row + b * 128u, *qh = row + p.nb * 128u + b * 64u;
    const int8_t *sc = reinterpret_cast<const int8_t *>(row + p.nb * 192u + b * 16u);
    const uint16_t dbits = *reinterpret_cast<const uint16_t *>(row + p.nb * 208u + b * 2u);
    // value t of the block: half h, quarter a, lane l (q6_k.rs:25-57)
    const uint32_t h = t >> 7, a = (t >> 5) & 3u, l = t & 31u;
    const uint8_t lb = ql[h * 64u + l + ((a & 1u) ? 32u : 0u)];
    const uint32_t lo = (a & 2u) ? (lb >> 4) : (lb & 0x0Fu);
    const uint32_t hi = (qh[h * 32u + l] >> (2u * a)) & 3u;
    const int q = (int)(lo | (hi << 4)) - 32;
    const float d = f16_bits_to_f32(dbits);
    const float w = __fmul_rn(__fmul_rn(d, (float)sc[h * 8u + (l >> 4) + 2u * a]), (float)q);
    p.hidden[b * 256u + t] = w;
    if (p.ids && b == 0 && t == 0) {
        p.ids[*p.step] = tok;
        *p.step += 1u;
    }
}

// softmax_inplace (attention.rs:45-73) of one vector by one CTA: the maximum
// (any order gives the strict-'>' scan's value), exp(v - max) with glibc's
// expf, the sequential sum, then v * (1 / sum); a non-finite maximum
// gives zeros, a sum that is not positive leaves the exponentials.  Dynamic
// shared memory: n floats, then exact_sum_scratch_bytes(512).
__global__ void __launch_bounds__(512) softmax_kernel(float *__restrict__ x, uint32_t n) {
    extern __shared__ __align__(16) float e[];
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    float m = -INFINITY;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        e[i] = x[i];
        m = fmaxf(m, e[i]);
    }
    const float mx = block_max(m, red);
    if (!isfinite(mx)) {
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) x[i] = 0.0f;
        return;
    }
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) e[i] = glibc_expf(__fsub_rn(e[i], mx));
    __syncthreads();
    const float sum = cta_exact_sum_nonneg(e, n, reinterpret_cast<uint8_t *>(e + ((n + 1u) & ~1u)));
    const bool norm = sum > 0.0f;
    const float inv = norm ? __fdiv_rn(1.0f, sum) : 1.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) x[i] = norm ? __fmul_rn(e[i], inv) : e[i];
}

// ---------------------------------------------------------------------------
// Final RMSNorm (one CTA), then the position advances: the step is done.
struct OutNormParams {
    const float *hidden;
    const float *w;
    float *out;
    uint32_t n;
    float eps;
    uint32_t *pos;
    uint32_t exact;  // sequential sum of squares (the reference's order)
};

// Exact-mode sum of squares of x[0..n) (n a multiple of 4, x 16-byte
// aligned): the CTA stores the squares into shared memory `buf` (one round of
// loads, one rounding per square), then forms their sum in the reference's
// order (cta_exact_sum_nonneg; scratch: exact_sum_scratch_bytes(blockDim.x)
// bytes of shared memory).
__device__ __forceinline__ float block_seq_sum_sq(const float *x, uint32_t n, float *buf,
                                                  uint8_t *scratch) {
    for (uint32_t i = threadIdx.x * 4u; i < n; i += blockDim.x * 4u) {
        const float4 v = *reinterpret_cast<const float4 *>(x + i);
        *reinterpret_cast<float4 *>(buf + i) = make_float4(
            __fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y), __fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w));
    }
    __syncthreads();
    return cta_exact_sum_nonneg(buf, n, scratch);
}

// rms_norm_f32 (primitives.rs:227-255) of one vector by one CTA:
// mean = sum(x*x) / n (the reference's sequential sum, bit for bit),
// rsqrt = 1 / sqrt(mean + eps), out = (x * rsqrt) * w.  Dynamic shared
// memory: n floats, then exact_sum_scratch_bytes(256).
__global__ void __launch_bounds__(256) rms_norm_kernel(const float *__restrict__ x,
                                                        const float *__restrict__ w, uint32_t n,
                                                        float eps, float *__restrict__ out) {
    extern __shared__ __align__(16) float sq[];
    pdl_launch_dependents();
    pdl_wait();
    const float sum_sq = block_seq_sum_sq(x, n, sq, reinterpret_cast<uint8_t *>(sq + n));
    const float mean = __fdiv_rn(sum_sq, (float)n);
    const float rsqrt = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], rsqrt), w[i]);
}

constexpr uint32_t OUT_NORM_MAX = 8192;  // shared-memory copy of the exact-mode input

__global__ void __launch_bounds__(256) out_norm_kernel(const __grid_constant__ OutNormParams p) {
    __shared__ float red[32];
    __shared__ __align__(16) float hs[OUT_NORM_MAX];
    __shared__ __align__(16) uint8_t xscr[exact_sum_scratch_bytes(256)];
    pdl_launch_dependents();
    pdl_wait();
    float sum_sq;
    if (p.exact) {
        sum_sq = block_seq_sum_sq(p.hidden, p.n, hs, xscr);
    } else {
        float ss = 0.0f;
        for (uint32_t i = threadIdx.x; i < p.n; i += blockDim.x)
            ss = __fadd_rn(ss, __fmul_rn(p.hidden[i], p.hidden[i]));
        sum_sq = block_sum(ss, red);
    }
    const float mean = __fdiv_rn(sum_sq, (float)p.n);
    const float rsqrt = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
    // distinct buffers: the loads of one pass need not wait for its stores
    const float *__restrict__ h = p.hidden;
    const float *__restrict__ w = p.w;
    float *__restrict__ o = p.out;
    for (uint32_t i = threadIdx.x; i < p.n; i += blockDim.x) o[i] = __fmul_rn(__fmul_rn(h[i], rsqrt), w[i]);
    __syncthreads();
    if (threadIdx.x == 0) *p.pos += 1u;
}

// ---------------------------------------------------------------------------
// Attention for one decode position, split over positions (grid: heads x
// splits x sequences; the last CTA of a head combines the splits).
//  1. RoPE (NEOX pairs for BitNet, Norm pairs for VanillaLlama,
//     cached_forward.rs:505-509) on every K head (every CTA, redundantly) and
//     on this CTA's Q head, from the host-filled (cos, sin) table.
//  2. Per-token absmax i8 quantisation of K and V (kv_cache.rs:245-259);
//     CTA (0, 0) appends them to the cache, every CTA keeps its own copy for
//     the current position (no cross-CTA dependency on the new entry).
//  3. scores[t] = (q . k_t) * scale, k_t = (f32)k8 * s_t, one thread per
//     position summing over the head in the reference's order (bit-exact
//     scores); per split: local max m, e = exp(s - m), l = sum e,
//     o = sum e * v_t.  Combine: M = max m, w = e * exp(m - M) / sum(l *
//     exp(m - M)) -- the reference's softmax (attention.rs:45-73) up to
//     rounding; a non-finite maximum gives zeros, as there.
struct AttnParams {
    const float *q, *k, *v;  // this step's projections: E, KV, KV
    float *att;              // E
    int8_t *k_cache, *v_cache;  // this layer: [max_seq][KV]
    float *k_scale, *v_scale;   // this layer: [max_seq]
    const float2 *rope;         // [max_seq][n_rot / 2] (cos, sin)
    const uint32_t *pos;
    uint32_t n_kv_heads, head_dim, n_rot, max_seq, group, splits;
    float scale;
    float *partial;             // [n_heads][splits][head_dim + 4]: o, max, sum
    uint32_t *counters;         // [n_heads], zero between launches
    uint32_t *status;
    uint32_t exact;             // splits == 1: softmax and V sums in the reference's order
    // Batched sequences (grid z): sequence z reads q / k / v at + z * qkv_stride,
    // writes att + z * att_stride, its cache at + z * cache_stride (scales
    // + z * scale_stride), its position pos[z], partials / counters of its own;
    // a zero active[z] skips the sequence.  One sequence: zeros / null.
    uint32_t qkv_stride, att_stride, scale_stride;
    size_t cache_stride;
    const uint32_t *active;
    uint32_t rope_pairs;        // 0: NEOX (j, j + n_rot/2); 1: Norm (2j, 2j + 1)
    uint32_t chunk;             // attn_gqa_batch_kernel: positions per split (grid z covers
                                // max_seq); a sequence uses ceil((pos + 1) / chunk) splits
    // Tensor parallel: q / k / v were gathered from every rank's row slice;
    // with tp.wait set, every CTA first waits (bounded) for every rank's stores.
    TpParams tp;
    // attn_exact_kernel: *pos was written well before the previous kernel
    // (a previous step), so the cache history may be staged before the
    // programmatic-dependency wait.
    uint32_t pos_stable;
    // attn_exact_kernel, batched: grid z index -> sequence (null: identity).
    // The engine lists the longest contexts first, so that their CTAs, the
    // longest-running, are dispatched first and the short ones fill in.
    const uint32_t *seq_order;
};

__device__ __forceinline__ void kv_quantise_block(const float *x, uint32_t n, int8_t *q,
                                                  float *scale_out, float *red) {
    float m = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, fabsf(x[i]));
    const float absmax = block_max(m, red);
    const bool zero = absmax == 0.0f || !isfinite(absmax);
    const float inv = zero ? 0.0f : __fdiv_rn(127.0f, absmax);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        int qi = 0;
        if (!zero) {
            qi = quant_round_i8(__fmul_rn(x[i], inv));
        }
        q[i] = (int8_t)qi;
    }
    if (threadIdx.x == 0) *scale_out = zero ? 0.0f : __fdiv_rn(absmax, 127.0f);
}

// f32::exp of the reference: glibc's expf, restated bit for bit.
__device__ __forceinline__ float exp_f32(float x) { return glibc_expf(x); }

// A cached K / V element as f32: (f32)q * s for the int8 layout, the exact
// value of the half for the f16 layout (s unused).
template <bool F16>
__device__ __forceinline__ float kv_value(typename std::conditional<F16, uint16_t, int8_t>::type raw,
                                          float s) {
    if constexpr (F16) return __half2float(__ushort_as_half(raw));
    else return __fmul_rn((float)raw, s);
}

// F16: the cache holds K and V as IEEE binary16 (round to nearest even from
// the f32 values; no scales) instead of the reference's per-token absmax
// int8 -- the KV layout of benchmark config 2.  Every read converts back to
// f32 exactly; the arithmetic around it is the int8 path's with the
// dequantised value (f32)k8 * s replaced by the f16 value.
template <bool F16>
__global__ void __launch_bounds__(ATTN_THREADS) attn_decode_kernel(const __grid_constant__ AttnParams p) {
    using KvT = typename std::conditional<F16, uint16_t, int8_t>::type;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[32];
    __shared__ float s_ks, s_vs;
    __shared__ uint32_t s_last;
    const uint32_t HD = p.head_dim, KV = p.n_kv_heads * HD, half = p.n_rot / 2u;
    const uint32_t h = blockIdx.x, sp = blockIdx.y, kvh = h / p.group, tid = threadIdx.x;
    // float regions rounded to 4 floats so the int8 rows after them stay 16-byte aligned
    const uint32_t chunk_max = ((p.max_seq + p.splits - 1) / p.splits + 3u) & ~3u;
    float *ks = reinterpret_cast<float *>(smem);  // KV: rotated k
    float *vs = ks + KV;                          // KV: v
    float *qh = vs + KV;                          // HD: rotated q of this head
    float *obuf = qh + HD;                        // ATTN_THREADS: partial outputs
    float *scores = obuf + ATTN_THREADS;          // chunk_max
    float *vsc = scores + chunk_max;              // chunk_max: V scales of the split
    float2 *rope = reinterpret_cast<float2 *>(vsc + chunk_max);  // half (rounded to 2)
    float *comb = reinterpret_cast<float *>(rope + ((half + 1u) & ~1u));  // splits*(2+HD)
    KvT *kq = reinterpret_cast<KvT *>(comb + ((p.splits * (2u + HD) + 3u) & ~3u));  // KV
    KvT *vq = kq + KV;                                                              // KV

    pdl_launch_dependents();
    pdl_wait();
    if (p.tp.world && p.tp.wait) {
        if (tid == 0 && !tp_wait(p.tp)) atomicOr(p.status, WL_DEV_ERR_PEER_TIMEOUT);
        __syncthreads();
    }
    const uint32_t z = blockIdx.z;
    if (p.active && !p.active[z]) return;
    const uint32_t pos = p.pos[z];
    if (pos >= p.max_seq) {
        if (tid == 0) atomicOr(p.status, WL_DEV_ERR_POSITION);
        return;
    }
    const float *q_in = p.q + (size_t)z * p.qkv_stride, *k_in = p.k + (size_t)z * p.qkv_stride,
                *v_in = p.v + (size_t)z * p.qkv_stride;
    float *att = p.att + (size_t)z * p.att_stride;
    KvT *k_cache = reinterpret_cast<KvT *>(p.k_cache) + z * p.cache_stride;
    KvT *v_cache = reinterpret_cast<KvT *>(p.v_cache) + z * p.cache_stride;
    float *k_scale = p.k_scale + (size_t)z * p.scale_stride,
          *v_scale = p.v_scale + (size_t)z * p.scale_stride;
    float *partial = p.partial + (size_t)z * gridDim.x * p.splits * (HD + 4u);
    uint32_t *counters = p.counters + (size_t)z * gridDim.x;
    // one round of independent loads: k, v, this head's q, the RoPE row
    const float2 *cs = p.rope + (size_t)pos * half;
    for (uint32_t i = tid; i < KV; i += blockDim.x) {
        ks[i] = k_in[i];
        vs[i] = v_in[i];
    }
    for (uint32_t i = tid; i < HD; i += blockDim.x) qh[i] = q_in[h * HD + i];
    for (uint32_t j = tid; j < half; j += blockDim.x) rope[j] = cs[j];
    __syncthreads();
    // pair (i0, i1) of rotation j: NEOX (j, j + half), Norm (2j, 2j + 1)
    const uint32_t pstep = p.rope_pairs ? 2u : 1u, poff = p.rope_pairs ? 1u : half;
    for (uint32_t i = tid; i < p.n_kv_heads * half; i += blockDim.x) {
        const uint32_t hk = i / half, j = i % half;
        float *x = ks + hk * HD;
        const uint32_t i0 = j * pstep, i1 = i0 + poff;
        const float a = x[i0], b = x[i1], c = rope[j].x, s = rope[j].y;
        x[i0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        x[i1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
    for (uint32_t j = tid; j < half; j += blockDim.x) {
        const uint32_t i0 = j * pstep, i1 = i0 + poff;
        const float a = qh[i0], b = qh[i1], c = rope[j].x, s = rope[j].y;
        qh[i0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        qh[i1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
    __syncthreads();
    if constexpr (F16) {
        for (uint32_t i = tid; i < KV; i += blockDim.x) {
            kq[i] = __half_as_ushort(__float2half_rn(ks[i]));
            vq[i] = __half_as_ushort(__float2half_rn(vs[i]));
        }
        if (tid == 0) s_ks = s_vs = 1.0f;  // no scales: the dequantised value is the f16's
    } else {
        kv_quantise_block(ks, KV, kq, &s_ks, red);
        kv_quantise_block(vs, KV, vq, &s_vs, red);
    }
    __syncthreads();
    if (h == 0 && sp == 0) {
        for (uint32_t i = tid; i < KV; i += blockDim.x) {
            k_cache[(size_t)pos * KV + i] = kq[i];
            v_cache[(size_t)pos * KV + i] = vq[i];
        }
        if (!F16 && tid == 0) {
            k_scale[pos] = s_ks;
            v_scale[pos] = s_vs;
        }
    }
    // this split's positions [t0, t1)
    const uint32_t n = pos + 1u, chunk = (n + p.splits - 1u) / p.splits;
    const uint32_t t0 = min(n, sp * chunk), t1 = min(n, t0 + chunk), cnt = t1 - t0;
    // scores: one thread per position, the head's row loaded whole first
    // (one memory round trip), then summed in the reference's order
    for (uint32_t i = tid; i < cnt && F16; i += blockDim.x) {
        // f16 rows: q . k with k the exact f32 of each half, in order
        const uint32_t t = t0 + i;
        const uint16_t *kr = reinterpret_cast<const uint16_t *>(
            t == pos ? kq + kvh * HD : k_cache + (size_t)t * KV + kvh * HD);
        float d = 0.0f;
        for (uint32_t c = 0; c < HD; c += 32u) {
            uint4 w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) w[j] = *reinterpret_cast<const uint4 *>(kr + c + 8u * j);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t wv[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float kf = __half2float(__ushort_as_half((uint16_t)(wv[e >> 1] >> (16 * (e & 1)))));
                    d = __fadd_rn(d, __fmul_rn(qh[c + 8u * j + e], kf));
                }
            }
        }
        scores[i] = __fmul_rn(d, p.scale);
        vsc[i] = 1.0f;
    }
    for (uint32_t i = tid; i < cnt && !F16; i += blockDim.x) {
        const uint32_t t = t0 + i;
        const int8_t *kr = reinterpret_cast<const int8_t *>(
            t == pos ? kq + kvh * HD : k_cache + (size_t)t * KV + kvh * HD);
        const float sk = t == pos ? s_ks : k_scale[t];
        vsc[i] = t == pos ? s_vs : v_scale[t];
        uint4 w[16];
#pragma unroll
        for (int c = 0; c < 16; ++c)
            if ((uint32_t)c * 16u < HD) w[c] = *reinterpret_cast<const uint4 *>(kr + c * 16);
        float d = 0.0f;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            if ((uint32_t)c * 16u >= HD) break;
            const uint32_t wv[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const float kv8 = (float)(int8_t)(wv[e >> 2] >> (8 * (e & 3)));
                d = __fadd_rn(d, __fmul_rn(qh[c * 16 + e], __fmul_rn(kv8, sk)));
            }
        }
        scores[i] = __fmul_rn(d, p.scale);
    }
    __syncthreads();
    if (p.exact) {
        // softmax_inplace (attention.rs:45-73) and out_h[d] += w * v_h[d]
        // (cached_forward.rs:441-449) in the reference's sequential order.
        // The maximum as a block reduction: the same value as the reference's
        // strict-'>' scan (NaN never wins either way; +0 and -0 maxima give
        // identical exponentials).  The sums below keep the reference's order,
        // with their loads run ahead of the dependent adds.
        __shared__ float s_inv;
        __shared__ uint32_t s_norm;
        float mloc = -INFINITY;
        for (uint32_t i = tid; i < cnt; i += blockDim.x) mloc = fmaxf(mloc, scores[i]);
        const float mxs = block_max(mloc, red);
        if (!isfinite(mxs)) {
            for (uint32_t i = tid; i < cnt; i += blockDim.x) scores[i] = 0.0f;
        } else {
            for (uint32_t i = tid; i < cnt; i += blockDim.x)
                scores[i] = exp_f32(__fsub_rn(scores[i], mxs));
            __syncthreads();
            if (tid == 0) {
                float sum = 0.0f;
                {
                    const uint32_t n4 = (cnt & ~31u) / 4u;
                    const float4 *x4 = reinterpret_cast<const float4 *>(scores);
                    for (uint32_t i = 0; i < n4; i += 8) {
                        float4 c8[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) c8[j] = x4[i + j];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            sum = __fadd_rn(sum, c8[j].x); sum = __fadd_rn(sum, c8[j].y);
                            sum = __fadd_rn(sum, c8[j].z); sum = __fadd_rn(sum, c8[j].w);
                        }
                    }
                    for (uint32_t i = n4 * 4u; i < cnt; ++i) sum = __fadd_rn(sum, scores[i]);
                }
                s_norm = sum > 0.0f ? 1u : 0u;
                s_inv = s_norm ? __fdiv_rn(1.0f, sum) : 1.0f;
            }
            __syncthreads();
            if (s_norm)
                for (uint32_t i = tid; i < cnt; i += blockDim.x) scores[i] = __fmul_rn(scores[i], s_inv);
        }
        __syncthreads();
        if (tid < HD) {
            float o = 0.0f;
            const KvT *vcol = v_cache + (size_t)t0 * KV + kvh * HD + tid;
            const KvT vcur = vq[kvh * HD + tid];
            for (uint32_t i0 = 0; i0 < cnt; i0 += 32u) {
                KvT vb[32];
#pragma unroll
                for (uint32_t u = 0; u < 32u; ++u)
                    vb[u] = (i0 + u < cnt && t0 + i0 + u != pos) ? vcol[(size_t)(i0 + u) * KV] : vcur;
#pragma unroll
                for (uint32_t u = 0; u < 32u; ++u)
                    if (i0 + u < cnt)
                        o = __fadd_rn(o, __fmul_rn(scores[i0 + u], kv_value<F16>(vb[u], vsc[i0 + u])));
            }
            att[h * HD + tid] = o;
        }
        return;
    }
    float m = -INFINITY;
    for (uint32_t i = tid; i < cnt; i += blockDim.x) m = fmaxf(m, scores[i]);
    const float mx = block_max(m, red);
    float lsum = 0.0f;
    const bool finite = isfinite(mx);
    if (finite) {
        for (uint32_t i = tid; i < cnt; i += blockDim.x) {
            const float e = exp_f32(__fsub_rn(scores[i], mx));
            scores[i] = e;
            lsum = __fadd_rn(lsum, e);
        }
    }
    const float l = block_sum(lsum, red);
    __syncthreads();
    // out[d] = sum_i e_i * ((f32)v8 * s): groups of HD threads split the
    // positions; 8 independent row loads per round trip
    const uint32_t groups = blockDim.x / HD, d = tid % HD, g = tid / HD;
    float acc = 0.0f;
    if (finite && g < groups) {
        const KvT *vbase = v_cache + (size_t)kvh * HD + d;
        for (uint32_t i0 = g; i0 < cnt; i0 += 8u * groups) {
            KvT vv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint32_t i = i0 + (uint32_t)u * groups;
                const uint32_t t = t0 + i;
                vv[u] = i >= cnt ? (KvT)0 : (t == pos ? vq[kvh * HD + d] : vbase[(size_t)t * KV]);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint32_t i = i0 + (uint32_t)u * groups;
                if (i < cnt) acc = __fadd_rn(acc, __fmul_rn(scores[i], kv_value<F16>(vv[u], vsc[i])));
            }
        }
    }
    obuf[tid] = acc;
    __syncthreads();
    float *part = partial + ((size_t)h * p.splits + sp) * (HD + 4u);  // o[HD], max, sum
    if (tid < HD) {
        float o = obuf[tid];
        for (uint32_t gg = 1; gg < groups; ++gg) o = __fadd_rn(o, obuf[gg * HD + tid]);
        part[tid] = o;
    }
    if (tid == 0) {
        part[HD] = mx;
        part[HD + 1] = l;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(counters + h, 1u) == p.splits - 1u ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // last CTA of the head: warp 0 reduces the splits' maxima and sums and
    // keeps the factors exp(m - M) in comb; then HD/4 threads combine the o
    // rows with float4 loads, eight splits per round of loads.
    const uint32_t S = p.splits, RS = HD + 4u;
    const float *base = partial + (size_t)h * S * RS;
    if (tid < 32) {
        float M = -INFINITY;
        for (uint32_t s2 = tid; s2 < S; s2 += 32u) M = fmaxf(M, __ldcg(base + s2 * RS + HD));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        const bool fin = isfinite(M);
        float L = 0.0f;
        for (uint32_t s2 = tid; s2 < S; s2 += 32u) {
            const float ms = __ldcg(base + s2 * RS + HD), ls = __ldcg(base + s2 * RS + HD + 1);
            const float f = (fin && ms > -INFINITY) ? exp_f32(__fsub_rn(ms, M)) : 0.0f;
            comb[s2] = f;
            L = __fadd_rn(L, __fmul_rn(ls, f));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) L = __fadd_rn(L, __shfl_xor_sync(0xffffffffu, L, off));
        if (tid == 0) {
            red[0] = !fin ? 2.0f : (L > 0.0f ? 1.0f : 0.0f);
            red[1] = L > 0.0f ? __fdiv_rn(1.0f, L) : 1.0f;
        }
    }
    __syncthreads();
    const float mode = red[0], inv = red[1];
    for (uint32_t c = tid; c < HD / 4u; c += blockDim.x) {
        float4 O = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (uint32_t s0 = 0; s0 < S; s0 += 8u) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (s0 + u < S) v[u] = __ldcg(reinterpret_cast<const float4 *>(base + (s0 + u) * RS) + c);
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (s0 + u < S) {
                    const float f = comb[s0 + u];
                    O.x = __fadd_rn(O.x, __fmul_rn(v[u].x, f));
                    O.y = __fadd_rn(O.y, __fmul_rn(v[u].y, f));
                    O.z = __fadd_rn(O.z, __fmul_rn(v[u].z, f));
                    O.w = __fadd_rn(O.w, __fmul_rn(v[u].w, f));
                }
        }
        if (mode == 2.0f) {
            O = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        } else if (mode == 1.0f) {
            O.x = __fmul_rn(O.x, inv);
            O.y = __fmul_rn(O.y, inv);
            O.z = __fmul_rn(O.z, inv);
            O.w = __fmul_rn(O.w, inv);
        }
        reinterpret_cast<float4 *>(att + h * HD)[c] = O;
    }
    if (tid == 0) counters[h] = 0u;  // re-arm for the next launch
}

// ---------------------------------------------------------------------------
// Exact-mode attention, one CTA per (query head, sequence): the reference's
// scaled_dot_product_attention_into (cached_forward.rs:417-449) with
// softmax_inplace (attention.rs:45-73) in its sequential order, bit for bit
// (exp is glibc's expf, restated in glibc_expf.cuh).  The head's whole K and V history
// (int8 rows and scales) is copied into shared memory with cp.async --
// before the programmatic-dependency wait when the position is not written
// by the kernels just before this one -- so the three sequential sums
// (q.k per position, the softmax sum, and per dimension the weighted V sum)
// read shared memory at the add's latency instead of waiting on global loads.
constexpr int AX_THREADS = 512;

__host__ __device__ inline uint32_t ax_cap(uint32_t max_seq) { return (max_seq + 3u) & ~3u; }
// The K history region also holds the softmax sum's scratch (at least
// exact_sum_scratch_bytes(AX_THREADS) bytes).
__host__ __device__ inline uint32_t ax_kcap(uint32_t max_seq) {
    constexpr uint32_t need = (exact_sum_scratch_bytes(AX_THREADS) / 32u + 3u) & ~3u;  // head_dim >= 32
    const uint32_t c = ax_cap(max_seq);
    return c > need ? c : need;
}

inline size_t attn_exact_smem_bytes(uint32_t kv, uint32_t hd, uint32_t max_seq) {
    const size_t cap = ax_cap(max_seq), kcap = ax_kcap(max_seq);
    const size_t half2 = ((hd / 2u + 1u) & ~1u) * 2u;  // float2 RoPE row, in floats
    return (kcap + cap) * hd + 3 * cap * 4 + (2 * (size_t)kv + hd + half2) * 4 + 2 * (size_t)kv;
}

// int8 -> exact float without the conversion unit: (2^23 + (b + 128)) -
// (2^23 + 128), where b + 128 = (unsigned byte) ^ 0x80.  Byte j (0..3) of a
// word already XORed with 0x80808080, or one byte.
__device__ __forceinline__ float i8_byte_to_f32(uint32_t w_xor80, uint32_t j) {
    return __fsub_rn(__uint_as_float(__byte_perm(w_xor80, 0x4B000000u, 0x7540u + j)), 8388736.0f);
}
__device__ __forceinline__ float i8_to_f32(int8_t b) {
    return __fsub_rn(__uint_as_float(((uint32_t)(uint8_t)b ^ 0x80u) | 0x4B000000u), 8388736.0f);
}

// Shared-memory accesses by 32-bit shared address (ld/st.shared): the V
// phase below indexes its buffers through computed offsets, and generic
// 64-bit addressing there cost about twice the time.
__device__ __forceinline__ float lds_f32(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds_u32x2(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts_f32x4(uint32_t a, float x, float y, float z, float w) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(x), "f"(y), "f"(z), "f"(w)
                 : "memory");
}

// Shared-memory layout (cap = max_seq rounded up to 4, kcap >= cap):
//   Ksm [kcap][HD] int8   K history; row t's 16-byte piece c sits at piece
//                         c ^ (t & smask), so the 8 rows a quarter-warp reads
//                         at once hit 8 different bank groups; after the
//                         scores the region is the softmax sum's scratch
//   Vsm [cap][HD] int8    V history, natural order
//   ksc, vsc, sc [cap]    K / V scales, scores then softmax weights
//   kf, vf [KV], qh [HD], rope [half (even)], kq, vq [KV]
__global__ void __launch_bounds__(AX_THREADS) attn_exact_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[32];
    __shared__ float s_ks, s_vs, s_inv;
    __shared__ uint32_t s_norm;
    const uint32_t HD = p.head_dim, KV = p.n_kv_heads * HD, half = p.n_rot / 2u;
    const uint32_t h = blockIdx.x, kvh = h / p.group, tid = threadIdx.x;
    const uint32_t z = p.seq_order ? p.seq_order[blockIdx.z] : blockIdx.z;
    const uint32_t cap = ax_cap(p.max_seq), kcap = ax_kcap(p.max_seq);
    const uint32_t pieces = HD / 16u, smask = (pieces < 8u ? pieces : 8u) - 1u;
    int8_t *Ksm = reinterpret_cast<int8_t *>(smem);
    int8_t *Vsm = Ksm + (size_t)kcap * HD;
    float *ksc = reinterpret_cast<float *>(Vsm + (size_t)cap * HD);
    float *vsc = ksc + cap;
    float *sc = vsc + cap;
    float *kf = sc + cap;
    float *vf = kf + KV;
    float *qh = vf + KV;
    float2 *rope = reinterpret_cast<float2 *>(qh + HD);
    int8_t *kq = reinterpret_cast<int8_t *>(rope + ((half + 1u) & ~1u));
    int8_t *vq = kq + KV;

    const int8_t *k_cache = p.k_cache + z * p.cache_stride;
    const int8_t *v_cache = p.v_cache + z * p.cache_stride;
    const float *k_scale = p.k_scale + (size_t)z * p.scale_stride;
    const float *v_scale = p.v_scale + (size_t)z * p.scale_stride;
    // The head's cached rows [0, pos) and their scales, 16 bytes per copy,
    // and this position's RoPE row: K first (the scores need it), then V in
    // a second copy group (the weighted sum needs it only after the softmax).
    auto stage_history = [&](uint32_t pos) {
        const uint32_t n = pos * pieces;
        for (uint32_t i = tid; i < n; i += AX_THREADS) {
            const uint32_t t = i / pieces, c = i % pieces;
            const size_t g = (size_t)t * KV + kvh * HD + c * 16u;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                             smem_u32(Ksm + t * HD + ((c ^ (t & smask)) * 16u))),
                         "l"(k_cache + g) : "memory");
        }
        for (uint32_t t = tid; t < pos; t += AX_THREADS)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(ksc + t)),
                         "l"(k_scale + t) : "memory");
        const float2 *cs = p.rope + (size_t)pos * half;
        for (uint32_t j = tid; j < half; j += AX_THREADS)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(rope + j)),
                         "l"(cs + j) : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
        for (uint32_t i = tid; i < n; i += AX_THREADS) {
            const uint32_t t = i / pieces, c = i % pieces;
            const size_t g = (size_t)t * KV + kvh * HD + c * 16u;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(Vsm + t * HD + c * 16u)),
                         "l"(v_cache + g) : "memory");
        }
        for (uint32_t t = tid; t < pos; t += AX_THREADS)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(vsc + t)),
                         "l"(v_scale + t) : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    uint32_t pos = 0;
    bool staged = false;
    if (p.pos_stable && !p.active) {
        pos = __ldcg(p.pos + z);
        if (pos < p.max_seq) {
            stage_history(pos);
            staged = true;
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    if (p.tp.world && p.tp.wait) {
        if (tid == 0 && !tp_wait(p.tp)) atomicOr(p.status, WL_DEV_ERR_PEER_TIMEOUT);
        __syncthreads();
    }
    if (p.active && !p.active[z]) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        return;
    }
    if (!staged) {
        pos = p.pos[z];
        if (pos < p.max_seq) stage_history(pos);
    }
    if (pos >= p.max_seq) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        if (tid == 0) atomicOr(p.status, WL_DEV_ERR_POSITION);
        return;
    }
    const float *q_in = p.q + (size_t)z * p.qkv_stride, *k_in = p.k + (size_t)z * p.qkv_stride,
                *v_in = p.v + (size_t)z * p.qkv_stride;
    float *att = p.att + (size_t)z * p.att_stride;
    for (uint32_t i = tid; i < KV / 4u; i += AX_THREADS) {  // KV, HD multiples of 32
        reinterpret_cast<float4 *>(kf)[i] = reinterpret_cast<const float4 *>(k_in)[i];
        reinterpret_cast<float4 *>(vf)[i] = reinterpret_cast<const float4 *>(v_in)[i];
    }
    for (uint32_t i = tid; i < HD / 4u; i += AX_THREADS)
        reinterpret_cast<float4 *>(qh)[i] = reinterpret_cast<const float4 *>(q_in + h * HD)[i];
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // K history and RoPE row
    __syncthreads();
    // RoPE on every K head (the K quantisation takes the absmax of all of
    // them) and on this query head: pair (i0, i1) = NEOX (j, j + half) or
    // Norm (2j, 2j + 1).
    const uint32_t pstep = p.rope_pairs ? 2u : 1u, poff = p.rope_pairs ? 1u : half;
    for (uint32_t i = tid; i < p.n_kv_heads * half; i += AX_THREADS) {
        const uint32_t hk = i / half, j = i % half;
        float *x = kf + hk * HD;
        const uint32_t i0 = j * pstep, i1 = i0 + poff;
        const float a = x[i0], b = x[i1], c = rope[j].x, sn = rope[j].y;
        x[i0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
        x[i1] = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
    }
    for (uint32_t j = tid; j < half; j += AX_THREADS) {
        const uint32_t i0 = j * pstep, i1 = i0 + poff;
        const float a = qh[i0], b = qh[i1], c = rope[j].x, sn = rope[j].y;
        qh[i0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
        qh[i1] = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
    }
    __syncthreads();
    // Per-token absmax i8 quantisation of K and V (kv_cache.rs:245-259), both
    // maxima in one block reduction.
    {
        float mk = 0.0f, mv = 0.0f;
        for (uint32_t i = tid; i < KV; i += AX_THREADS) {
            mk = fmaxf(mk, fabsf(kf[i]));
            mv = fmaxf(mv, fabsf(vf[i]));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, off));
            mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, off));
        }
        if ((tid & 31) == 0) {
            red[tid >> 5] = mk;
            red[16 + (tid >> 5)] = mv;
        }
        __syncthreads();
        mk = red[0];
        mv = red[16];
        for (uint32_t w = 1; w < AX_THREADS / 32; ++w) {
            mk = fmaxf(mk, red[w]);
            mv = fmaxf(mv, red[16 + w]);
        }
        const bool zk = mk == 0.0f || !isfinite(mk), zv = mv == 0.0f || !isfinite(mv);
        const float ik = zk ? 0.0f : __fdiv_rn(127.0f, mk), iv = zv ? 0.0f : __fdiv_rn(127.0f, mv);
        for (uint32_t i = tid; i < KV; i += AX_THREADS) {
            kq[i] = (int8_t)(zk ? 0 : quant_round_i8(__fmul_rn(kf[i], ik)));
            vq[i] = (int8_t)(zv ? 0 : quant_round_i8(__fmul_rn(vf[i], iv)));
        }
        if (tid == 0) {
            s_ks = zk ? 0.0f : __fdiv_rn(mk, 127.0f);
            s_vs = zv ? 0.0f : __fdiv_rn(mv, 127.0f);
        }
    }
    __syncthreads();
    if (h == 0) {  // one CTA per sequence appends the position to the cache
        int8_t *kc = p.k_cache + z * p.cache_stride, *vc = p.v_cache + z * p.cache_stride;
        for (uint32_t i = tid; i < KV / 4u; i += AX_THREADS) {
            reinterpret_cast<uint32_t *>(kc + (size_t)pos * KV)[i] = reinterpret_cast<const uint32_t *>(kq)[i];
            reinterpret_cast<uint32_t *>(vc + (size_t)pos * KV)[i] = reinterpret_cast<const uint32_t *>(vq)[i];
        }
        if (tid == 0) {
            p.k_scale[(size_t)z * p.scale_stride + pos] = s_ks;
            p.v_scale[(size_t)z * p.scale_stride + pos] = s_vs;
        }
    }
    // scores[t] = (sum_d q[d] * ((f32)k8[t][d] * s_t)) * scale, d in order,
    // one thread per position.  The int8 -> f32 conversion and the two
    // products run as packed pairs (each lane rounded as the scalar
    // operation); the dependent adds stay scalar, in order (a packed product
    // feeding a packed add could be contracted into one FMA).
    const uint32_t n = pos + 1u;
    const float2 cbias = make_float2(-8388736.0f, -8388736.0f);
    for (uint32_t t = tid; t < n; t += AX_THREADS) {
        const bool hist = t < pos;
        const int8_t *kr = hist ? Ksm + (size_t)t * HD : kq + kvh * HD;
        const uint32_t sw = hist ? (t & smask) : 0u;
        const float sk = hist ? ksc[t] : s_ks;
        const float2 sk2 = make_float2(sk, sk);
        float d = 0.0f;
        for (uint32_t c = 0; c < pieces; ++c) {
            const uint4 w = *reinterpret_cast<const uint4 *>(kr + ((c ^ sw) * 16u));
            const uint32_t wv[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u,
                                    w.w ^ 0x80808080u};
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
                const uint32_t wd = wv[e >> 2];
                const float2 kv8 = f2_add_rn(
                    make_float2(__uint_as_float(__byte_perm(wd, 0x4B000000u, 0x7540u + (e & 3))),
                                __uint_as_float(__byte_perm(wd, 0x4B000000u, 0x7541u + (e & 3)))),
                    cbias);
                const float2 qk = f2_mul_rn(*reinterpret_cast<const float2 *>(qh + c * 16u + e),
                                            f2_mul_rn(kv8, sk2));
                d = __fadd_rn(d, qk.x);
                d = __fadd_rn(d, qk.y);
            }
        }
        sc[t] = __fmul_rn(d, p.scale);
    }
    __syncthreads();
    // softmax_inplace: the maximum (a block reduction gives the strict-'>'
    // scan's value: NaN never wins, and +0 / -0 maxima give the same
    // exponentials), exp, the sequential sum, the scaling by 1 / sum.
    float mloc = -INFINITY;
    for (uint32_t t = tid; t < n; t += AX_THREADS) mloc = fmaxf(mloc, sc[t]);
    const float mx = block_max(mloc, red);
    if (!isfinite(mx)) {
        for (uint32_t t = tid; t < n; t += AX_THREADS) sc[t] = 0.0f;
    } else {
        for (uint32_t t = tid; t < n; t += AX_THREADS) sc[t] = exp_f32(__fsub_rn(sc[t], mx));
        __syncthreads();
        // the reference's sequential sum; the K region is free after the scores
        const float sum = cta_exact_sum_nonneg(sc, n, reinterpret_cast<uint8_t *>(Ksm));
        if (tid == 0) {
            s_norm = sum > 0.0f ? 1u : 0u;
            s_inv = s_norm ? __fdiv_rn(1.0f, sum) : 1.0f;
        }
        __syncthreads();
        if (s_norm)
            for (uint32_t t = tid; t < n; t += AX_THREADS) sc[t] = __fmul_rn(sc[t], s_inv);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");  // the V history is in
    __syncthreads();
    // out[d] = 0 + sum_t w_t * ((f32)v8[t][d] * s_t), t in order.  HD threads
    // add (one per d, a shared-memory load and an add per position) while the
    // other warps form the next block of B positions' products into the K
    // region (free after the softmax), double-buffered, one barrier per
    // block.  (One thread per d forming its own products ran at about 29
    // cycles per position with 4 of the 16 warps busy.)
    if (HD <= AX_THREADS / 2u) {
        const uint32_t B = kcap >= 512u ? 64u : kcap >= 256u ? 32u : 16u;  // 8 * B <= kcap
        float *pbuf = reinterpret_cast<float *>(Ksm);
        const uint32_t nb = (pos + B - 1u) / B, q = HD / 8u;
        // producer pr = tid - HD: row pr / q of each pass, dimensions 8 * (pr % q) ..
        // + 7; conversions and products as packed pairs (each lane rounded as
        // the scalar operation; an add feeding a multiply is not contracted)
        const uint32_t pr = tid - HD, rows_pass = (AX_THREADS - HD) / q;
        const uint32_t prow = pr / q, d8 = 8u * (pr % q);
        const float2 cbias = make_float2(-8388736.0f, -8388736.0f);
        const uint32_t pb = smem_u32(pbuf), vb = smem_u32(Vsm), scb = smem_u32(sc), vsb = smem_u32(vsc);
        auto produce = [&](uint32_t b) {
            const uint32_t dst = pb + (b & 1u) * B * HD * 4u + d8 * 4u;
            const uint32_t t0 = b * B, cnt = min(B, pos - t0);
            for (uint32_t tt = prow; tt < cnt; tt += rows_pass) {
                const uint32_t t = t0 + tt;
                const uint2 w = lds_u32x2(vb + t * HD + d8);
                const float st = lds_f32(vsb + 4u * t), wt = lds_f32(scb + 4u * t);
                const uint32_t wx = w.x ^ 0x80808080u, wy = w.y ^ 0x80808080u;
                const float2 s2 = make_float2(st, st), w2 = make_float2(wt, wt);
                float2 r[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t wd = j < 2 ? wx : wy, e = 2u * (j & 1);
                    const float2 v = f2_add_rn(
                        make_float2(__uint_as_float(__byte_perm(wd, 0x4B000000u, 0x7540u + e)),
                                    __uint_as_float(__byte_perm(wd, 0x4B000000u, 0x7541u + e))),
                        cbias);
                    r[j] = f2_mul_rn(w2, f2_mul_rn(v, s2));
                }
                const uint32_t o = dst + tt * HD * 4u;
                sts_f32x4(o, r[0].x, r[0].y, r[1].x, r[1].y);
                sts_f32x4(o + 16u, r[2].x, r[2].y, r[3].x, r[3].y);
            }
        };
        const bool producer = tid >= HD && prow < rows_pass;
        if (producer && nb > 0u) produce(0u);
        __syncthreads();
        float o = 0.0f;
        const uint32_t stride = HD * 4u;
        for (uint32_t b = 0; b < nb; ++b) {
            if (tid < HD) {
                const uint32_t src = pb + (b & 1u) * B * HD * 4u + tid * 4u;
                const uint32_t cnt = min(B, pos - b * B);
                if (cnt == B) {  // 16 loads in flight ahead of the 16 adds that use the previous ones
                    float x[16];
#pragma unroll
                    for (int u = 0; u < 16; ++u) x[u] = lds_f32(src + u * stride);
                    for (uint32_t tt = 16; tt < B; tt += 16) {
                        float y[16];
#pragma unroll
                        for (int u = 0; u < 16; ++u) y[u] = lds_f32(src + (tt + u) * stride);
#pragma unroll
                        for (int u = 0; u < 16; ++u) o = __fadd_rn(o, x[u]);
#pragma unroll
                        for (int u = 0; u < 16; ++u) x[u] = y[u];
                    }
#pragma unroll
                    for (int u = 0; u < 16; ++u) o = __fadd_rn(o, x[u]);
                } else {
                    for (uint32_t tt = 0; tt < cnt; ++tt) o = __fadd_rn(o, lds_f32(src + tt * stride));
                }
            } else if (producer && b + 1u < nb) {
                produce(b + 1u);
            }
            __syncthreads();
        }
        if (tid < HD) {
            o = __fadd_rn(o, __fmul_rn(sc[pos], __fmul_rn(i8_to_f32(vq[kvh * HD + tid]), s_vs)));
            att[h * HD + tid] = o;
        }
        return;
    }
    for (uint32_t d = tid; d < HD; d += AX_THREADS) {
        float o = 0.0f;
        for (uint32_t t = 0; t < pos; ++t)
            o = __fadd_rn(o, __fmul_rn(sc[t], __fmul_rn(i8_to_f32(Vsm[(size_t)t * HD + d]), vsc[t])));
        o = __fadd_rn(o, __fmul_rn(sc[pos], __fmul_rn(i8_to_f32(vq[kvh * HD + d]), s_vs)));
        att[h * HD + d] = o;
    }
}

inline size_t attn_smem_bytes(uint32_t kv, uint32_t hd, uint32_t max_seq, uint32_t splits,
                              bool f16 = false) {
    const uint32_t chunk = ((max_seq + splits - 1) / splits + 3u) & ~3u;
    const uint32_t half2 = ((hd / 2u + 1u) & ~1u) * 2u;  // float2 RoPE row, in floats
    const uint32_t comb = (splits * (2u + hd) + 3u) & ~3u;
    return (size_t)(2 * kv + hd + ATTN_THREADS + 2 * chunk + half2 + comb) * 4u +
           2u * kv * (f16 ? 2u : 1u) + 16u;
}

}  // namespace wl
