// bitnet_mega.cuh -- the whole BitNet b1.58 decode forward (every layer, one
// token) as ONE persistent cooperative kernel: one CTA per SM, grid-wide
// barriers between the dependent phases, and every CTA streams the packed
// weight rows of its next matvec phases into shared memory with bulk copies
// (TMA engine) before it waits at a barrier, so weight streaming overlaps the
// barriers, the norms and the attention instead of sitting on the critical
// path of 150 kernel launches.
//
// Reference step: cached_forward.rs:206-504 (same op order and per-element
// arithmetic as bitnet_decode.cuh, which holds the per-op kernels).
//
// Phases per layer (B = grid barrier):
//   P1  every CTA: x = attn_norm(hidden) (layer 0: of the token's embedding),
//       absmax int8; its rows of [Wq; Wk; Wv] -> qkv               B
//   P2  CTA (h, split): RoPE, K/V quantise (CTA 0 appends the cache), scores
//       and a split-local softmax -> partial (max, sum, sum e*v)     B
//   P3  every CTA: combine all heads -> att, attn_sub_norm, int8; its rows of
//       Wo, residual into hidden                                    B
//   P4  every CTA: ffn_norm(hidden), int8; its rows of [Wgate; Wup]  B
//   P5  every CTA: relu(gate)^2 * up, ffn_sub_norm, int8; its rows of Wdown,
//       residual into hidden (non-finite -> status)                 B
// After the last layer CTA 0 applies output_norm and advances the position.
//
// Weight buffers: A holds the CTA's rows for P1 and P4, B for P3 and P5.  A
// phase's rows are requested as soon as the buffer is free, i.e. one to two
// phases before they are needed.
//
// Barriers: a monotonic 64-bit arrival counter; barrier j of launch n waits
// for (n * per_launch + j + 1) * grid arrivals, with n read from a launch
// counter that CTA 0 bumps after the last barrier.  Every wait is bounded
// (2 s): a timeout sets a status bit and an abort flag that releases every
// other waiter, in-flight copies are drained (bounded), and the kernel ends.
#pragma once

#include <cstdint>

#include "bitnet_decode.cuh"
#include "i2s_matvec.cuh"
#include "wl_ptx.cuh"

namespace wl {

constexpr int MEGA_THREADS = 256;
constexpr int MEGA_LPR = 8;  // lanes per weight row
constexpr uint32_t WL_DEV_ERR_MEGA = 16u;  // a grid barrier or weight copy timed out

struct MegaLayer {
    const uint8_t *w[7];  // q, k, v, o, gate, up, down (packed I2_S, row-major)
    float scale[7];
    const float *norm;    // attn_norm[E], attn_sub_norm[E], ffn_norm[E], ffn_sub_norm[F]
};

struct MegaParams {
    const MegaLayer *layers;
    uint32_t n_layers, E, F, KV, HD, n_heads, group, n_rot, max_seq, splits;
    float eps, scale;
    uint32_t exact;
    // embedding (repacked Q6_K rows) and the token
    const uint8_t *q6k;
    uint32_t nb, q6k_stride;
    const uint32_t *token;
    uint32_t *ids, *step;   // optional commit of the token
    // activations
    float *hidden, *qkv, *gu, *att, *final_h;
    float *partial;         // [n_heads][splits][HD + 4]: o[HD], max, sum
    const float *out_norm;
    // KV cache
    int8_t *kq, *vq;
    float *ks, *vs;
    const float2 *rope;
    uint32_t *pos;
    // barrier state
    unsigned long long *arrivals;
    uint32_t *launches, *abort;
    uint32_t *status;
    // shared-memory layout
    uint32_t buf_a, buf_b, norm_a, norm_b, xs_off, qs_off, att_off, cmb_off, hloc_off;
};

struct MegaShared {
    uint64_t bar[2];  // weight buffers A, B
    float red[32];
    float s_scale, s_ks, s_vs;
    uint32_t s_flag;
};

// ---------------------------------------------------------------------------
// Global (L2, written by other CTAs) -> shared copies with all of a thread's
// loads issued before its stores: with generic pointers the compiler cannot
// prove the two do not alias, and an interleaved loop would pay one L2 round
// trip per element.  K is a multiple of 4; pointers 16-byte aligned.
__device__ __forceinline__ void stage_f32(float *__restrict__ dst, const float *__restrict__ src,
                                          uint32_t K) {
    const uint32_t n4 = K / 4u, tid = threadIdx.x, T = blockDim.x;
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 *d4 = reinterpret_cast<float4 *>(dst);
    for (uint32_t i0 = tid; i0 < n4; i0 += 8u * T) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (i0 + u * T < n4) v[u] = __ldcg(s4 + i0 + u * T);
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (i0 + u * T < n4) d4[i0 + u * T] = v[u];
    }
}

// xs = relu(gate)^2 * up (ffn.rs:37-65), same load discipline.
__device__ __forceinline__ void stage_relu2_mul(float *__restrict__ dst,
                                                const float *__restrict__ gate,
                                                const float *__restrict__ up, uint32_t K) {
    const uint32_t n4 = K / 4u, tid = threadIdx.x, T = blockDim.x;
    const float4 *g4 = reinterpret_cast<const float4 *>(gate);
    const float4 *u4 = reinterpret_cast<const float4 *>(up);
    float4 *d4 = reinterpret_cast<float4 *>(dst);
    for (uint32_t i0 = tid; i0 < n4; i0 += 4u * T) {
        float4 g[4], v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (i0 + u * T < n4) {
                g[u] = __ldcg(g4 + i0 + u * T);
                v[u] = __ldcg(u4 + i0 + u * T);
            }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (i0 + u * T < n4) {
                float e[4] = {g[u].x, g[u].y, g[u].z, g[u].w};
                const float f[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float r = e[c] > 0.0f ? e[c] : 0.0f;
                    e[c] = __fmul_rn(__fmul_rn(r, r), f[c]);
                }
                d4[i0 + u * T] = make_float4(e[0], e[1], e[2], e[3]);
            }
    }
}

// ---------------------------------------------------------------------------
// Grid barrier (bounded).  Returns false when the grid must stop.
__device__ __forceinline__ uint64_t ld_acquire_gpu_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ bool mega_barrier(const MegaParams &p, unsigned long long target,
                                             MegaShared &sh) {
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t ok = 1;
        __threadfence();
        atomicAdd(p.arrivals, 1ull);
        const uint64_t t0 = globaltimer_ns(), limit = wait_limit_ns();
        while (ld_acquire_gpu_u64(p.arrivals) < target) {
            if (*(volatile uint32_t *)p.abort) { ok = 0; break; }
            if (globaltimer_ns() - t0 > limit) {
                atomicOr(p.status, WL_DEV_ERR_MEGA);
                atomicExch(p.abort, 1u);
                ok = 0;
                break;
            }
        }
        sh.s_flag = ok;
    }
    __syncthreads();
    return sh.s_flag != 0;
}

// ---------------------------------------------------------------------------
// A matvec phase's row space: up to three weights stacked (rows in order).
struct MegaSet {
    const uint8_t *w[3];
    float scale[3];
    uint32_t rows[3];
    int n;
    uint32_t row_bytes;
    __device__ uint32_t total() const { return rows[0] + (n > 1 ? rows[1] : 0u) + (n > 2 ? rows[2] : 0u); }
};

__device__ __forceinline__ void mega_range(uint32_t total, uint32_t &r0, uint32_t &r1) {
    const uint32_t per = (total + gridDim.x - 1) / gridDim.x;
    r0 = min(total, blockIdx.x * per);
    r1 = min(total, r0 + per);
}

// Thread 0: request rows [r0, r1) of the set into dst (one bulk copy per
// weight the range touches), completing on bar.
__device__ __forceinline__ void mega_issue(const MegaSet &s, uint32_t r0, uint32_t r1,
                                           uint8_t *dst, uint64_t *bar, uint64_t policy,
                                           const float *norm, float *norm_dst, uint32_t norm_n) {
    mbar_arrive_expect_tx(bar, (r1 - r0) * s.row_bytes + norm_n * 4u);
    bulk_g2s(norm_dst, norm, norm_n * 4u, bar);  // the phase's RMSNorm weights
    uint32_t base = 0, off = 0;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        if (j >= s.n) break;
        const uint32_t a = max(r0, base), b = min(r1, base + s.rows[j]);
        if (a < b) {
            const uint32_t bytes = (b - a) * s.row_bytes;
            bulk_g2s_evict_first(dst + off, s.w[j] + (size_t)(a - base) * s.row_bytes, bytes, bar,
                                 policy);
            off += bytes;
        }
        base += s.rows[j];
    }
}

// Norm (+ absmax int8) of the CTA's input already staged in xs[0..K):
// xs = (xs * rsqrt) * w, q = quantised xs.  Sum of squares as a tree, or, in
// exact mode, in the reference's sequential order (one thread).
__device__ __noinline__ float mega_norm_quantize(const MegaParams &p, float *xs, int8_t *qs,
                                                    const float *w, uint32_t K, MegaShared &sh) {
    const uint32_t tid = threadIdx.x;
    float sum_sq;
    __syncthreads();
    if (p.exact) {
        if (tid == 0) {
            sh.s_scale = seq_sum_sq(xs, K);
        }
        __syncthreads();
        sum_sq = sh.s_scale;
    } else {
        float ss = 0.0f;
        for (uint32_t i = tid; i < K; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(xs[i], xs[i]));
        sum_sq = block_sum(ss, sh.red);
    }
    const float mean = __fdiv_rn(sum_sq, (float)K);
    const float rsqrt = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
    float m = 0.0f;
    {
        const uint32_t n4 = K / 4u, T = blockDim.x;
        const float4 *w4 = reinterpret_cast<const float4 *>(w);
        float4 *x4 = reinterpret_cast<float4 *>(xs);
        for (uint32_t i0 = tid; i0 < n4; i0 += 8u * T) {
            float4 wv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (i0 + u * T < n4) wv[u] = w4[i0 + u * T];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (i0 + u * T < n4) {
                    float4 v = x4[i0 + u * T];
                    v.x = __fmul_rn(__fmul_rn(v.x, rsqrt), wv[u].x);
                    v.y = __fmul_rn(__fmul_rn(v.y, rsqrt), wv[u].y);
                    v.z = __fmul_rn(__fmul_rn(v.z, rsqrt), wv[u].z);
                    v.w = __fmul_rn(__fmul_rn(v.w, rsqrt), wv[u].w);
                    x4[i0 + u * T] = v;
                    m = fmaxf(fmaxf(m, fabsf(v.x)), fmaxf(fabsf(v.y), fmaxf(fabsf(v.z), fabsf(v.w))));
                }
        }
    }
    const float max_abs = block_max(m, sh.red);  // NaN never wins (bitlinear_sse2.rs:285-304)
    const float inv = max_abs == 0.0f ? 0.0f : __fdiv_rn(127.0f, max_abs);
    for (uint32_t i = tid; i < K; i += blockDim.x) {
        int qi = 0;
        if (max_abs != 0.0f) {
            qi = quant_round_i8(__fmul_rn(xs[i], inv));
        }
        qs[i] = (int8_t)qi;
    }
    __syncthreads();
    return max_abs == 0.0f ? 1.0f : __fdiv_rn(max_abs, 127.0f);
}

// The CTA's rows [r0, r1) of a set, staged in rows (smem), against the
// quantised input qs (smem).  MODE 0: out[r] = y; MODE 1: out[r] += y
// (residual; non-finite -> status bit).
template <bool C3, int MODE, int LPR, int NP>
__device__ __noinline__ void mega_matvec_t(const MegaParams &p, const MegaSet &s, uint32_t r0,
                                              uint32_t r1, const uint8_t *rows, const int8_t *qs,
                                              uint32_t K, float act_scale, float *out,
                                              float *hloc) {
    // LPR lanes per row; lane sl owns slots pp = sl + LPR*i, i < NP, whose
    // activations stay in registers for every row (one shared-memory read
    // per phase instead of one per row).
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t sl = lane % LPR, sub = lane / LPR;
    const uint32_t P = K >> 6;  // 16-byte slots per row
    uint4 act[NP][4];
    int32_t asum = 0;
#pragma unroll
    for (int i = 0; i < NP; ++i) {
        const uint32_t pp = sl + LPR * i;
        if (pp < P) {
            i2s_load_act<false>(qs, pp, 0u, act[i]);
#pragma unroll
            for (int o = 0; o < 4; ++o) asum += sum_bytes(act[i][o]);
        } else {
#pragma unroll
            for (int o = 0; o < 4; ++o) act[i][o] = make_uint4(0, 0, 0, 0);
        }
    }
    // row -> weight of the set, and its scale (no dynamically indexed arrays)
    const uint32_t b1 = s.rows[0], b2 = s.rows[0] + (s.n > 1 ? s.rows[1] : 0u);
    const float sc0 = __fmul_rn(s.scale[0], act_scale);
    const float sc1 = __fmul_rn(s.n > 1 ? s.scale[1] : 0.0f, act_scale);
    const float sc2 = __fmul_rn(s.n > 2 ? s.scale[2] : 0.0f, act_scale);
    constexpr uint32_t RPI = (MEGA_THREADS / 32) * (32 / LPR);
    const uint32_t R = r1 - r0, rb = s.row_bytes;
    for (uint32_t base = 0; base < R; base += RPI) {
        const uint32_t rl = base + warp * (32 / LPR) + sub;
        const uint8_t *rp = rows + (size_t)rl * rb;
        I2sAcc acc = {0, 0, 0, 0};
        uint32_t c3 = 0;
        if (rl < R) {
#pragma unroll
            for (int i = 0; i < NP; ++i) {
                const uint32_t pp = sl + LPR * i;
                if (pp < P) i2s_slot<C3>(*reinterpret_cast<const uint4 *>(rp + 16 * pp), act[i], acc, c3);
            }
        }
        int32_t dot = i2s_acc_total(acc) - asum;
#pragma unroll
        for (int off = LPR / 2; off > 0; off >>= 1) {
            dot += __shfl_xor_sync(0xffffffffu, dot, off);
            if constexpr (C3) c3 |= __shfl_xor_sync(0xffffffffu, c3, off);
        }
        if constexpr (C3) {
            if ((c3 & 0x55555555u) != 0u) {  // uniform across the row's lanes
                int32_t corr = rl < R ? i2s_row_c3<false>(rp, qs, 0u, sl, LPR, P) : 0;
                const uint32_t grp = __match_any_sync(__activemask(), rl);
#pragma unroll
                for (int off = LPR / 2; off > 0; off >>= 1) corr += __shfl_xor_sync(grp, corr, off);
                dot -= 2 * corr;
            }
        }
        if (sl == 0 && rl < R) {
            const uint32_t r = r0 + rl;
            const float combined = r < b1 ? sc0 : (r < b2 ? sc1 : sc2);
            const float yv = __fmul_rn(combined, __int2float_rn(dot));
            if constexpr (MODE == 0) {
                out[r] = yv;
            } else {  // residual: this CTA's rows of hidden live in hloc
                const float nv = __fadd_rn(hloc[rl], yv);
                hloc[rl] = nv;
                out[r] = nv;
                if (!isfinite(nv)) atomicOr(p.status, WL_DEV_ERR_NONFINITE);
            }
        }
    }
}

// Slot split by row length: 8 lanes x 5 slots up to K = 2560, 32 lanes x 4
// slots up to K = 8192 (the fused-input limit).  The combined scale is
// (w_scale * act_scale) * (f32)acc, the reference's two multiplies.
template <bool C3, int MODE>
__device__ __forceinline__ void mega_matvec(const MegaParams &p, const MegaSet &s, uint32_t r0,
                                            uint32_t r1, const uint8_t *rows, const int8_t *qs,
                                            uint32_t K, float act_scale, float *out, float *hloc) {
    if ((K >> 6) <= 40u) mega_matvec_t<C3, MODE, 8, 5>(p, s, r0, r1, rows, qs, K, act_scale, out, hloc);
    else mega_matvec_t<C3, MODE, 32, 4>(p, s, r0, r1, rows, qs, K, act_scale, out, hloc);
}

__device__ __forceinline__ MegaSet mega_set(const MegaParams &p, const MegaLayer &L, int phase) {
    MegaSet s;
    if (phase == 0) {  // q, k, v
        s.n = 3;
        s.w[0] = L.w[0]; s.w[1] = L.w[1]; s.w[2] = L.w[2];
        s.scale[0] = L.scale[0]; s.scale[1] = L.scale[1]; s.scale[2] = L.scale[2];
        s.rows[0] = p.E; s.rows[1] = p.KV; s.rows[2] = p.KV;
        s.row_bytes = p.E / 4u;
    } else if (phase == 1) {  // o
        s.n = 1;
        s.w[0] = L.w[3]; s.scale[0] = L.scale[3]; s.rows[0] = p.E;
        s.row_bytes = p.E / 4u;
    } else if (phase == 2) {  // gate, up
        s.n = 2;
        s.w[0] = L.w[4]; s.w[1] = L.w[5];
        s.scale[0] = L.scale[4]; s.scale[1] = L.scale[5];
        s.rows[0] = p.F; s.rows[1] = p.F;
        s.row_bytes = p.E / 4u;
    } else {  // down
        s.n = 1;
        s.w[0] = L.w[6]; s.scale[0] = L.scale[6]; s.rows[0] = p.E;
        s.row_bytes = p.F / 4u;
    }
    return s;
}

// Attention of one (head, split) item: the split-local part of
// attn_decode_kernel (same arithmetic); exact mode (one split) writes the
// head's output directly in the reference's order.
__device__ __noinline__ void mega_attention(const MegaParams &p, uint32_t layer, uint32_t item, uint8_t *smem,
                               MegaShared &sh) {
    const uint32_t HD = p.HD, KV = p.KV, half = p.n_rot / 2u, tid = threadIdx.x;
    const uint32_t h = item / p.splits, sp = item % p.splits, kvh = h / p.group;
    const uint32_t chunk_max = ((p.max_seq + p.splits - 1) / p.splits + 3u) & ~3u;
    float *ks = reinterpret_cast<float *>(smem);
    float *vs = ks + KV;
    float *qh = vs + KV;
    float *obuf = qh + HD;
    float *scores = obuf + MEGA_THREADS;
    float *vsc = scores + chunk_max;
    float2 *rope = reinterpret_cast<float2 *>(vsc + chunk_max);
    int8_t *kq = reinterpret_cast<int8_t *>(rope + ((half + 1u) & ~1u));
    int8_t *vq = kq + KV;
    int8_t *kc = p.kq + (size_t)layer * p.max_seq * KV;
    int8_t *vc = p.vq + (size_t)layer * p.max_seq * KV;
    float *ksc = p.ks + (size_t)layer * p.max_seq, *vsc_g = p.vs + (size_t)layer * p.max_seq;
    const uint32_t pos = *p.pos;
    const float *q = p.qkv, *k = p.qkv + p.E, *v = p.qkv + p.E + KV;
    stage_f32(ks, k, KV);
    stage_f32(vs, v, KV);
    stage_f32(qh, q + h * HD, HD);
    for (uint32_t j = tid; j < half; j += blockDim.x) rope[j] = p.rope[(size_t)pos * half + j];
    __syncthreads();
    for (uint32_t i = tid; i < (KV / HD) * half; i += blockDim.x) {
        const uint32_t hk = i / half, j = i % half;
        float *x = ks + hk * HD;
        const float a = x[j], b = x[j + half], c = rope[j].x, s = rope[j].y;
        x[j] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        x[j + half] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
    for (uint32_t j = tid; j < half; j += blockDim.x) {
        const float a = qh[j], b = qh[j + half], c = rope[j].x, s = rope[j].y;
        qh[j] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        qh[j + half] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
    __syncthreads();
    kv_quantise_block(ks, KV, kq, &sh.s_ks, sh.red);
    kv_quantise_block(vs, KV, vq, &sh.s_vs, sh.red);
    __syncthreads();
    const float s_ks = sh.s_ks, s_vs = sh.s_vs;
    if (item == 0) {
        for (uint32_t i = tid; i < KV; i += blockDim.x) {
            kc[(size_t)pos * KV + i] = kq[i];
            vc[(size_t)pos * KV + i] = vq[i];
        }
        if (tid == 0) {
            ksc[pos] = s_ks;
            vsc_g[pos] = s_vs;
        }
    }
    const uint32_t n = pos + 1u, chunk = (n + p.splits - 1u) / p.splits;
    const uint32_t t0 = min(n, sp * chunk), t1 = min(n, t0 + chunk), cnt = t1 - t0;
    for (uint32_t i = tid; i < cnt; i += blockDim.x) {
        const uint32_t t = t0 + i;
        const int8_t *kr = t == pos ? kq + kvh * HD : kc + (size_t)t * KV + kvh * HD;
        const float sk = t == pos ? s_ks : ksc[t];
        vsc[i] = t == pos ? s_vs : vsc_g[t];
        float d = 0.0f;
        for (uint32_t c0 = 0; c0 < HD; c0 += 128u) {  // 128 dims per round of loads
            uint4 w[8];
#pragma unroll
            for (int c = 0; c < 8; ++c)
                if (c0 + (uint32_t)c * 16u < HD) w[c] = *reinterpret_cast<const uint4 *>(kr + c0 + c * 16);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                if (c0 + (uint32_t)c * 16u >= HD) break;
                const uint32_t wv[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const float kv8 = (float)(int8_t)(wv[e >> 2] >> (8 * (e & 3)));
                    d = __fadd_rn(d, __fmul_rn(qh[c0 + c * 16 + e], __fmul_rn(kv8, sk)));
                }
            }
        }
        scores[i] = __fmul_rn(d, p.scale);
    }
    __syncthreads();
    if (p.exact) {  // one split: the reference's sequential softmax and weighted sum
        if (tid == 0) {
            float mxs = -INFINITY;
            for (uint32_t i = 0; i < cnt; ++i)
                if (scores[i] > mxs) mxs = scores[i];
            sh.s_scale = mxs;
        }
        __syncthreads();
        const float mxs = sh.s_scale;
        if (!isfinite(mxs)) {
            for (uint32_t i = tid; i < cnt; i += blockDim.x) scores[i] = 0.0f;
        } else {
            for (uint32_t i = tid; i < cnt; i += blockDim.x)
                scores[i] = exp_f32(__fsub_rn(scores[i], mxs));
            __syncthreads();
            if (tid == 0) {
                float sum = 0.0f;
                for (uint32_t i = 0; i < cnt; ++i) sum = __fadd_rn(sum, scores[i]);
                sh.s_flag = sum > 0.0f ? 1u : 0u;
                sh.s_scale = sh.s_flag ? __fdiv_rn(1.0f, sum) : 1.0f;
            }
            __syncthreads();
            if (sh.s_flag)
                for (uint32_t i = tid; i < cnt; i += blockDim.x) scores[i] = __fmul_rn(scores[i], sh.s_scale);
        }
        __syncthreads();
        if (tid < HD) {
            float o = 0.0f;
            for (uint32_t i = 0; i < cnt; ++i) {
                const uint32_t t = t0 + i;
                const int8_t vv = t == pos ? vq[kvh * HD + tid] : vc[(size_t)t * KV + kvh * HD + tid];
                o = __fadd_rn(o, __fmul_rn(scores[i], __fmul_rn((float)vv, vsc[i])));
            }
            p.att[h * HD + tid] = o;
        }
        return;
    }
    float m = -INFINITY;
    for (uint32_t i = tid; i < cnt; i += blockDim.x) m = fmaxf(m, scores[i]);
    const float mx = block_max(m, sh.red);
    float lsum = 0.0f;
    const bool finite = isfinite(mx);
    if (finite) {
        for (uint32_t i = tid; i < cnt; i += blockDim.x) {
            const float e = exp_f32(__fsub_rn(scores[i], mx));
            scores[i] = e;
            lsum = __fadd_rn(lsum, e);
        }
    }
    const float l = block_sum(lsum, sh.red);
    __syncthreads();
    const uint32_t groups = blockDim.x / HD, d = tid % HD, g = tid / HD;
    float acc = 0.0f;
    if (finite && g < groups) {
        const int8_t *vbase = vc + (size_t)kvh * HD + d;
        for (uint32_t i0 = g; i0 < cnt; i0 += 8u * groups) {
            int8_t vv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint32_t i = i0 + (uint32_t)u * groups;
                const uint32_t t = t0 + i;
                vv[u] = i >= cnt ? (int8_t)0 : (t == pos ? vq[kvh * HD + d] : vbase[(size_t)t * KV]);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint32_t i = i0 + (uint32_t)u * groups;
                if (i < cnt) acc = __fadd_rn(acc, __fmul_rn(scores[i], __fmul_rn((float)vv[u], vsc[i])));
            }
        }
    }
    obuf[tid] = acc;
    __syncthreads();
    float *part = p.partial + ((size_t)h * p.splits + sp) * (HD + 4u);
    if (tid < HD) {
        float o = obuf[tid];
        for (uint32_t gg = 1; gg < groups; ++gg) o = __fadd_rn(o, obuf[gg * HD + tid]);
        part[tid] = o;
    }
    if (tid == 0) {
        part[HD] = mx;
        part[HD + 1] = l;
    }
}

// Every CTA: the attention output of all heads into att (E floats), from the
// splits' partials (fast mode) or from the exact-mode output in global.
// Partial rows: o[HD], then max, sum (stride HD + 4 floats, 16-byte aligned).
// One warp per head: lanes reduce the splits' maxima and sums, keep the split
// factors exp(m - M) in shared memory (cmb, S floats per warp), then combine
// the o rows with float4 loads, eight splits per round of loads.
__device__ __noinline__ void mega_combine(const MegaParams &p, float *att, float *cmb) {
    const uint32_t HD = p.HD, tid = threadIdx.x, S = p.splits, RS = HD + 4u;
    if (p.exact) {
        for (uint32_t i = tid; i < p.E; i += blockDim.x) att[i] = __ldcg(p.att + i);
        return;
    }
    const uint32_t lane = tid & 31u, warp = tid >> 5, nw = blockDim.x >> 5;
    float *fs = cmb + warp * S;
    for (uint32_t h = warp; h < p.n_heads; h += nw) {
        const float *hb = p.partial + (size_t)h * S * RS;
        float M = -INFINITY;
        for (uint32_t s2 = lane; s2 < S; s2 += 32u) M = fmaxf(M, __ldcg(hb + s2 * RS + HD));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        const bool fin = isfinite(M);
        float L = 0.0f;
        for (uint32_t s2 = lane; s2 < S; s2 += 32u) {
            const float ms = __ldcg(hb + s2 * RS + HD), ls = __ldcg(hb + s2 * RS + HD + 1);
            const float f = (fin && ms > -INFINITY) ? exp_f32(__fsub_rn(ms, M)) : 0.0f;
            fs[s2] = f;
            L = __fadd_rn(L, __fmul_rn(ls, f));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) L = __fadd_rn(L, __shfl_xor_sync(0xffffffffu, L, off));
        __syncwarp();
        const float inv = L > 0.0f ? __fdiv_rn(1.0f, L) : 1.0f;
        for (uint32_t c = lane; c < HD / 4u; c += 32u) {
            float4 O = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (uint32_t s0 = 0; s0 < S; s0 += 8u) {
                float4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (s0 + u < S)
                        v[u] = __ldcg(reinterpret_cast<const float4 *>(hb + (s0 + u) * RS) + c);
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (s0 + u < S) {
                        const float f = fs[s0 + u];
                        O.x = __fadd_rn(O.x, __fmul_rn(v[u].x, f));
                        O.y = __fadd_rn(O.y, __fmul_rn(v[u].y, f));
                        O.z = __fadd_rn(O.z, __fmul_rn(v[u].z, f));
                        O.w = __fadd_rn(O.w, __fmul_rn(v[u].w, f));
                    }
            }
            if (!fin) {
                O = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            } else if (L > 0.0f) {
                O.x = __fmul_rn(O.x, inv);
                O.y = __fmul_rn(O.y, inv);
                O.z = __fmul_rn(O.z, inv);
                O.w = __fmul_rn(O.w, inv);
            }
            reinterpret_cast<float4 *>(att + h * HD)[c] = O;
        }
        __syncwarp();
    }
}

inline size_t mega_cmb_floats(uint32_t n_heads, uint32_t splits) {
    (void)n_heads;
    return (size_t)(MEGA_THREADS / 32) * splits;  // split factors, one row per warp
}

// Bounded wait for a weight buffer; on timeout the grid aborts.
__device__ __forceinline__ bool mega_wait_rows(const MegaParams &p, uint64_t *bar, uint32_t &phase,
                                               MegaShared &sh) {
    const bool ok = mbar_wait(bar, phase);
    phase ^= 1u;
    if (!__syncthreads_and(ok)) {
        if (threadIdx.x == 0) {
            atomicOr(p.status, WL_DEV_ERR_MEGA);
            atomicExch(p.abort, 1u);
        }
        return false;
    }
    return true;
}

template <bool C3>
__global__ void __launch_bounds__(MEGA_THREADS, 1)
    bitnet_mega_kernel(const __grid_constant__ MegaParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ MegaShared sh;
    const uint32_t tid = threadIdx.x, G = gridDim.x;
    uint8_t *bufA = smem + p.buf_a, *bufB = smem + p.buf_b;
    float *normA = reinterpret_cast<float *>(smem + p.norm_a);
    float *normB = reinterpret_cast<float *>(smem + p.norm_b);
    float *hloc = reinterpret_cast<float *>(smem + p.hloc_off);  // this CTA's hidden rows
    float *xs = reinterpret_cast<float *>(smem + p.xs_off);
    int8_t *qs = reinterpret_cast<int8_t *>(smem + p.qs_off);
    uint8_t *att_smem = smem + p.att_off;
    float *cmb = reinterpret_cast<float *>(smem + p.cmb_off);
    const uint64_t policy = l2_policy_evict_first();
    const unsigned long long per_launch = 5ull * p.n_layers;
    const unsigned long long base = (unsigned long long)(*(volatile uint32_t *)p.launches) * per_launch;
    uint32_t nb = 0;  // barriers passed in this launch
    uint32_t phA = 0, phB = 0;
    bool pendA = false, pendB = false;
    if (tid == 0) {
        mbar_init(&sh.bar[0], 1);
        mbar_init(&sh.bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto barrier = [&]() -> bool {
        ++nb;
        return mega_barrier(p, (base + nb) * G, sh);
    };
    auto issue = [&](int which, uint32_t layer, int phase) {
        if (layer >= p.n_layers) return;
        const MegaLayer &L = p.layers[layer];
        const MegaSet s = mega_set(p, L, phase);
        uint32_t r0, r1;
        mega_range(s.total(), r0, r1);
        if (which == 0) pendA = true; else pendB = true;
        // norm weights of the phase: P1 attn_norm, P3 attn_sub_norm, P4 ffn_norm,
        // P5 ffn_sub_norm
        const uint32_t noff = phase == 0 ? 0u : (phase == 1 ? p.E : (phase == 2 ? 2u * p.E : 3u * p.E));
        const uint32_t nn = phase == 3 ? p.F : p.E;
        if (tid == 0)
            mega_issue(s, r0, r1, which == 0 ? bufA : bufB, &sh.bar[which], policy, L.norm + noff,
                       which == 0 ? normA : normB, nn);
    };
    bool ok = true;
    issue(0, 0, 0);  // QKV(0) -> A
    issue(1, 0, 1);  // O(0)   -> B
    const uint32_t tok = *p.token;
    if (p.ids && blockIdx.x == 0 && tid == 0) {
        p.ids[*p.step] = tok;
        *p.step += 1u;
    }
    // the token's embedding: every CTA keeps it whole (P1 of layer 0), and
    // each writes its slice of the residual stream
    {
        const uint32_t E = p.E;
        const uint8_t *row = p.q6k + (size_t)tok * p.q6k_stride;
        for (uint32_t i = tid; i < E; i += blockDim.x) {
            const uint32_t b = i >> 8, t = i & 255u;
            const uint8_t *ql = row + b * 128u, *qh = row + p.nb * 128u + b * 64u;
            const int8_t *sc = reinterpret_cast<const int8_t *>(row + p.nb * 192u + b * 16u);
            const uint16_t dbits = *reinterpret_cast<const uint16_t *>(row + p.nb * 208u + b * 2u);
            const uint32_t hh = t >> 7, a = (t >> 5) & 3u, l = t & 31u;
            const uint8_t lb = ql[hh * 64u + l + ((a & 1u) ? 32u : 0u)];
            const uint32_t lo = (a & 2u) ? (lb >> 4) : (lb & 0x0Fu);
            const uint32_t hi = (qh[hh * 32u + l] >> (2u * a)) & 3u;
            const int q = (int)(lo | (hi << 4)) - 32;
            const float w = __fmul_rn(__fmul_rn(f16_bits_to_f32(dbits),
                                                (float)sc[hh * 8u + (l >> 4) + 2u * a]), (float)q);
            xs[i] = w;
            const uint32_t per = (E + G - 1) / G;
            if (i >= blockIdx.x * per && i < (blockIdx.x + 1) * per) {
                p.hidden[i] = w;
                hloc[i - blockIdx.x * per] = w;
            }
        }
    }
    for (uint32_t l = 0; l < p.n_layers && ok; ++l) {
        const MegaLayer &L = p.layers[l];
        // P1: attn_norm + Q/K/V
        if (l > 0) stage_f32(xs, p.hidden, p.E);
        float sc;
        {
            if (!(ok = mega_wait_rows(p, &sh.bar[0], phA, sh))) break;  // rows + attn_norm
            pendA = false;
            sc = mega_norm_quantize(p, xs, qs, normA, p.E, sh);
        }
        {
            const MegaSet s = mega_set(p, L, 0);
            uint32_t r0, r1;
            mega_range(s.total(), r0, r1);
            mega_matvec<C3, 0>(p, s, r0, r1, bufA, qs, p.E, sc, p.qkv, hloc);
        }
        __syncthreads();
        issue(0, l, 2);  // gate/up(l) -> A
        if (!(ok = barrier())) break;
        // P2: attention items
        const uint32_t items = p.n_heads * p.splits;
        for (uint32_t it = blockIdx.x; it < items; it += G) {
            mega_attention(p, l, it, att_smem, sh);
            __syncthreads();
        }
        if (!(ok = barrier())) break;
        // P3: combine, attn_sub_norm, O, residual
        mega_combine(p, xs, cmb);
        if (!(ok = mega_wait_rows(p, &sh.bar[1], phB, sh))) break;  // rows + attn_sub_norm
        pendB = false;
        sc = mega_norm_quantize(p, xs, qs, normB, p.E, sh);
        {
            const MegaSet s = mega_set(p, L, 1);
            uint32_t r0, r1;
            mega_range(s.total(), r0, r1);
            mega_matvec<C3, 1>(p, s, r0, r1, bufB, qs, p.E, sc, p.hidden, hloc);
        }
        __syncthreads();
        issue(1, l, 3);  // down(l) -> B
        if (!(ok = barrier())) break;
        // P4: ffn_norm, gate / up
        stage_f32(xs, p.hidden, p.E);
        if (!(ok = mega_wait_rows(p, &sh.bar[0], phA, sh))) break;  // rows + ffn_norm
        pendA = false;
        sc = mega_norm_quantize(p, xs, qs, normA, p.E, sh);
        {
            const MegaSet s = mega_set(p, L, 2);
            uint32_t r0, r1;
            mega_range(s.total(), r0, r1);
            mega_matvec<C3, 0>(p, s, r0, r1, bufA, qs, p.E, sc, p.gu, hloc);
        }
        __syncthreads();
        issue(0, l + 1, 0);  // QKV(l+1) -> A
        if (!(ok = barrier())) break;
        // P5: relu^2 * up, ffn_sub_norm, down, residual
        stage_relu2_mul(xs, p.gu, p.gu + p.F, p.F);
        if (!(ok = mega_wait_rows(p, &sh.bar[1], phB, sh))) break;  // rows + ffn_sub_norm
        pendB = false;
        sc = mega_norm_quantize(p, xs, qs, normB, p.F, sh);
        {
            const MegaSet s = mega_set(p, L, 3);
            uint32_t r0, r1;
            mega_range(s.total(), r0, r1);
            mega_matvec<C3, 1>(p, s, r0, r1, bufB, qs, p.F, sc, p.hidden, hloc);
        }
        __syncthreads();
        issue(1, l + 1, 1);  // O(l+1) -> B
        if (!(ok = barrier())) break;
    }
    if (!ok) {
        // drain the weight copies still in flight (bounded) before exiting
        if (pendA) (void)mbar_wait(&sh.bar[0], phA);
        if (pendB) (void)mbar_wait(&sh.bar[1], phB);
        __syncthreads();
        return;
    }
    if (blockIdx.x == 0) {
        // output_norm (cached_forward.rs:252-254), then the position advances
        stage_f32(xs, p.hidden, p.E);
        __syncthreads();
        float sum_sq;
        if (p.exact) {
            if (tid == 0) {
                sh.s_scale = seq_sum_sq(xs, p.E);
            }
            __syncthreads();
            sum_sq = sh.s_scale;
        } else {
            float ss = 0.0f;
            for (uint32_t i = tid; i < p.E; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(xs[i], xs[i]));
            sum_sq = block_sum(ss, sh.red);
        }
        const float mean = __fdiv_rn(sum_sq, (float)p.E);
        const float rsqrt = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
        for (uint32_t i = tid; i < p.E; i += blockDim.x)
            p.final_h[i] = __fmul_rn(__fmul_rn(xs[i], rsqrt), p.out_norm[i]);
        __syncthreads();
        if (tid == 0) {
            *p.pos += 1u;
            *p.launches += 1u;  // every CTA has passed every barrier of this launch
        }
    }
}

}  // namespace wl
