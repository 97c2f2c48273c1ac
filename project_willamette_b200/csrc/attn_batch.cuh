// attn_batch.cuh -- decode attention for many independent sequences, one
// CTA per (KV head, sequence, split) serving the KV head's whole group of
// query heads (GQA), so every cached K / V row is read once per step.
//
// Reference: scaled_dot_product_attention_into (src/model/cached_forward.rs:
// 421-451), softmax_inplace (src/model/attention.rs:45-73), KVCache append /
// read_into (src/model/kv_cache.rs:154-259), apply_rope_f32
// (src/model/primitives.rs:283-345).
//
// Per CTA:
//  1. k, v (all KV heads, needed for the per-token absmax of the cache's i8
//     quantisation), the group's q heads and the RoPE row, one round of loads;
//     RoPE on k and the q heads; absmax of k and of v in one block reduction.
//  2. This CTA's K / V head slice of the current position quantised; split 0
//     appends it to the cache (head 0 also the two scales).  Earlier
//     positions come from the cache, the current one from shared memory, so
//     no CTA waits on another's append.
//  3. Scores, one thread per position: the position's K head row (HD bytes)
//     is loaded in one round and dotted with every q head of the group.
//  4. Softmax statistics per q head (max, sum of exp) in block reductions.
//  5. V: a thread owns 16 dimensions of one position per round (one 16-byte
//     load) and accumulates them for every q head; positions are reduced
//     over lanes, then warps.
//  6. splits > 1: unnormalised partials (o, max, sum) per split, the last
//     CTA of the (sequence, KV head) combines them.
// Sums run as trees and products are fused (the engine's fast mode); the
// exact mode keeps attn_decode_kernel.  A non-finite score maximum gives a
// zero output, as in the reference.
#pragma once

#include <cstdint>

#include "bitnet_decode.cuh"  // AttnParams, WL_DEV_ERR_*

namespace wl {

constexpr int AB_THREADS = 256;
constexpr uint32_t AB_MAX_GROUP = 4;  // q heads per KV head
constexpr uint32_t AB_WARPS = AB_THREADS / 32;

// dynamic shared memory of attn_gqa_batch_kernel
inline size_t attn_gqa_smem_bytes(uint32_t kv, uint32_t hd, uint32_t group, uint32_t max_seq,
                                  uint32_t splits) {
    const uint32_t chunk = ((max_seq + splits - 1) / splits + 3u) & ~3u;
    const uint32_t half2 = ((hd / 2u + 1u) & ~1u) * 2u;
    size_t f = 2u * kv                          // k, v (rotated k)
               + group * hd                     // q heads
               + half2                          // RoPE row
               + (size_t)group * chunk          // scores / weights
               + chunk                          // V scales
               + (size_t)AB_WARPS * group * hd  // per-warp V partial sums
               + 4u * group + 64u;              // combine factors
    return f * 4u + 2u * hd + 16u;              // + the current position's i8 K / V slice
}

__global__ void __launch_bounds__(AB_THREADS, 2) attn_gqa_batch_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[AB_WARPS * 2 * AB_MAX_GROUP];
    __shared__ float s_sc[2];
    __shared__ uint32_t s_last;
    const uint32_t HD = p.head_dim, KV = p.n_kv_heads * HD, half = p.n_rot / 2u, G = p.group;
    const uint32_t kvh = blockIdx.x, z = blockIdx.y, sp = blockIdx.z, S = gridDim.z;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t chunk_max = ((p.max_seq + S - 1) / S + 3u) & ~3u;
    float *ks = reinterpret_cast<float *>(smem);      // KV
    float *vs = ks + KV;                              // KV
    float *qg = vs + KV;                              // G * HD
    float2 *rope = reinterpret_cast<float2 *>(qg + G * HD);  // half (rounded to 2)
    float *scores = reinterpret_cast<float *>(rope + ((half + 1u) & ~1u));  // G * chunk_max
    float *vsc = scores + (size_t)G * chunk_max;      // chunk_max
    float *vpart = vsc + chunk_max;                   // AB_WARPS * G * HD
    float *stat = vpart + (size_t)AB_WARPS * G * HD;  // 4 * G + 64
    int8_t *kq = reinterpret_cast<int8_t *>(stat + 4u * G + 64u);  // HD
    int8_t *vq = kq + HD;                                          // HD

    pdl_launch_dependents();
    pdl_wait();
    if (p.active && !p.active[z]) return;
    const uint32_t pos = p.pos[z];
    if (pos >= p.max_seq) {
        if (tid == 0) atomicOr(p.status, WL_DEV_ERR_POSITION);
        return;
    }
    const float *q_in = p.q + (size_t)z * p.qkv_stride, *k_in = p.k + (size_t)z * p.qkv_stride,
                *v_in = p.v + (size_t)z * p.qkv_stride;
    int8_t *k_cache = p.k_cache + z * p.cache_stride, *v_cache = p.v_cache + z * p.cache_stride;
    float *k_scale = p.k_scale + (size_t)z * p.scale_stride,
          *v_scale = p.v_scale + (size_t)z * p.scale_stride;
    const float2 *cs = p.rope + (size_t)pos * half;
    for (uint32_t i = tid; i < KV; i += AB_THREADS) {
        ks[i] = k_in[i];
        vs[i] = v_in[i];
    }
    for (uint32_t i = tid; i < G * HD; i += AB_THREADS) qg[i] = q_in[kvh * G * HD + i];
    for (uint32_t j = tid; j < half; j += AB_THREADS) rope[j] = cs[j];
    __syncthreads();
    const uint32_t pstep = p.rope_pairs ? 2u : 1u, poff = p.rope_pairs ? 1u : half;
    for (uint32_t i = tid; i < (p.n_kv_heads + G) * half; i += AB_THREADS) {
        const uint32_t hh = i / half, j = i % half;
        float *x = hh < p.n_kv_heads ? ks + hh * HD : qg + (hh - p.n_kv_heads) * HD;
        const uint32_t i0 = j * pstep, i1 = i0 + poff;
        const float a = x[i0], b = x[i1], c = rope[j].x, s = rope[j].y;
        x[i0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        x[i1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
    __syncthreads();
    // per-token absmax quantisation of k and v (kv_cache.rs:245-259)
    {
        float mk = 0.0f, mv = 0.0f;
        for (uint32_t i = tid; i < KV; i += AB_THREADS) {
            mk = fmaxf(mk, fabsf(ks[i]));
            mv = fmaxf(mv, fabsf(vs[i]));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, off));
            mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, off));
        }
        if (lane == 0) {
            red[warp * 2] = mk;
            red[warp * 2 + 1] = mv;
        }
        __syncthreads();
        if (tid < 2) {
            float m = red[tid];
            for (uint32_t w = 1; w < AB_WARPS; ++w) m = fmaxf(m, red[w * 2 + tid]);
            s_sc[tid] = m;
        }
        __syncthreads();
        const float ak = s_sc[0], av = s_sc[1];
        const bool zk = ak == 0.0f || !isfinite(ak), zv = av == 0.0f || !isfinite(av);
        const float ik = zk ? 0.0f : __fdiv_rn(127.0f, ak), iv = zv ? 0.0f : __fdiv_rn(127.0f, av);
        for (uint32_t i = tid; i < 2u * HD; i += AB_THREADS) {
            const bool isv = i >= HD;
            const uint32_t d = isv ? i - HD : i;
            const float x = isv ? vs[kvh * HD + d] : ks[kvh * HD + d];
            int qi = 0;
            if (!(isv ? zv : zk)) {
                const float r = roundf(__fmul_rn(x, isv ? iv : ik));
                qi = isnan(r) ? 0 : (int)fminf(fmaxf(r, -127.0f), 127.0f);
            }
            (isv ? vq : kq)[d] = (int8_t)qi;
            if (sp == 0) (isv ? v_cache : k_cache)[(size_t)pos * KV + kvh * HD + d] = (int8_t)qi;
        }
        __syncthreads();  // red / s_sc reused below; kq / vq complete
        if (tid == 0) {
            s_sc[0] = zk ? 0.0f : __fdiv_rn(ak, 127.0f);
            s_sc[1] = zv ? 0.0f : __fdiv_rn(av, 127.0f);
            if (sp == 0 && kvh == 0) {
                k_scale[pos] = s_sc[0];
                v_scale[pos] = s_sc[1];
            }
        }
        __syncthreads();
    }
    const float sk_cur = s_sc[0], sv_cur = s_sc[1];
    // this split's positions [t0, t1)
    const uint32_t n = pos + 1u, chunk = (n + S - 1u) / S;
    const uint32_t t0 = min(n, sp * chunk), t1 = min(n, t0 + chunk), cnt = t1 - t0;
    // 3. scores (G heads) per position
    for (uint32_t i = tid; i < cnt; i += AB_THREADS) {
        const uint32_t t = t0 + i;
        const int8_t *kr = t == pos ? kq : k_cache + (size_t)t * KV + kvh * HD;
        const float sk = t == pos ? sk_cur : k_scale[t];
        vsc[i] = t == pos ? sv_cur : v_scale[t];
        float d[AB_MAX_GROUP];
#pragma unroll
        for (uint32_t g = 0; g < AB_MAX_GROUP; ++g) d[g] = 0.0f;
        uint4 w[16];  // the whole head row in one round of loads (HD <= 256)
#pragma unroll
        for (uint32_t c = 0; c < 16u; ++c)
            if (c * 16u < HD) w[c] = *reinterpret_cast<const uint4 *>(kr + c * 16u);
#pragma unroll
        for (uint32_t c = 0; c < 16u; ++c) {
            if (c * 16u >= HD) break;
            const uint32_t wv[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const float k8 = __fmul_rn((float)(int8_t)(wv[e >> 2] >> (8 * (e & 3))), sk);
#pragma unroll
                for (uint32_t g = 0; g < AB_MAX_GROUP; ++g)
                    if (g < G) d[g] = __fmaf_rn(qg[g * HD + c * 16u + e], k8, d[g]);
            }
        }
#pragma unroll
        for (uint32_t g = 0; g < AB_MAX_GROUP; ++g)
            if (g < G) scores[g * chunk_max + i] = __fmul_rn(d[g], p.scale);
    }
    __syncthreads();
    // 4. per-head max and sum of exp
    float mx[AB_MAX_GROUP], sum[AB_MAX_GROUP];
    {
        float m[AB_MAX_GROUP];
#pragma unroll
        for (uint32_t g = 0; g < AB_MAX_GROUP; ++g) m[g] = -INFINITY;
        for (uint32_t i = tid; i < cnt; i += AB_THREADS)
#pragma unroll
            for (uint32_t g = 0; g < AB_MAX_GROUP; ++g)
                if (g < G) m[g] = fmaxf(m[g], scores[g * chunk_max + i]);
#pragma unroll
        for (uint32_t g = 0; g < AB_MAX_GROUP; ++g) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) m[g] = fmaxf(m[g], __shfl_xor_sync(0xffffffffu, m[g], off));
            if (lane == 0) red[warp * AB_MAX_GROUP + g] = m[g];
        }
        __syncthreads();
#pragma unroll
        for (uint32_t g = 0; g < AB_MAX_GROUP; ++g) {
            float t = red[g];
            for (uint32_t w = 1; w < AB_WARPS; ++w) t = fmaxf(t, red[w * AB_MAX_GROUP + g]);
            mx[g] = t;
        }
        __syncthreads();
        float l[AB_MAX_GROUP];
#pragma unroll
        for (uint32_t g = 0; g < AB_MAX_GROUP; ++g) l[g] = 0.0f;
        for (uint32_t i = tid; i < cnt; i += AB_THREADS)
#pragma unroll
            for (uint32_t g = 0; g < AB_MAX_GROUP; ++g)
                if (g < G) {
                    const float e = isfinite(mx[g]) ? expf(scores[g * chunk_max + i] - mx[g]) : 0.0f;
                    scores[g * chunk_max + i] = __fmul_rn(e, vsc[i]);  // the V scale folded in
                    l[g] += e;
                }
#pragma unroll
        for (uint32_t g = 0; g < AB_MAX_GROUP; ++g) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) l[g] += __shfl_xor_sync(0xffffffffu, l[g], off);
            if (lane == 0) red[warp * AB_MAX_GROUP + g] = l[g];
        }
        __syncthreads();
#pragma unroll
        for (uint32_t g = 0; g < AB_MAX_GROUP; ++g) {
            float t = red[g];
            for (uint32_t w = 1; w < AB_WARPS; ++w) t += red[w * AB_MAX_GROUP + g];
            sum[g] = t;
        }
    }
    // 5. o[g][d] = sum_i w_i * v8[i][d]: thread = (position lane, 16-dim quad)
    const uint32_t DQ = HD / 16u, PL = AB_THREADS / DQ;  // quads per row, positions per round
    const uint32_t dq = tid % DQ, pl = tid / DQ;
    float acc[AB_MAX_GROUP][16];
#pragma unroll
    for (uint32_t g = 0; g < AB_MAX_GROUP; ++g)
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[g][e] = 0.0f;
    for (uint32_t i0 = pl; i0 < cnt; i0 += 4u * PL) {
        uint4 w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint32_t i = i0 + (uint32_t)u * PL, t = t0 + i;
            w[u] = make_uint4(0u, 0u, 0u, 0u);
            if (i < cnt)
                w[u] = *reinterpret_cast<const uint4 *>(t == pos ? vq + dq * 16u
                                                                 : v_cache + (size_t)t * KV + kvh * HD + dq * 16u);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint32_t i = i0 + (uint32_t)u * PL;
            if (i >= cnt) break;
            const uint32_t wv[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
            for (uint32_t g = 0; g < AB_MAX_GROUP; ++g) {
                if (g >= G) break;
                const float wt = scores[g * chunk_max + i];
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    acc[g][e] = __fmaf_rn(wt, (float)(int8_t)(wv[e >> 2] >> (8 * (e & 3))), acc[g][e]);
            }
        }
    }
    // reduce over the position lanes of a warp (lanes with the same quad)
#pragma unroll
    for (uint32_t g = 0; g < AB_MAX_GROUP; ++g) {
        if (g >= G) break;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            float v = acc[g][e];
            for (uint32_t off = DQ; off < 32u; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            acc[g][e] = v;
        }
    }
    if (lane < DQ) {
#pragma unroll
        for (uint32_t g = 0; g < AB_MAX_GROUP; ++g) {
            if (g >= G) break;
#pragma unroll
            for (int e = 0; e < 16; ++e) vpart[((size_t)warp * G + g) * HD + dq * 16u + e] = acc[g][e];
        }
    }
    __syncthreads();
    const uint32_t RS = HD + 4u;  // partial row: o[HD], max, sum
    float *part = p.partial + (((size_t)z * gridDim.x + kvh) * S + sp) * G * RS;
    for (uint32_t i = tid; i < G * HD; i += AB_THREADS) {
        const uint32_t g = i / HD, d = i % HD;
        float o = 0.0f;
        for (uint32_t w = 0; w < AB_WARPS; ++w) o += vpart[((size_t)w * G + g) * HD + d];
        if (S == 1) {
            const float L = sum[g];
            o = !isfinite(mx[g]) ? 0.0f : (L > 0.0f ? __fdiv_rn(o, L) : o);
            p.att[(size_t)z * p.att_stride + (kvh * G + g) * HD + d] = o;
        } else {
            part[g * RS + d] = o;
        }
    }
    if (S == 1) return;
    if (tid < G) {
        part[tid * RS + HD] = mx[tid];
        part[tid * RS + HD + 1] = sum[tid];
    }
    __threadfence();
    __syncthreads();
    uint32_t *ctr = p.counters + (size_t)z * gridDim.x + kvh;
    if (tid == 0) s_last = atomicAdd(ctr, 1u) == S - 1u ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // combine: M = max m_s, f_s = exp(m_s - M), O = sum f_s o_s / sum f_s l_s
    const float *base = p.partial + ((size_t)z * gridDim.x + kvh) * S * G * RS;
    float *fac = stat;  // [S][G] combine factors (S * G <= 64 + 4G)
    if (tid < G) {
        const uint32_t g = tid;
        float M = -INFINITY;
        for (uint32_t s2 = 0; s2 < S; ++s2) M = fmaxf(M, __ldcg(base + ((size_t)s2 * G + g) * RS + HD));
        float L = 0.0f;
        for (uint32_t s2 = 0; s2 < S; ++s2) {
            const float ms = __ldcg(base + ((size_t)s2 * G + g) * RS + HD);
            const float f = (isfinite(M) && ms > -INFINITY) ? expf(ms - M) : 0.0f;
            fac[s2 * G + g] = f;
            L += __ldcg(base + ((size_t)s2 * G + g) * RS + HD + 1) * f;
        }
        red[g] = !isfinite(M) ? 0.0f : (L > 0.0f ? __fdiv_rn(1.0f, L) : 1.0f);
    }
    __syncthreads();
    for (uint32_t i = tid; i < G * HD; i += AB_THREADS) {
        const uint32_t g = i / HD, d = i % HD;
        float o = 0.0f;
        for (uint32_t s2 = 0; s2 < S; ++s2)
            o = __fmaf_rn(__ldcg(base + ((size_t)s2 * G + g) * RS + d), fac[s2 * G + g], o);
        p.att[(size_t)z * p.att_stride + (kvh * G + g) * HD + d] = __fmul_rn(o, red[g]);
    }
    if (tid == 0) *ctr = 0u;  // re-arm for the next launch
}

}  // namespace wl
