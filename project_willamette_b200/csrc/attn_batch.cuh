// attn_batch.cuh -- decode attention for many independent sequences, one
// CTA per (KV head, sequence, split of `chunk` positions) serving the KV
// head's whole group of query heads (GQA), so every cached K / V row is read
// once per step.
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
//  3. The split's cached K / V head rows and scales are requested (cp.async,
//     one round) right after the dependency wait and land in shared memory
//     while step 1 runs.  Scores: one thread per (position, q head) when the
//     split's positions x heads fit one pass of the CTA, else one thread per
//     position for all G heads (q read as float4 broadcasts); each dot runs
//     over the head dimensions in order either way.
//  4. Softmax statistics per q head (max, sum of exp) in block reductions.
//  5. V: each warp takes every 8th position, a lane owns HD/32 dimensions of
//     the row (one coalesced row load per warp and position) and accumulates
//     them for every q head; the 8 warps' sums meet in shared memory.
//  6. splits > 1: unnormalised partials (o, max, sum) per split, the last
//     CTA of the (sequence, KV head) combines them.
// Sums run as trees and products are fused (the engine's fast mode); the
// exact mode keeps attn_decode_kernel.  A non-finite score maximum gives a
// zero output, as in the reference.  Templated on head_dim and group so
// every loop has a static trip count.
#pragma once

#include <cstdint>

#include "bitnet_decode.cuh"  // AttnParams, WL_DEV_ERR_*

namespace wl {

constexpr int AB_THREADS = 256;
constexpr uint32_t AB_MAX_GROUP = 4;  // q heads per KV head
constexpr uint32_t AB_WARPS = AB_THREADS / 32;
constexpr uint32_t AB_COMBINE = 256;  // splits x group <= this (the combine's factor table)

// dynamic shared memory of attn_gqa_batch_kernel
inline size_t attn_gqa_smem_bytes(uint32_t kv, uint32_t hd, uint32_t group, uint32_t chunk_pos) {
    const uint32_t chunk = (chunk_pos + 3u) & ~3u;
    const uint32_t half2 = ((hd / 2u + 1u) & ~1u) * 2u;
    size_t f = 2u * kv                          // k, v (rotated k)
               + group * (hd + 4u)              // q heads (rows padded by 4 floats)
               + half2                          // RoPE row
               + (size_t)group * chunk          // scores / weights
               + 2u * chunk                     // K and V scales of the split's positions
               + (size_t)AB_WARPS * group * hd  // per-warp V partial sums
               + 4u * group + 2u * AB_COMBINE;  // combine factors and sums
    return f * 4u + 2u * hd                     // + the current position's i8 K / V slice
           + (size_t)chunk * (2u * hd + 16u)    // + the split's cached K (padded) / V rows
           + 16u;
}

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
                 "l"(gmem_src)
                 : "memory");
}

__device__ __forceinline__ void cp_async4(void *smem_dst, const void *gmem_src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)),
                 "l"(gmem_src)
                 : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <uint32_t HD, uint32_t G>
__global__ void __launch_bounds__(AB_THREADS, 2) attn_gqa_batch_kernel(const __grid_constant__ AttnParams p) {
    static_assert((HD == 64 || HD == 128) && G >= 1 && G <= AB_MAX_GROUP, "shape");
    // (the host runs this kernel with n_rot % 4 == 0 and 16-byte aligned q / k / v rows)
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[AB_WARPS * 2 * AB_MAX_GROUP];
    __shared__ float s_sc[2];
    __shared__ uint32_t s_last;
    const uint32_t KV = p.n_kv_heads * HD, half = p.n_rot / 2u;
    const uint32_t kvh = blockIdx.x, z = blockIdx.y, sp = blockIdx.z;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t chunk_max = (p.chunk + 3u) & ~3u;
    float *ks = reinterpret_cast<float *>(smem);      // KV
    float *vs = ks + KV;                              // KV
    constexpr uint32_t QS = HD + 4u;                  // padded q row: the G heads on distinct banks
    float *qg = vs + KV;                              // G * QS
    float2 *rope = reinterpret_cast<float2 *>(qg + G * QS);  // half (rounded to 2)
    float *scores = reinterpret_cast<float *>(rope + ((half + 1u) & ~1u));  // G * chunk_max
    float *vsc = scores + (size_t)G * chunk_max;      // chunk_max
    float *ksc = vsc + chunk_max;                     // chunk_max
    float *vpart = ksc + chunk_max;                   // AB_WARPS * G * HD
    float *stat = vpart + (size_t)AB_WARPS * G * HD;  // 4 * G + 2 * AB_COMBINE
    int8_t *kq = reinterpret_cast<int8_t *>(stat + 4u * G + 2u * AB_COMBINE);  // HD
    int8_t *vq = kq + HD;                                          // HD
    constexpr uint32_t KR = HD + 16u;                 // padded K row: conflict-free 16-byte reads
    int8_t *ksm = vq + HD;                            // chunk_max * KR
    int8_t *vsm = ksm + (size_t)chunk_max * KR;       // chunk_max * HD

    pdl_launch_dependents();
    pdl_wait();
    if (p.tp.world && p.tp.wait) {  // q / k / v were gathered from every rank
        if (tid == 0 && !tp_wait(p.tp)) atomicOr(p.status, WL_DEV_ERR_PEER_TIMEOUT);
        __syncthreads();
    }
    const uint32_t pos = p.pos[z];  // (both loads in flight together)
    if (p.active && !p.active[z]) return;
    if (pos >= p.max_seq) {
        if (tid == 0) atomicOr(p.status, WL_DEV_ERR_POSITION);
        return;
    }
    const float *q_in = p.q + (size_t)z * p.qkv_stride, *k_in = p.k + (size_t)z * p.qkv_stride,
                *v_in = p.v + (size_t)z * p.qkv_stride;
    int8_t *k_cache = p.k_cache + z * p.cache_stride, *v_cache = p.v_cache + z * p.cache_stride;
    float *k_scale = p.k_scale + (size_t)z * p.scale_stride,
          *v_scale = p.v_scale + (size_t)z * p.scale_stride;
    // this split's positions [t0, t1) (splits of p.chunk positions: long
    // contexts take more CTAs, short ones fewer, so CTAs are equally long);
    // the cached ones (< pos) are requested now and land in shared memory
    // while the current position is prepared
    const uint32_t n = pos + 1u, S = (n + p.chunk - 1u) / p.chunk;
    if (sp >= S) return;
    const uint32_t t0 = sp * p.chunk, t1 = min(n, t0 + p.chunk), cnt = t1 - t0;
    const uint32_t nh = min(t1, pos) > t0 ? min(t1, pos) - t0 : 0u;  // cached positions
    // one round of 16-byte async copies: this step's k, v, the group's q
    // heads and the RoPE row (group 1), then the split's cached rows (group 2)
    const float2 *cs = p.rope + (size_t)pos * half;
    for (uint32_t i = tid; i < KV / 4u; i += AB_THREADS) {
        cp_async16(ks + 4u * i, k_in + 4u * i);
        cp_async16(vs + 4u * i, v_in + 4u * i);
    }
    for (uint32_t i = tid; i < G * HD / 4u; i += AB_THREADS)
        cp_async16(qg + (4u * i / HD) * QS + (4u * i) % HD, q_in + kvh * G * HD + 4u * i);
    for (uint32_t j = tid; j < half / 2u; j += AB_THREADS) cp_async16(rope + 2u * j, cs + 2u * j);
    cp_async_commit();
    {
        constexpr uint32_t U = HD / 16u;  // 16-byte units per row
        for (uint32_t i = tid; i < nh * U; i += AB_THREADS) {
            const uint32_t r = i / U, u = i % U;
            const size_t src = (size_t)(t0 + r) * KV + kvh * HD + u * 16u;
            cp_async16(ksm + (size_t)r * KR + u * 16u, k_cache + src);
            cp_async16(vsm + (size_t)r * HD + u * 16u, v_cache + src);
        }
        for (uint32_t i = tid; i < nh; i += AB_THREADS) {
            cp_async4(ksc + i, k_scale + t0 + i);
            cp_async4(vsc + i, v_scale + t0 + i);
        }
    }
    cp_async_commit();
    cp_async_wait_group<1>();  // group 1 has landed (group 2 may still be in flight)
    __syncthreads();
    const uint32_t pstep = p.rope_pairs ? 2u : 1u, poff = p.rope_pairs ? 1u : half;
    for (uint32_t i = tid; i < (p.n_kv_heads + G) * half; i += AB_THREADS) {
        const uint32_t hh = i / half, j = i % half;
        float *x = hh < p.n_kv_heads ? ks + hh * HD : qg + (hh - p.n_kv_heads) * QS;
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
                qi = quant_round_i8(__fmul_rn(x, isv ? iv : ik));
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
    cp_async_wait_all();
    __syncthreads();
    // 3. scores.  Each head's dot runs over the dimensions in order.  Short
    //    splits (positions x heads within one pass of the CTA) take one
    //    thread per (position, head), the G threads of a position adjacent so
    //    its K row is read once per warp, with the K bytes turned into floats
    //    by the 2^23 construction, (2^23 + (b + 128)) - (2^23 + 128) = b
    //    (exact, and cheaper than the convert instruction when few threads
    //    are busy); longer splits one thread per position for all G heads,
    //    each K row converted once.  Both give the same sums.
    if (cnt * G <= AB_THREADS) {
        if (tid < cnt * G) {
            const uint32_t i = tid / G, g = tid % G;
            const uint32_t t = t0 + i;
            const int8_t *kr = t == pos ? kq : ksm + (size_t)i * KR;
            const float sk = t == pos ? sk_cur : ksc[i];
            if (t == pos && g == 0) vsc[i] = sv_cur;
            const float *qh = qg + g * QS;
            float d = 0.0f;
#pragma unroll 2
            for (uint32_t c = 0; c < HD / 16u; ++c) {
                const uint4 w = *reinterpret_cast<const uint4 *>(kr + c * 16u);
                const uint32_t wv[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u,
                                        w.w ^ 0x80808080u};
#pragma unroll
                for (uint32_t e4 = 0; e4 < 4u; ++e4) {
                    const float4 q4 = *reinterpret_cast<const float4 *>(qh + c * 16u + e4 * 4u);
                    const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                    for (uint32_t e = 0; e < 4u; ++e) {
                        const float k8 = __fmul_rn(
                            __fsub_rn(__uint_as_float(__byte_perm(wv[e4], 0x4B000000u, 0x7440u + e)),
                                      8388736.0f),
                            sk);
                        d = __fmaf_rn(qv[e], k8, d);
                    }
                }
            }
            scores[g * chunk_max + i] = __fmul_rn(d, p.scale);
        }
    } else {
        for (uint32_t i = tid; i < cnt; i += AB_THREADS) {
            const uint32_t t = t0 + i;
            const int8_t *kr = t == pos ? kq : ksm + (size_t)i * KR;
            const float sk = t == pos ? sk_cur : ksc[i];
            if (t == pos) vsc[i] = sv_cur;
            float d[G];
#pragma unroll
            for (uint32_t g = 0; g < G; ++g) d[g] = 0.0f;
#pragma unroll
            for (uint32_t c = 0; c < HD / 16u; ++c) {
                const uint4 w = *reinterpret_cast<const uint4 *>(kr + c * 16u);
                const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (uint32_t e4 = 0; e4 < 4u; ++e4) {
                    float k8[4];
#pragma unroll
                    for (uint32_t e = 0; e < 4u; ++e)
                        k8[e] = __fmul_rn((float)(int8_t)(wv[e4] >> (8 * e)), sk);
#pragma unroll
                    for (uint32_t g = 0; g < G; ++g) {
                        const float4 q4 =
                            *reinterpret_cast<const float4 *>(qg + g * QS + c * 16u + e4 * 4u);
                        d[g] = __fmaf_rn(q4.x, k8[0], d[g]);
                        d[g] = __fmaf_rn(q4.y, k8[1], d[g]);
                        d[g] = __fmaf_rn(q4.z, k8[2], d[g]);
                        d[g] = __fmaf_rn(q4.w, k8[3], d[g]);
                    }
                }
            }
#pragma unroll
            for (uint32_t g = 0; g < G; ++g) scores[g * chunk_max + i] = __fmul_rn(d[g], p.scale);
        }
    }
    __syncthreads();
    // 4. per-head max and sum of exp
    float mx[G], sum[G];
    {
        float m[G];
#pragma unroll
        for (uint32_t g = 0; g < G; ++g) m[g] = -INFINITY;
        for (uint32_t i = tid; i < cnt; i += AB_THREADS)
#pragma unroll
            for (uint32_t g = 0; g < G; ++g)
                m[g] = fmaxf(m[g], scores[g * chunk_max + i]);
#pragma unroll
        for (uint32_t g = 0; g < G; ++g) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) m[g] = fmaxf(m[g], __shfl_xor_sync(0xffffffffu, m[g], off));
            if (lane == 0) red[warp * G + g] = m[g];
        }
        __syncthreads();
#pragma unroll
        for (uint32_t g = 0; g < G; ++g) {
            float t = red[g];
            for (uint32_t w = 1; w < AB_WARPS; ++w) t = fmaxf(t, red[w * G + g]);
            mx[g] = t;
        }
        __syncthreads();
        float l[G];
#pragma unroll
        for (uint32_t g = 0; g < G; ++g) l[g] = 0.0f;
        for (uint32_t i = tid; i < cnt; i += AB_THREADS)
#pragma unroll
            for (uint32_t g = 0; g < G; ++g)
                {
                    const float e = isfinite(mx[g]) ? exp_f32(__fsub_rn(scores[g * chunk_max + i], mx[g])) : 0.0f;
                    scores[g * chunk_max + i] = __fmul_rn(e, vsc[i]);  // the V scale folded in
                    l[g] += e;
                }
#pragma unroll
        for (uint32_t g = 0; g < G; ++g) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) l[g] += __shfl_xor_sync(0xffffffffu, l[g], off);
            if (lane == 0) red[warp * G + g] = l[g];
        }
        __syncthreads();
#pragma unroll
        for (uint32_t g = 0; g < G; ++g) {
            float t = red[g];
            for (uint32_t w = 1; w < AB_WARPS; ++w) t += red[w * G + g];
            sum[g] = t;
        }
    }
    // 5. o[g][d] = sum_i w_i * v8[i][d]: warp = every 8th position, lane =
    //    HD/32 dimensions (a 64-byte row of HD = 64 is one coalesced load)
    constexpr uint32_t DL = HD / 32u;  // dimensions per lane
    float acc[G][DL];
#pragma unroll
    for (uint32_t g = 0; g < G; ++g)
#pragma unroll
        for (uint32_t e = 0; e < DL; ++e) acc[g][e] = 0.0f;
    for (uint32_t i0 = warp; i0 < cnt; i0 += 8u * AB_WARPS) {
        uint32_t w[8];
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u) {
            const uint32_t i = i0 + u * AB_WARPS, t = t0 + i;
            w[u] = 0u;
            if (i < cnt) {
                const int8_t *vr = t == pos ? vq : vsm + (size_t)i * HD;
                if (DL == 4) w[u] = reinterpret_cast<const uint32_t *>(vr)[lane];
                else w[u] = reinterpret_cast<const uint16_t *>(vr)[lane];
            }
        }
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u) {
            const uint32_t i = i0 + u * AB_WARPS;
            if (i >= cnt) break;
            float v8[DL];
#pragma unroll
            for (uint32_t e = 0; e < DL; ++e) v8[e] = (float)(int8_t)(w[u] >> (8 * e));
#pragma unroll
            for (uint32_t g = 0; g < G; ++g) {
                const float wt = scores[g * chunk_max + i];
#pragma unroll
                for (uint32_t e = 0; e < DL; ++e) acc[g][e] = __fmaf_rn(wt, v8[e], acc[g][e]);
            }
        }
    }
#pragma unroll
    for (uint32_t g = 0; g < G; ++g)
#pragma unroll
        for (uint32_t e = 0; e < DL; ++e) vpart[((size_t)warp * G + g) * HD + lane * DL + e] = acc[g][e];
    __syncthreads();
    const uint32_t RS = HD + 4u;  // partial row: o[HD], max, sum
    float *part = p.partial + (((size_t)z * gridDim.x + kvh) * gridDim.z + sp) * G * RS;
#pragma unroll
    for (uint32_t g = 0; g < G; ++g)
        for (uint32_t d = tid; d < HD; d += AB_THREADS) {
            float o = 0.0f;
#pragma unroll
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
    if (tid == 0) {
#pragma unroll
        for (uint32_t g = 0; g < G; ++g) {
            part[g * RS + HD] = mx[g];
            part[g * RS + HD + 1] = sum[g];
        }
    }
    // Split hand-off: the barrier orders every thread's partial stores before
    // thread 0's acquire-release count (release is cumulative over them); the
    // last split's acquire, then the barrier, order its reads of the other
    // splits' partials after their stores.  (One atomic round trip instead of
    // a fence per thread plus the atomic.)
    __syncthreads();
    uint32_t *ctr = p.counters + (size_t)z * gridDim.x + kvh;
    if (tid == 0) {
        uint32_t old;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(ctr) : "memory");
        s_last = old == S - 1u ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    // combine: M = max m_s, f_s = exp(m_s - M), O = sum f_s o_s / sum f_s l_s.
    // Every split's (max, sum) pair and the first 16 splits' o values of this
    // thread's outputs are requested in one round of loads (the partials are
    // L2-resident, so the rounds, not the bytes, set the time); further
    // splits follow in rounds of 16.
    const float *base = p.partial + ((size_t)z * gridDim.x + kvh) * gridDim.z * G * RS;
    float *fac = stat;               // [S][G] maxima, then combine factors
    float *lsm = stat + AB_COMBINE;  // [S][G] sums (S * G <= AB_COMBINE, checked by the host)
    constexpr uint32_t OPT = (G * HD + AB_THREADS - 1u) / AB_THREADS;  // outputs per thread
    float v0[OPT][16];
#pragma unroll
    for (uint32_t k = 0; k < OPT; ++k) {
        const uint32_t i = tid + k * AB_THREADS;
        const uint32_t g = i / HD, d = i % HD;
#pragma unroll
        for (uint32_t u = 0; u < 16u; ++u)
            v0[k][u] = (i < G * HD && u < S) ? __ldcg(base + ((size_t)u * G + g) * RS + d) : 0.0f;
    }
    for (uint32_t i = tid; i < S * G; i += AB_THREADS) {
        fac[i] = __ldcg(base + (size_t)i * RS + HD);
        lsm[i] = __ldcg(base + (size_t)i * RS + HD + 1);
    }
    __syncthreads();
    if (tid < G) {
        const uint32_t g = tid;
        float M = -INFINITY;
        for (uint32_t s2 = 0; s2 < S; ++s2) M = fmaxf(M, fac[s2 * G + g]);
        float L = 0.0f;
        for (uint32_t s2 = 0; s2 < S; ++s2) {
            const float ms = fac[s2 * G + g];
            const float f = (isfinite(M) && ms > -INFINITY) ? expf(ms - M) : 0.0f;
            fac[s2 * G + g] = f;
            L += lsm[s2 * G + g] * f;
        }
        red[g] = !isfinite(M) ? 0.0f : (L > 0.0f ? __fdiv_rn(1.0f, L) : 1.0f);
    }
    __syncthreads();
#pragma unroll
    for (uint32_t k = 0; k < OPT; ++k) {
        const uint32_t i = tid + k * AB_THREADS;
        if (i >= G * HD) break;
        const uint32_t g = i / HD, d = i % HD;
        float o = 0.0f;
#pragma unroll
        for (uint32_t u = 0; u < 16u; ++u)
            if (u < S) o = __fmaf_rn(v0[k][u], fac[u * G + g], o);
        for (uint32_t s0 = 16u; s0 < S; s0 += 16u) {
            float v[16];
#pragma unroll
            for (uint32_t u = 0; u < 16u; ++u)
                v[u] = s0 + u < S ? __ldcg(base + ((size_t)(s0 + u) * G + g) * RS + d) : 0.0f;
#pragma unroll
            for (uint32_t u = 0; u < 16u; ++u)
                if (s0 + u < S) o = __fmaf_rn(v[u], fac[(s0 + u) * G + g], o);
        }
        p.att[(size_t)z * p.att_stride + (kvh * G + g) * HD + d] = __fmul_rn(o, red[g]);
    }
    if (tid == 0) *ctr = 0u;  // re-arm for the next launch
}

}  // namespace wl
