// q6k_lmhead.cuh -- Q6_K tied lm-head (logits + greedy argmax) for sm_100a.
//
// Reference: compute_logits (src/model/lm_head.rs:29-108) -> q6_k::dot_row
// (src/model/q6_k.rs:71-82) -> dot_row_sse2_validated
// (src/model/q6_k_sse2.rs:46-116); argmax (src/model/lm_head.rs:161-174).
//
// Bit-exact logits.  The reference's SSE2 row dot keeps 16 independent f32
// accumulation chains: 4 vector accumulators (one per quarter a = q1..q4 of
// each 128-value half) x 4 lanes k.  Chain (a, k) visits, in order, blocks
// b, halves h, and l = k, k+4, ..., k+28 of
//     acc += (q * (d * sc)) * x          (two roundings, never an FMA)
// with q = 6-bit value - 32, then reduces
//     v_k = (acc_0k + acc_1k) + (acc_2k + acc_3k),
//     logit = (v_0 + v_3) + (v_1 + v_2).
// Here one thread owns quarter a of one row and runs that quarter's four
// chains with the same IEEE round-to-nearest operations (__fmul_rn /
// __fadd_rn: no contraction), then the four threads of a row combine their
// chains with the same tree.  The int->float conversion of q uses the
// 2^23 magic-number construction, which is exact; it and q * (d * sc) run as
// packed f32 pairs (two values per instruction), which round each lane as
// the scalar operations do.
//
// Device layout (one-time repack, q6k_repack_kernel): each row becomes
//   [ql: nb x 128][qh: nb x 64][sc: nb x 16][d: nb x 2][pad to 16 B]
// (nb = n_embd / 256; 2112 bytes per row at n_embd 2560, 0.57 % above the
// GGUF 2100) so rows and sections are 16-byte aligned for bulk copies.
//
// Streaming: one launch for the whole batch.  The batch is cut into groups of
// BG hidden rows (BG = 1, 2, 4 or 8); the grid is (batch groups) x (vocab
// ranges), about one CTA per SM, and each CTA stages its group's hidden rows
// in shared memory once.  A producer warp streams the range's 32-row chunks
// into a 2-3 stage shared-memory ring with 1-D bulk copies; two consumer
// groups of 4 warps take alternate chunks, and each decoded weight value is
// used for all BG hidden rows.  The CTAs of different batch groups stream the
// same vocab range at the same time, so with more than one group the weight
// bytes come from DRAM once and from L2 for the other groups.
//
// Argmax: key = (orderable(logit) << 32) | (0xFFFFFFFF - row); the maximum
// key is the reference's answer (ties -> lowest row, -0.0 == +0.0, NaN never
// wins, except a NaN at row 0, which the strict '>' scan keeps).  CTAs
// atomicMax into a per-batch-row slot; the last CTA to finish writes the ids
// of every batch row and re-zeroes the slots and its counter.
#pragma once

#include <cstdint>

#include "tp.cuh"
#include "wl_ptx.cuh"

namespace wl {

constexpr int Q6K_CONSUMER_WARPS = 8;
constexpr int Q6K_THREADS = (Q6K_CONSUMER_WARPS + 1) * 32;
constexpr int Q6K_GROUP_THREADS = 128;  // 4 warps per consumer group
constexpr int Q6K_ROWS_PER_CHUNK = Q6K_GROUP_THREADS / 4;  // 4 threads per row
constexpr int Q6K_STAGES = 3;
constexpr int Q6K_MAX_BG = 8;

__host__ __device__ constexpr uint32_t q6k_row_stride(uint32_t nb) {
    return (nb * 208u + ((nb * 2u + 15u) & ~15u));
}

// x index -> padded shared-memory index (4 floats of padding per 32 so the
// four quarters of a row read distinct banks).
__device__ __forceinline__ uint32_t q6k_xpad(uint32_t i) { return i + (i >> 5) * 4u; }

struct Q6kParams {
    const uint8_t *packed;   // vocab x row_stride bytes, device layout
    uint32_t n_embd, vocab, nb, row_stride;
    uint32_t rows_per_cta;   // rows of one vocab range
    uint32_t n_ranges;       // vocab ranges; CTA c: range c % n_ranges, group c / n_ranges
    uint32_t batch;          // hidden rows (all groups)
    uint32_t nstages;        // 2 or 3 (<= Q6K_STAGES), whatever fits in shared memory
    uint32_t l2_keep;        // several groups read each range: no evict-first hint
    const float *hidden;     // batch x n_embd
    float *logits;           // batch x vocab or null
    uint32_t *ids;           // batch or null
    unsigned long long *slots;  // batch argmax slots (zero on entry)
    uint32_t *counter;          // CTA completion counter (zero on entry)
    uint32_t *status;
    uint32_t row_offset;        // vocab shard: global id of local row 0
    TpParams tp;                // world 0: single GPU (ids written here)
};

// Vocab-sharded argmax exchange: rank s writes its best key for batch row b
// to keys[s][b] of every rank's symmetric block.
constexpr uint32_t TP_KEYS_OFF = 1024;
constexpr uint32_t TP_MAX_BATCH = 64;
// Key slots: [set 0..1][source rank][batch row].  Successive lm-head calls
// alternate sets (the parity of this rank's lm-head call counter, bumped by
// the finalize kernel), so a rank that runs ahead into the next call cannot
// overwrite keys a slower rank has not reduced yet: it can only get one call
// ahead, since its next finalize waits for the slower rank's arrivals.
static_assert(TP_KEYS_OFF + 2 * TP_MAX_WORLD * TP_MAX_BATCH * 8 <= TP_HEADER_BYTES, "key slots");
__device__ __forceinline__ unsigned long long *tp_key_slot(uint8_t *base, uint32_t set, int src,
                                                           uint32_t b) {
    return reinterpret_cast<unsigned long long *>(base + TP_KEYS_OFF) +
           (set * TP_MAX_WORLD + src) * TP_MAX_BATCH + b;
}
__device__ __forceinline__ uint32_t tp_key_set(const TpParams &tp) {
    return *reinterpret_cast<volatile uint32_t *>(tp.local_base + TP_LMCALL_OFF) & 1u;
}

// After every rank's lm-head shard: wait for all keys, reduce, decode ids,
// then advance this rank's lm-head call counter (selects the next key set).
__global__ void q6k_tp_finalize_kernel(const TpParams tp, uint32_t batch, uint32_t *ids,
                                       uint32_t *status) {
    __shared__ uint32_t ok, set;
    if (threadIdx.x == 0) {
        set = tp_key_set(tp);
        ok = tp_wait(tp) ? 1u : 0u;
        if (!ok) atomicOr(status, WL_DEV_ERR_PEER_TIMEOUT);
    }
    __syncthreads();
    for (uint32_t b = threadIdx.x; b < batch; b += blockDim.x) {
        unsigned long long best = 0ull;
        for (int s = 0; s < tp.world; ++s) {
            const unsigned long long k =
                *(volatile unsigned long long *)tp_key_slot(tp.local_base, set, s, b);
            best = best > k ? best : k;
        }
        ids[b] = 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        volatile uint32_t *calls =
            reinterpret_cast<volatile uint32_t *>(tp.local_base + TP_LMCALL_OFF);
        *calls = *calls + 1u;
    }
}

__device__ __forceinline__ uint32_t f32_order_key(float v, uint32_t row) {
    if (isnan(v)) return row == 0 ? 0xFFFFFFFFu : 0u;
    if (v == 0.0f) v = 0.0f;  // -0.0 ties with +0.0
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    // primitives.rs:61-88, exact (incl. subnormals, inf, NaN payload).
    const uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    if (exp == 0) {
        if (man == 0) return __uint_as_float(sign << 31);
        const float val = __fmul_rn((float)man, 5.9604644775390625e-8f);  // 2^-24
        return sign ? -val : val;
    }
    if (exp == 0x1F) return __uint_as_float((sign << 31) | (0xFFu << 23) | (man << 13));
    return __uint_as_float((sign << 31) | ((exp + 112u) << 23) | (man << 13));
}

// Repack GGUF Q6_K rows (210-byte super-blocks) into the device layout.
__global__ void q6k_repack_kernel(const uint8_t *__restrict__ raw, uint32_t nb, uint32_t vocab,
                                  uint8_t *__restrict__ out) {
    const uint32_t stride = q6k_row_stride(nb);
    const size_t total = (size_t)vocab * nb;
    for (size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (size_t)gridDim.x * blockDim.x) {
        const uint32_t row = (uint32_t)(t / nb), b = (uint32_t)(t % nb);
        const uint8_t *src = raw + ((size_t)row * nb + b) * 210u;
        uint8_t *dst = out + (size_t)row * stride;
        for (int i = 0; i < 128; ++i) dst[b * 128u + i] = src[i];
        for (int i = 0; i < 64; ++i) dst[nb * 128u + b * 64u + i] = src[128 + i];
        for (int i = 0; i < 16; ++i) dst[nb * 192u + b * 16u + i] = src[192 + i];
        dst[nb * 208u + b * 2u] = src[208];
        dst[nb * 208u + b * 2u + 1] = src[209];
        if (b == 0)
            for (uint32_t i = nb * 210u; i < stride; ++i) dst[i] = 0;
    }
}

template <int BG>
__global__ void __launch_bounds__(Q6K_THREADS, 1)
    q6k_lmhead_kernel(const __grid_constant__ Q6kParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[Q6K_STAGES];
    __shared__ __align__(8) uint64_t empty_bar[Q6K_STAGES];
    __shared__ unsigned long long cta_best[BG];
    __shared__ uint32_t s_timeout;
    __shared__ uint32_t s_last;

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t chunk_bytes = Q6K_ROWS_PER_CHUNK * p.row_stride;
    const uint32_t nst = p.nstages;
    float *xs = reinterpret_cast<float *>(smem + nst * chunk_bytes);
    const uint32_t xs_len = p.n_embd + p.n_embd / 8;  // padded floats per batch row

    const uint32_t range = blockIdx.x % p.n_ranges, bgrp = blockIdx.x / p.n_ranges;
    const uint32_t b0 = bgrp * BG;                              // first hidden row
    const uint32_t gcnt = min((uint32_t)BG, p.batch - b0);      // rows of this group
    const uint32_t r0 = range * p.rows_per_cta;
    const uint32_t r1 = min(r0 + p.rows_per_cta, p.vocab);
    const uint32_t nchunks = r0 < r1 ? (r1 - r0 + Q6K_ROWS_PER_CHUNK - 1) / Q6K_ROWS_PER_CHUNK : 0;

    if (tid == 0) {
        for (uint32_t s = 0; s < nst; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], Q6K_GROUP_THREADS / 32);
        }
        fence_mbar_init();
        s_timeout = 0;
    }
    if (tid < BG) cta_best[tid] = 0ull;
    __syncthreads();

    pdl_launch_dependents();

    if (warp == Q6K_CONSUMER_WARPS) {
        // Producer warp: one elected lane streams the chunks.  The weights do
        // not depend on the previous kernel, so streaming starts before the
        // programmatic-dependency wait.
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            for (uint32_t c = 0; c < nchunks; ++c) {
                const uint32_t st = c % nst;
                if (c >= nst) {
                    if (!mbar_wait(&empty_bar[st], ((c / nst) - 1u) & 1u)) {
                        atomicOr(&s_timeout, 1u);
                        break;
                    }
                }
                const uint32_t a = r0 + c * Q6K_ROWS_PER_CHUNK;
                const uint32_t b = min(a + Q6K_ROWS_PER_CHUNK, r1);
                const uint32_t bytes = (b - a) * p.row_stride;
                mbar_arrive_expect_tx(&full_bar[st], bytes);
                if (p.l2_keep)
                    bulk_g2s(smem + st * chunk_bytes, p.packed + (size_t)a * p.row_stride, bytes,
                             &full_bar[st]);
                else
                    bulk_g2s_evict_first(smem + st * chunk_bytes,
                                         p.packed + (size_t)a * p.row_stride, bytes, &full_bar[st],
                                         policy);
            }
        }
    } else {
        // Consumers: wait for the previous kernel (the hidden rows, and the
        // argmax scratch of a previous call), then stage this group's hidden
        // rows (padded; rows past the batch as zeros) in shared memory.
        pdl_wait();
        for (uint32_t i = tid; i < BG * p.n_embd; i += Q6K_CONSUMER_WARPS * 32) {
            const uint32_t bg = i / p.n_embd, e = i % p.n_embd;
            xs[bg * xs_len + q6k_xpad(e)] = bg < gcnt ? p.hidden[(size_t)(b0 + bg) * p.n_embd + e] : 0.0f;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(Q6K_CONSUMER_WARPS * 32));

        const uint32_t group = warp / 4;
        const uint32_t gtid = tid - group * Q6K_GROUP_THREADS;
        const uint32_t row_local = gtid >> 2;
        const uint32_t a = gtid & 3u;
        const uint32_t nb = p.nb;
        unsigned long long best[BG];
#pragma unroll
        for (int g = 0; g < BG; ++g) best[g] = 0ull;

        for (uint32_t c = group; c < nchunks; c += 2) {
            const uint32_t st = c % nst;
            // Warp-uniform decision, so a timeout never splits a warp.
            if (!__all_sync(0xffffffffu, mbar_wait(&full_bar[st], (c / nst) & 1u))) {
                if (lane == 0) atomicOr(&s_timeout, 1u);
                break;
            }
            const uint32_t row = r0 + c * Q6K_ROWS_PER_CHUNK + row_local;
            const uint8_t *rp = smem + st * chunk_bytes + row_local * p.row_stride;
            float acc[BG][4];
#pragma unroll
            for (int g = 0; g < BG; ++g)
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[g][k] = 0.0f;

            if (row < r1) {
                const uint8_t *ql_sec = rp, *qh_sec = rp + nb * 128u, *sc_sec = rp + nb * 192u;
                const uint16_t *d_sec = reinterpret_cast<const uint16_t *>(rp + nb * 208u);
                const uint32_t ql_shift = (a >> 1) * 4u, qh_shift = a * 2u;
                for (uint32_t b = 0; b < nb; ++b) {
                    const float d = f16_bits_to_f32(d_sec[b]);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int8_t *sc = reinterpret_cast<const int8_t *>(sc_sec + b * 16u + h * 8);
                        const float s0 = __fmul_rn(d, (float)sc[a * 2]);
                        const float s1 = __fmul_rn(d, (float)sc[a * 2 + 1]);
                        const uint4 qlv0 = *reinterpret_cast<const uint4 *>(
                            ql_sec + b * 128u + h * 64 + (a & 1u) * 32u);
                        const uint4 qlv1 = *reinterpret_cast<const uint4 *>(
                            ql_sec + b * 128u + h * 64 + (a & 1u) * 32u + 16u);
                        const uint4 qhv0 =
                            *reinterpret_cast<const uint4 *>(qh_sec + b * 64u + h * 32);
                        const uint4 qhv1 =
                            *reinterpret_cast<const uint4 *>(qh_sec + b * 64u + h * 32 + 16);
                        const uint32_t qlw[8] = {qlv0.x, qlv0.y, qlv0.z, qlv0.w,
                                                 qlv1.x, qlv1.y, qlv1.z, qlv1.w};
                        const uint32_t qhw[8] = {qhv0.x, qhv0.y, qhv0.z, qhv0.w,
                                                 qhv1.x, qhv1.y, qhv1.z, qhv1.w};
                        const uint32_t xbase = b * 256u + h * 128u + a * 32u;
                        const float2 bias = make_float2(-8388640.0f, -8388640.0f);
#pragma unroll
                        for (int m = 0; m < 8; ++m) {
                            const uint32_t u4 = ((qlw[m] >> ql_shift) & 0x0F0F0F0Fu) |
                                                (((qhw[m] >> qh_shift) & 0x03030303u) << 4);
                            const float sc_f = m < 4 ? s0 : s1;
                            const float2 sc2 = make_float2(sc_f, sc_f);
                            // (2^23 + u) - (2^23 + 32) = u - 32, then q * (d * sc):
                            // both exact, as packed pairs (an add feeding a
                            // multiply cannot become an FMA).
                            float2 w[2];
#pragma unroll
                            for (int j = 0; j < 2; ++j) {
                                const float2 qf = f2_add_rn(
                                    make_float2(
                                        __uint_as_float(__byte_perm(u4, 0x4B000000u, 0x7440 + 2 * j)),
                                        __uint_as_float(
                                            __byte_perm(u4, 0x4B000000u, 0x7441 + 2 * j))),
                                    bias);
                                w[j] = f2_mul_rn(qf, sc2);
                            }
#pragma unroll
                            for (int g = 0; g < BG; ++g) {
                                const float4 xv = *reinterpret_cast<const float4 *>(
                                    xs + g * xs_len + q6k_xpad(xbase + 4u * m));
                                // (q * (d * sc)) * x rounded once, then the
                                // chain add rounded once: the product as an
                                // FMA with a +0 addend (never simplified to a
                                // plain multiply, so never fused with the add;
                                // equal to the product here because a chain
                                // that starts at +0 is never -0).
                                const float2 p0 = f2_fma_rn(w[0], make_float2(xv.x, xv.y),
                                                            make_float2(0.0f, 0.0f));
                                const float2 p1 = f2_fma_rn(w[1], make_float2(xv.z, xv.w),
                                                            make_float2(0.0f, 0.0f));
                                const float2 a01 = f2_add_rn(make_float2(acc[g][0], acc[g][1]), p0);
                                const float2 a23 = f2_add_rn(make_float2(acc[g][2], acc[g][3]), p1);
                                acc[g][0] = a01.x;
                                acc[g][1] = a01.y;
                                acc[g][2] = a23.x;
                                acc[g][3] = a23.y;
                            }
                        }
                    }
                }
            }
            // Release the stage (all loads of this chunk are done).
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[st]);

            // Combine the 16 chains exactly as _mm_add_ps / hsum do.
#pragma unroll
            for (int g = 0; g < BG; ++g) {
                float v[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float other = __shfl_down_sync(0xffffffffu, acc[g][k], 1);
                    const float pair = __fadd_rn(acc[g][k], other);  // lanes a=0: q1+q2, a=2: q3+q4
                    const float hi = __shfl_down_sync(0xffffffffu, pair, 2);
                    v[k] = __fadd_rn(pair, hi);                      // lane a=0
                }
                const float logit = __fadd_rn(__fadd_rn(v[0], v[3]), __fadd_rn(v[1], v[2]));
                if (a == 0 && row < r1 && (uint32_t)g < gcnt) {
                    if (p.logits) p.logits[(size_t)(b0 + g) * p.vocab + row] = logit;
                    const unsigned long long key =
                        ((unsigned long long)f32_order_key(logit, row + p.row_offset) << 32) |
                        (unsigned long long)(0xFFFFFFFFu - (row + p.row_offset));
                    best[g] = best[g] > key ? best[g] : key;
                }
            }
        }
        if (p.ids) {
#pragma unroll
            for (int g = 0; g < BG; ++g) {
                unsigned long long k = best[g];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
                    k = k > o ? k : o;
                }
                if (lane == 0) atomicMax(&cta_best[g], k);
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        if (s_timeout) atomicOr(p.status, WL_DEV_ERR_TIMEOUT);
        if (p.ids) {
            for (uint32_t g = 0; g < gcnt; ++g) atomicMax(&p.slots[b0 + g], cta_best[g]);
            __threadfence();
            s_last = atomicAdd(p.counter, 1u) == gridDim.x - 1 ? 1u : 0u;
        } else {
            s_last = 0;
        }
    }
    __syncthreads();
    if (s_last) {
        __threadfence();
        const uint32_t set = p.tp.world ? tp_key_set(p.tp) : 0u;
        for (uint32_t b = tid; b < p.batch; b += blockDim.x) {
            const unsigned long long k = atomicExch(&p.slots[b], 0ull);
            if (p.tp.world) {
                for (int r = 0; r < p.tp.world; ++r)
                    *tp_key_slot(p.tp.peer_base[r], set, p.tp.rank, b) = k;
            } else {
                p.ids[b] = 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
            }
        }
        if (tid == 0) *p.counter = 0u;
    }
    if (p.tp.world && s_last) {  // one arrival per rank per launch, after the key stores
        __syncthreads();
        if (tid == 0) tp_signal(p.tp);
    }
}

}  // namespace wl
