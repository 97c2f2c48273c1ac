// i2s_stream.cuh -- many independent I2_S matvecs in one persistent launch.
//
// Same arithmetic as i2s_matvec_kernel (bitlinear_sse2.rs:313-342 semantics,
// bit-exact), organised for sustained HBM streaming: the rows of all ops
// are concatenated into one row space, each of the (one per SM) CTAs owns a
// contiguous, byte-balanced range of it, a producer warp streams that range
// through a 6-stage shared-memory ring with 1-D bulk copies, and eight
// consumer warps compute rows as stages land.  A CTA's range touches only a
// few ops, so activation reloads (op switches) are rare.  Inputs are
// quantised beforehand by quantize_jobs_kernel (one CTA per distinct input).
#pragma once

#include <cstdint>

#include "i2s_matvec.cuh"
#include "wl_ptx.cuh"

namespace wl {

constexpr int STREAM_CONSUMER_WARPS = 8;
constexpr int STREAM_THREADS = (STREAM_CONSUMER_WARPS + 1) * 32;
constexpr int STREAM_LPR = 16;  // lanes per row
constexpr int STREAM_NP = 7;    // 16-byte weight slots per lane -> K <= 7168
constexpr uint32_t STREAM_MAX_K = STREAM_LPR * STREAM_NP * 64;
constexpr int STREAM_STAGES = 6;
constexpr uint32_t STREAM_STAGE_BYTES = 32u * 1024u;
constexpr uint32_t STREAM_ROWS_PER_PASS = STREAM_CONSUMER_WARPS * (32 / STREAM_LPR);

struct I2sStreamOp {
    const uint8_t *w;         // N x K/4 packed bytes, 16-byte aligned
    const int8_t *q;          // quantised input, K bytes
    const float *act_scale;   // its scale
    float *y;
    int32_t *acc;             // may be null
    float w_scale;
    uint32_t K, N, row_begin;
};

struct I2sStreamParams {
    const I2sStreamOp *ops;
    uint32_t n_ops;
    const uint32_t *cta_rows;  // gridDim.x + 1 row boundaries
    uint32_t *status;
};

struct QuantJob {
    const float *x;
    int8_t *q;
    float *scale;
    uint32_t n;
};

// One CTA per distinct input vector; same steps as quantize_absmax_kernel.
__global__ void __launch_bounds__(QUANT_THREADS)
    quantize_jobs_kernel(const QuantJob *__restrict__ jobs) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float red[QUANT_THREADS / 32];
    const QuantJob j = jobs[blockIdx.x];
    float m = 0.0f;
    for (uint32_t i = threadIdx.x * 4; i < j.n; i += QUANT_THREADS * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(j.x + i);
        m = fmaxf(fmaxf(fmaxf(m, fabsf(v.x)), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    float max_abs = red[0];
#pragma unroll
    for (int w = 1; w < QUANT_THREADS / 32; ++w) max_abs = fmaxf(max_abs, red[w]);
    const float inv = max_abs == 0.0f ? 0.0f : __fdiv_rn(127.0f, max_abs);
    for (uint32_t i = threadIdx.x * 4; i < j.n; i += QUANT_THREADS * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(j.x + i);
        const float e[4] = {v.x, v.y, v.z, v.w};
        uint32_t packed = 0;
        if (max_abs != 0.0f) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float r = roundf(__fmul_rn(e[k], inv));
                const int qi = isnan(r) ? 0 : (int)fminf(fmaxf(r, -127.0f), 127.0f);
                packed |= (uint32_t)(qi & 0xFF) << (8 * k);
            }
        }
        *reinterpret_cast<uint32_t *>(j.q + i) = packed;
    }
    if (threadIdx.x == 0) *j.scale = max_abs == 0.0f ? 1.0f : __fdiv_rn(max_abs, 127.0f);
}

__host__ __device__ constexpr uint32_t stream_chunk_rows(uint32_t K) {
    return (STREAM_STAGE_BYTES / (STREAM_ROWS_PER_PASS * (K >> 2)) > 0
                ? STREAM_STAGE_BYTES / (STREAM_ROWS_PER_PASS * (K >> 2))
                : 1u) *
           STREAM_ROWS_PER_PASS;
}

// Deterministic chunk walk over [r, r1): producer and consumers step through
// the same sequence.  A chunk never crosses an op boundary.
struct ChunkWalk {
    uint32_t j, r, n;
};

__device__ __forceinline__ bool chunk_next(const I2sStreamOp *__restrict__ ops, uint32_t n_ops,
                                           uint32_t r1, ChunkWalk &w) {
    w.r += w.n;
    if (w.r >= r1) return false;
    while (w.j < n_ops && w.r >= ops[w.j].row_begin + ops[w.j].N) ++w.j;
    if (w.j >= n_ops) return false;
    const I2sStreamOp &op = ops[w.j];
    w.n = min(min(stream_chunk_rows(op.K), op.row_begin + op.N - w.r), r1 - w.r);
    return true;
}

template <bool C3>
__global__ void __launch_bounds__(STREAM_THREADS, 1)
    i2s_stream_kernel(const __grid_constant__ I2sStreamParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[STREAM_STAGES];
    __shared__ __align__(8) uint64_t empty_bar[STREAM_STAGES];
    __shared__ uint32_t s_timeout;

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t r0 = p.cta_rows[blockIdx.x], r1 = p.cta_rows[blockIdx.x + 1];
    // first op of the range
    uint32_t j0 = 0;
    {
        uint32_t lo = 0, hi = p.n_ops;
        while (lo + 1 < hi) {
            const uint32_t mid = (lo + hi) / 2;
            if (p.ops[mid].row_begin <= r0) lo = mid; else hi = mid;
        }
        j0 = lo;
    }
    if (tid == 0) {
        for (int s = 0; s < STREAM_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], STREAM_CONSUMER_WARPS);
        }
        fence_mbar_init();
        s_timeout = 0;
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == STREAM_CONSUMER_WARPS) {
        if (lane == 0) {  // producer: weights do not depend on the previous kernel
            const uint64_t policy = l2_policy_evict_first();
            ChunkWalk w = {j0, r0, 0};
            for (uint32_t k = 0; chunk_next(p.ops, p.n_ops, r1, w); ++k) {
                const uint32_t st = k % STREAM_STAGES;
                if (k >= STREAM_STAGES &&
                    !mbar_wait(&empty_bar[st], ((k / STREAM_STAGES) - 1u) & 1u)) {
                    atomicOr(&s_timeout, 1u);
                    break;
                }
                const I2sStreamOp &op = p.ops[w.j];
                const uint32_t rb = op.K >> 2;
                mbar_arrive_expect_tx(&full_bar[st], w.n * rb);
                bulk_g2s_evict_first(smem + st * STREAM_STAGE_BYTES,
                                     op.w + (size_t)(w.r - op.row_begin) * rb, w.n * rb,
                                     &full_bar[st], policy);
            }
        }
    } else {
        pdl_wait();  // quantised inputs come from the previous kernel
        const uint32_t s = lane % STREAM_LPR, sub = lane / STREAM_LPR;
        uint4 act[STREAM_NP][4];
        int32_t asum = 0;
        float combined = 0.0f;
        uint32_t cur = 0xFFFFFFFFu, P = 0;
        ChunkWalk w = {j0, r0, 0};
        for (uint32_t k = 0; chunk_next(p.ops, p.n_ops, r1, w); ++k) {
            const uint32_t st = k % STREAM_STAGES;
            if (!__all_sync(0xffffffffu, mbar_wait(&full_bar[st], (k / STREAM_STAGES) & 1u))) {
                if (lane == 0) atomicOr(&s_timeout, 1u);
                break;
            }
            const I2sStreamOp &op = p.ops[w.j];
            if (w.j != cur) {  // op switch: reload this lane's activations
                cur = w.j;
                P = op.K >> 6;
                asum = 0;
#pragma unroll
                for (int i = 0; i < STREAM_NP; ++i) {
                    const uint32_t pp = s + STREAM_LPR * i;
                    if (pp < P) {
                        i2s_load_act(op.q, pp, act[i]);
#pragma unroll
                        for (int o = 0; o < 4; ++o) asum += sum_bytes(act[i][o]);
                    } else {
#pragma unroll
                        for (int o = 0; o < 4; ++o) act[i][o] = make_uint4(0, 0, 0, 0);
                    }
                }
                combined = __fmul_rn(op.w_scale, *op.act_scale);
            }
            const uint32_t rb = op.K >> 2;
            const uint8_t *stage = smem + st * STREAM_STAGE_BYTES;
            for (uint32_t base = 0; base < w.n; base += STREAM_ROWS_PER_PASS) {
                const uint32_t row_local = base + warp * (32 / STREAM_LPR) + sub;
                const bool valid = row_local < w.n;
                const uint8_t *rp = stage + row_local * rb;
                I2sAcc acc = {0, 0, 0, 0};
                uint32_t c3 = 0;
                if (valid) {
#pragma unroll
                    for (int i = 0; i < STREAM_NP; ++i) {
                        const uint32_t pp = s + STREAM_LPR * i;
                        if (pp < P)
                            i2s_slot<C3>(*reinterpret_cast<const uint4 *>(rp + 16 * pp), act[i],
                                         acc, c3);
                    }
                }
                int32_t dot = i2s_acc_total(acc) - asum;
#pragma unroll
                for (int off = STREAM_LPR / 2; off > 0; off >>= 1) {
                    dot += __shfl_xor_sync(0xffffffffu, dot, off);
                    if constexpr (C3) c3 |= __shfl_xor_sync(0xffffffffu, c3, off);
                }
                if constexpr (C3) {
                    if ((c3 & 0x55555555u) != 0u) {
                        int32_t corr = valid ? i2s_row_c3(rp, op.q, s, STREAM_LPR, P) : 0;
                        const uint32_t grp = __match_any_sync(__activemask(), row_local);
#pragma unroll
                        for (int off = STREAM_LPR / 2; off > 0; off >>= 1)
                            corr += __shfl_xor_sync(grp, corr, off);
                        dot -= 2 * corr;
                    }
                }
                if (s == 0 && valid) {
                    const uint32_t local = w.r + row_local - op.row_begin;
                    op.y[local] = __fmul_rn(combined, __int2float_rn(dot));
                    if (op.acc) op.acc[local] = dot;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[st]);
        }
    }
    __syncthreads();
    if (tid == 0 && s_timeout) atomicOr(p.status, WL_DEV_ERR_TIMEOUT);
}

}  // namespace wl
