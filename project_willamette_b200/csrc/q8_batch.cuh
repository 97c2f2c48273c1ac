// q8_batch.cuh -- batched Q8_0 linears for decoding many independent
// sequences at once (one token per sequence per step), and the batched
// embedding / final-norm kernels around them.
//
// Reference: q8_0_matvec_f32 (src/model/linear.rs:171-224), one call per
// sequence, rows through q8_0::dot_row (src/model/q8_0.rs:50-70) ->
// dot_row_avx2 (src/model/q8_0_simd.rs:72-104); the lm-head arm of
// compute_logits (src/model/lm_head.rs:103) + argmax (lm_head.rs:161-174).
//
// Work split.  A CTA owns 32 * rg weight rows (paired mode: 32 * rg rows of
// each of two jobs, gate and up) and a group of TG tokens.  Its weight rows
// (contiguous in the repacked layout) arrive in shared memory by one bulk
// copy per job, issued before the wait on the previous kernel (the weights
// do not depend on it); the activations follow by bulk copy after it.  The 8
// warps are (row group x block phase): lane = row, every lane of a warp reads
// the SAME 32 activations of a token (broadcast).  Each weight block is
// converted to f32 once and used for all TG tokens.
//
// Arithmetic per (row, token), exact mode (the reference's, bit for bit):
//     s_j = (((0 + q_j x_j) + q_{8+j} x_{8+j}) + q_{16+j} x_{16+j}) + q_{24+j} x_{24+j}
//     hs  = ((s_0 + s_4) + (s_2 + s_6)) + ((s_1 + s_5) + (s_3 + s_7))
//     total = (((0 + d_0 hs_0) + d_1 hs_1) + ...)      blocks in order
// Block terms of different phases meet in shared memory and are summed in
// block order.  Fast mode contracts q_j x_j + s_j into one FMA (rounding-level
// differences; everything else is the same).
//
// Epilogues: store; residual add (hidden += y, non-finite flagged, as
// cached_forward.rs:507-517 does after each layer); SiLU pair
// (silu(gate) * up, ffn.rs:45-65); argmax (the greedy id of every token).
#pragma once

#include <cstdint>

#include "bitnet_decode.cuh"  // block reductions, exp_f32, WL_DEV_ERR_*
#include "q8_0.cuh"           // q8_row_stride, f16_bits_to_f32

namespace wl {

constexpr int QB_THREADS = 256;
constexpr uint32_t QB_WARPS = QB_THREADS / 32;
constexpr uint32_t QB_MAX_JOBS = 3;

enum : uint32_t { QB_PRE_NONE = 0, QB_PRE_RMSNORM = 1 };
enum : uint32_t { QB_EPI_STORE = 0, QB_EPI_RESIDUAL = 1, QB_EPI_SILU_PAIR = 2, QB_EPI_ARGMAX = 3 };

struct Q8BatchJob {
    const uint8_t *w;  // repacked Q8_0 rows, q8_row_stride(K) bytes each
    uint32_t n;        // rows
    uint32_t y_off;    // column of the job's row 0 in a token's output row
    uint32_t tile0;    // first row tile of the job (grid x)
};

struct Q8BatchParams {
    Q8BatchJob job[QB_MAX_JOBS];
    uint32_t n_jobs;
    uint32_t K;         // multiple of 32
    uint32_t n_tokens;  // tokens of the launch (grid y covers them in groups)
    uint32_t rg;        // 32-row groups per job set (1, 2, 4, 8; paired: 1, 2, 4)
    uint32_t stage_w;   // 1: the CTA's weight rows are bulk-copied to shared memory before
                        // the dependency wait; 0: each lane reads its row from global memory
                        // (the lm-head: no wait worth hiding, and its 256-row tiles would
                        // not leave room for 32 tokens)
    const float *x;     // token t: x + t * x_stride (16-byte aligned rows)
    uint32_t x_stride;
    float *y;           // token t: y + t * y_stride
    uint32_t y_stride;
    uint32_t pre;
    const float *norm_w;
    float eps;
    uint32_t exact_norm;  // sequential sum of squares (the reference's order)
    uint32_t epi;
    const uint32_t *active;  // [n_tokens] 0 / 1, or null: all active
    uint32_t *status;        // WL_DEV_ERR_NONFINITE / _TIMEOUT
    // argmax epilogue
    unsigned long long *slots;  // [n_tokens], zero on entry, re-zeroed by the last CTA
    uint32_t *counter;          // zero on entry, re-zeroed by the last CTA
    uint32_t *tokens;           // [n_tokens] out: the greedy ids
    uint32_t *ids;              // optional history: ids[*step * n_tokens + t]
    uint32_t *step;             // incremented by the last CTA when ids is set
};

// f32 of the 4 signed bytes of a word: byte ^ 0x80 is q + 128; placed in the
// low byte of 2^23's bit pattern it is 2^23 + q + 128, and subtracting
// 2^23 + 128 leaves q exactly.
__device__ __forceinline__ void q8_word_to_f32(uint32_t word, float *f) {
    const uint32_t u = word ^ 0x80808080u;
#pragma unroll
    for (int e = 0; e < 4; ++e)
        f[e] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u | (uint32_t)e)),
                         8388736.0f);
}

// weight rows (when staged) | RMSNorm weights [K] (when staged) | x [TG][K] |
// block terms [nb][TG][rows] (phases > 1) | totals [TG][rows]
inline size_t q8_batch_smem_bytes(uint32_t K, uint32_t tg, uint32_t rows, uint32_t phases,
                                  bool stage_w = true, bool norm = false) {
    const size_t terms = phases > 1 ? (size_t)(K / 32u) * tg * rows : 0;
    return (stage_w ? (size_t)rows * q8_row_stride(K) + (norm ? (size_t)K * 4u : 0) : 0) +
           ((size_t)tg * K + terms + (size_t)tg * rows) * sizeof(float);
}

template <int TG, bool FMA>
__global__ void __launch_bounds__(QB_THREADS) q8_batch_kernel(const __grid_constant__ Q8BatchParams p) {
    extern __shared__ __align__(16) uint8_t qbs[];
    __shared__ __align__(8) uint64_t s_bar[2];  // weights, activations
    __shared__ uint32_t s_act[TG];
    __shared__ unsigned long long s_best[TG];
    __shared__ uint32_t s_last;
    const uint32_t K = p.K, nb = K / 32u, stride = q8_row_stride(K);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const bool paired = p.epi == QB_EPI_SILU_PAIR;
    const uint32_t tile = blockIdx.x;
    uint32_t j = 0;
    if (!paired)
        while (j + 1u < p.n_jobs && tile >= p.job[j + 1u].tile0) ++j;
    const uint32_t RT = 32u * p.rg;            // rows per job set
    const uint32_t R2 = paired ? 2u * RT : RT;  // rows of the CTA
    const uint32_t groups = R2 / 32u, P = QB_WARPS / groups;
    const uint32_t r0 = (tile - p.job[j].tile0) * RT;
    const uint32_t t0 = blockIdx.y * TG;
    const uint32_t ntok = min((uint32_t)TG, p.n_tokens - t0);
    uint8_t *wsm = qbs;                                                // [R2][stride] weight rows
    const bool stage_nw = p.stage_w && p.pre == QB_PRE_RMSNORM;        // norm weights staged too
    float *nws = reinterpret_cast<float *>(qbs + (p.stage_w ? (size_t)R2 * stride : 0));  // [K]
    float *xs = nws + (stage_nw ? K : 0u);                             // [TG][K]
    float *terms = xs + (size_t)TG * K;                                // [nb][TG][R2] (P > 1)
    float *outs = terms + (P > 1 ? (size_t)nb * TG * R2 : 0);          // [TG][R2]

    // this warp's row (lane) and block phase
    const uint32_t g = warp % groups, ph = warp / groups;
    const uint32_t jj = paired ? g / p.rg : j;
    const uint32_t row = r0 + (g % p.rg) * 32u + lane;
    const bool row_ok = row < p.job[jj].n;
    const uint32_t rl = g * 32u + lane;
    // this lane's row: in shared memory (staged) or in global memory
    const uint8_t *rs = p.stage_w ? wsm + (size_t)rl * stride
                                  : p.job[jj].w + (size_t)(row_ok ? row : 0u) * stride;

    if (tid == 0) {
        mbar_init(&s_bar[0], 1);
        mbar_init(&s_bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    if (tid == 0 && p.stage_w) {  // the weights do not depend on earlier kernels: fetch them now
        const uint32_t sets = paired ? 2u : 1u;
        uint32_t bytes[2];
        uint32_t total = 0;
        for (uint32_t st = 0; st < sets; ++st) {
            const uint32_t jx = paired ? st : j;
            bytes[st] = min(RT, p.job[jx].n - r0) * stride;
            total += bytes[st];
        }
        mbar_arrive_expect_tx(&s_bar[0], total + (stage_nw ? K * 4u : 0u));
        for (uint32_t st = 0; st < sets; ++st) {
            const uint32_t jx = paired ? st : j;
            bulk_g2s(wsm + (size_t)st * RT * stride, p.job[jx].w + (size_t)r0 * stride, bytes[st],
                     &s_bar[0]);
        }
        if (stage_nw) bulk_g2s(nws, p.norm_w, K * 4u, &s_bar[0]);
    }
    pdl_wait();
    if (tid == 0) {  // this group's activation rows
        mbar_arrive_expect_tx(&s_bar[1], ntok * K * 4u);
        if (p.x_stride == K) {
            bulk_g2s(xs, p.x + (size_t)t0 * K, ntok * K * 4u, &s_bar[1]);
        } else {
            for (uint32_t t = 0; t < ntok; ++t)
                bulk_g2s(xs + (size_t)t * K, p.x + (size_t)(t0 + t) * p.x_stride, K * 4u, &s_bar[1]);
        }
    }
    if (tid < (uint32_t)TG) {
        s_act[tid] = (tid < ntok && (!p.active || p.active[t0 + tid])) ? 1u : 0u;
        s_best[tid] = 0ull;
    }
    const bool got_x = mbar_wait(&s_bar[1], 0);
    const bool got_w = !p.stage_w || mbar_wait(&s_bar[0], 0);
    if (!__syncthreads_and(got_x && got_w)) {
        if (tid == 0) atomicOr(p.status, WL_DEV_ERR_TIMEOUT);
        return;
    }
    if (p.pre == QB_PRE_RMSNORM) {
        // rms_norm_f32 (primitives.rs:227-254): one warp per token
        for (uint32_t t = warp; t < ntok; t += QB_WARPS) {
            float *xt = xs + (size_t)t * K;
            float ss = 0.0f;
            if (p.exact_norm) {  // the reference's sequential loop, loads run ahead
                if (lane == 0) ss = seq_sum_sq(xt, K);
                ss = __shfl_sync(0xffffffffu, ss, 0);
            } else {
                for (uint32_t i = lane; i < K; i += 32u) ss = __fadd_rn(ss, __fmul_rn(xt[i], xt[i]));
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
            }
            const float mean = __fdiv_rn(ss, (float)K);
            const float rsq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
            __syncwarp();
            const float *nw = stage_nw ? nws : p.norm_w;
            for (uint32_t i = lane; i < K; i += 32u) xt[i] = __fmul_rn(__fmul_rn(xt[i], rsq), nw[i]);
        }
        __syncthreads();
    }

    float tot[TG];
#pragma unroll
    for (int t = 0; t < TG; ++t) tot[t] = 0.0f;
    for (uint32_t b = ph; b < nb; b += P) {
        uint4 v0 = make_uint4(0u, 0u, 0u, 0u), v1 = v0;
        uint32_t dbits = 0;
        if (row_ok) {
            if (p.stage_w) {
                v0 = lds128(rs + 32u * b);
                v1 = lds128(rs + 32u * b + 16u);
                dbits = reinterpret_cast<const uint16_t *>(rs + K)[b];
            } else {
                v0 = __ldg(reinterpret_cast<const uint4 *>(rs + 32u * b));
                v1 = __ldg(reinterpret_cast<const uint4 *>(rs + 32u * b + 16u));
                dbits = __ldg(reinterpret_cast<const uint16_t *>(rs + K) + b);
            }
        }
        float w[32];
        q8_word_to_f32(v0.x, w + 0);
        q8_word_to_f32(v0.y, w + 4);
        q8_word_to_f32(v0.z, w + 8);
        q8_word_to_f32(v0.w, w + 12);
        q8_word_to_f32(v1.x, w + 16);
        q8_word_to_f32(v1.y, w + 20);
        q8_word_to_f32(v1.z, w + 24);
        q8_word_to_f32(v1.w, w + 28);
        const float d = f16_bits_to_f32(dbits);
#pragma unroll
        for (int t = 0; t < TG; ++t) {
            if (!s_act[t]) continue;  // uniform over the CTA
            const float4 *xb = reinterpret_cast<const float4 *>(xs + (size_t)t * K + 32u * b);
            float s[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 a = xb[2 * q], c = xb[2 * q + 1];
                const float xv[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
                for (int l = 0; l < 8; ++l) {
                    if (FMA)
                        s[l] = q == 0 ? __fmul_rn(w[8 * q + l], xv[l]) : __fmaf_rn(w[8 * q + l], xv[l], s[l]);
                    else
                        s[l] = __fadd_rn(q == 0 ? 0.0f : s[l], __fmul_rn(w[8 * q + l], xv[l]));
                }
            }
            const float hs = __fadd_rn(__fadd_rn(__fadd_rn(s[0], s[4]), __fadd_rn(s[2], s[6])),
                                       __fadd_rn(__fadd_rn(s[1], s[5]), __fadd_rn(s[3], s[7])));
            const float term = __fmul_rn(d, hs);
            if (P == 1)
                tot[t] = __fadd_rn(tot[t], term);
            else
                terms[((size_t)b * TG + t) * R2 + rl] = term;
        }
    }
    if (P == 1) {
#pragma unroll
        for (int t = 0; t < TG; ++t) outs[t * R2 + rl] = tot[t];
    }
    __syncthreads();
    if (P > 1) {
        for (uint32_t i = tid; i < (uint32_t)TG * R2; i += QB_THREADS) {
            const uint32_t r = i % R2, t = i / R2;
            if (!s_act[t]) continue;
            float total = 0.0f;
            for (uint32_t b = 0; b < nb; ++b) total = __fadd_rn(total, terms[((size_t)b * TG + t) * R2 + r]);
            outs[t * R2 + r] = total;
        }
        __syncthreads();
    }

    // epilogues
    if (p.epi == QB_EPI_ARGMAX) {
        for (uint32_t i = tid; i < (uint32_t)TG * R2; i += QB_THREADS) {
            const uint32_t r = i % R2, t = i / R2, rw = r0 + r;  // R2 % 32 == 0: a warp shares t
            unsigned long long key = 0ull;
            if (rw < p.job[0].n && s_act[t])
                key = ((unsigned long long)f32_order_key(outs[t * R2 + r], rw) << 32) |
                      (unsigned long long)(0xFFFFFFFFu - rw);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const unsigned long long o = __shfl_xor_sync(0xffffffffu, key, off);
                key = key > o ? key : o;
            }
            if ((i & 31u) == 0 && key) atomicMax(&s_best[t], key);
        }
        __syncthreads();
        if (tid < ntok && s_best[tid]) atomicMax(&p.slots[t0 + tid], s_best[tid]);
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(p.counter, 1u) == gridDim.x * gridDim.y - 1u ? 1u : 0u;
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        const uint32_t st = p.ids ? *p.step : 0u;
        for (uint32_t t = tid; t < p.n_tokens; t += QB_THREADS) {
            const unsigned long long k = atomicExch(&p.slots[t], 0ull);
            if (p.active && !p.active[t]) continue;
            const uint32_t id = 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
            p.tokens[t] = id;
            if (p.ids) p.ids[(size_t)st * p.n_tokens + t] = id;
        }
        __syncthreads();
        if (tid == 0) {
            if (p.ids) *p.step = st + 1u;
            *p.counter = 0u;
        }
        return;
    }
    const uint32_t rows_out = paired ? RT : R2;
    for (uint32_t i = tid; i < (uint32_t)TG * rows_out; i += QB_THREADS) {
        const uint32_t r = i % rows_out, t = i / rows_out, rw = r0 + r;
        if (!s_act[t] || rw >= p.job[j].n) continue;
        float *yp = p.y + (size_t)(t0 + t) * p.y_stride + p.job[j].y_off + rw;
        const float v = outs[t * R2 + r];
        if (p.epi == QB_EPI_STORE) {
            *yp = v;
        } else if (p.epi == QB_EPI_RESIDUAL) {
            const float h = __fadd_rn(*yp, v);
            *yp = h;
            if (!isfinite(h)) atomicOr(p.status, WL_DEV_ERR_NONFINITE);
        } else {  // silu(gate) * up: gate / (1 + exp(-gate)), then * up
            const float u = outs[t * R2 + RT + r];
            const float sg = __fdiv_rn(v, __fadd_rn(1.0f, exp_f32(-v)));
            *yp = __fmul_rn(sg, u);
        }
    }
}

// ---------------------------------------------------------------------------
// Embedding (embedding_gather, primitives.rs:120-190, Q8_0 arm: w = d * q,
// q8_0.rs:35-47) of every active sequence's token, from the repacked tied
// table; the sequence's position is latched for this step (cur_pos) and
// advanced.  Grid: sequences.
struct EmbedQ8BatchParams {
    const uint8_t *packed;  // repacked Q8_0 rows
    uint32_t K;
    const uint32_t *tokens;  // [n]
    const uint32_t *active;  // [n] or null
    float *hidden;           // [n][K]
    uint32_t *pos, *cur_pos; // [n]
};

__global__ void __launch_bounds__(256) embed_q8_batch_kernel(const __grid_constant__ EmbedQ8BatchParams p) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t z = blockIdx.x;
    if (p.active && !p.active[z]) return;
    const uint8_t *row = p.packed + (size_t)p.tokens[z] * q8_row_stride(p.K);
    for (uint32_t i = threadIdx.x; i < p.K; i += blockDim.x) {
        const uint32_t dbits = reinterpret_cast<const uint16_t *>(row + p.K)[i / 32u];
        p.hidden[(size_t)z * p.K + i] = __fmul_rn(f16_bits_to_f32(dbits), (float)(int8_t)row[i]);
    }
    if (threadIdx.x == 0) {
        const uint32_t pos = p.pos[z];
        p.cur_pos[z] = pos;
        p.pos[z] = pos + 1u;
    }
}

// Final RMSNorm of every sequence's hidden (one CTA each).
struct OutNormBatchParams {
    const float *hidden;
    const float *w;
    float *out;
    uint32_t n;
    float eps;
    uint32_t exact;
};

__global__ void __launch_bounds__(256) out_norm_batch_kernel(const __grid_constant__ OutNormBatchParams p) {
    __shared__ float red[32];
    __shared__ __align__(16) float hs[OUT_NORM_MAX];
    __shared__ __align__(16) uint8_t xscr[exact_sum_scratch_bytes(256)];
    pdl_launch_dependents();
    pdl_wait();
    const float *__restrict__ h = p.hidden + (size_t)blockIdx.x * p.n;
    float *__restrict__ o = p.out + (size_t)blockIdx.x * p.n;
    const float *__restrict__ nw = p.w;
    float sum_sq;
    if (p.exact) {
        sum_sq = block_seq_sum_sq(h, p.n, hs, xscr);
    } else {
        float ss = 0.0f;
        for (uint32_t i = threadIdx.x; i < p.n; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(h[i], h[i]));
        sum_sq = block_sum(ss, red);
    }
    const float mean = __fdiv_rn(sum_sq, (float)p.n);
    const float rsq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
    for (uint32_t i = threadIdx.x; i < p.n; i += blockDim.x) o[i] = __fmul_rn(__fmul_rn(h[i], rsq), nw[i]);
}

}  // namespace wl
