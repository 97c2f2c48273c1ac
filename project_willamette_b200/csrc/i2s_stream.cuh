// i2s_stream.cuh -- many independent I2_S matvecs in one persistent launch.
//
// Same arithmetic as i2s_matvec_kernel (bitlinear_sse2.rs:313-342 semantics,
// bit-exact), organised for sustained HBM streaming:
//  * every op's weight is cut into 32-row blocks; the blocks of all ops form
//    one list, and each CTA (one per SM) owns a contiguous, byte-balanced
//    range of it;
//  * each of the 12 warps of a CTA takes every 12th block of that range (or,
//    in a CTA with few blocks, an equal contiguous run of its boxes, partial
//    row dots combined in shared memory) and
//    streams it as 64-row x 128-byte boxes with 2-D TMA tensor copies
//    (cp.async.bulk.tensor, 128-byte swizzle) through its own 2-stage
//    shared-memory ring (12 x 2 beat 8 x 3 and 6-7 x 4 with the same bytes
//    in flight: the consumer warps, not the copies, set the pace, and a pure
//    TMA stream of these boxes runs at about 7 TB/s) -- lane l owns rows l
//    and l+32 of the box, so there
//    are no cross-lane reductions, and the swizzle makes the 32 lanes' 16-byte
//    reads (one per row) hit distinct banks;
//  * activations (quantised beforehand by quantize_jobs_kernel, one CTA per
//    distinct input) are read with warp-uniform loads that L1 broadcasts, and
//    each load serves two rows: register write-back of the broadcast
//    activations, not DRAM, limited the one-row-per-lane form.
// Rows past an op's end and bytes past a row's end arrive as zeros (TMA
// out-of-bounds fill) and are skipped.
#pragma once

#include <cuda.h>

#include <cstdint>

#include "i2s_matvec.cuh"
#include "tp.cuh"
#include "wl_ptx.cuh"

namespace wl {

constexpr int STREAM_WARPS = 12;
constexpr int STREAM_THREADS = STREAM_WARPS * 32;
constexpr int STREAM_WSTAGES = 2;            // TMA boxes in flight per warp
constexpr int STREAM_RPL = 2;                // rows per lane: activations loaded once per 2 rows
constexpr uint32_t STREAM_BOX_ROWS = 32 * STREAM_RPL;
constexpr uint32_t STREAM_BOX_BYTES = 128;   // 8 weight slots of 16 bytes
constexpr uint32_t STREAM_BOX = STREAM_BOX_ROWS * STREAM_BOX_BYTES;
constexpr uint32_t STREAM_MIN_K = 512;   // a row spans at least one 128-byte box
constexpr uint32_t STREAM_MAX_K = 65536;
constexpr size_t STREAM_SMEM = (size_t)STREAM_WARPS * STREAM_WSTAGES * STREAM_BOX + 1024;

struct I2sStreamOp {
    const int8_t *q;          // quantised input, K bytes
    const float *act_scale;   // its scale
    float *y;
    int32_t *acc;             // may be null
    float w_scale;
    uint32_t K, N;
    uint32_t block_begin;     // first 32-row block of this op in the block list
    uint32_t row_off;         // tensor parallel: first global row of this slice in y
};

struct I2sStreamParams {
    const I2sStreamOp *ops;
    const CUtensorMap *maps;  // one per op, 64-byte aligned, in global memory
    uint32_t n_ops;
    const uint32_t *cta_blocks;  // gridDim.x + 1 block boundaries
    uint32_t *status;
    TpParams tp;                 // world 0: single GPU
};

struct QuantJob {
    const float *x;
    int8_t *q;
    float *scale;
    uint32_t n;
};

// One CTA per distinct input vector; same steps as quantize_absmax_kernel.
// An input of up to QJ_REGS float4 per thread is loaded once, all loads in
// flight together, and quantised from registers (a loop waiting for each
// load in turn, twice, took about 5 us for a 6912-element input).
constexpr int QJ_REGS = 4;
__device__ __forceinline__ uint32_t quant_pack4(float4 v, float inv, bool nz) {
    const float e[4] = {v.x, v.y, v.z, v.w};
    uint32_t packed = 0;
    if (nz) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int qi = quant_round_i8(__fmul_rn(e[k], inv));
            packed |= (uint32_t)(qi & 0xFF) << (8 * k);
        }
    }
    return packed;
}
__device__ __forceinline__ float absmax4(float m, float4 v) {
    return fmaxf(fmaxf(fmaxf(m, fabsf(v.x)), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}
__global__ void __launch_bounds__(QUANT_THREADS)
    quantize_jobs_kernel(const QuantJob *__restrict__ jobs) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float red[QUANT_THREADS / 32];
    const QuantJob j = jobs[blockIdx.x];
    const float4 *x4 = reinterpret_cast<const float4 *>(j.x);
    const uint32_t n4 = j.n / 4u;  // n is a multiple of 512
    const bool in_regs = n4 <= (uint32_t)(QUANT_THREADS * QJ_REGS);
    float4 v[QJ_REGS];
    float m = 0.0f;
    if (in_regs) {
#pragma unroll
        for (int k = 0; k < QJ_REGS; ++k) {
            const uint32_t i = threadIdx.x + (uint32_t)k * QUANT_THREADS;
            v[k] = i < n4 ? x4[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int k = 0; k < QJ_REGS; ++k) m = absmax4(m, v[k]);
    } else {
        for (uint32_t i = threadIdx.x; i < n4; i += QUANT_THREADS) m = absmax4(m, x4[i]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    float max_abs = red[0];
#pragma unroll
    for (int w = 1; w < QUANT_THREADS / 32; ++w) max_abs = fmaxf(max_abs, red[w]);
    const float inv = max_abs == 0.0f ? 0.0f : __fdiv_rn(127.0f, max_abs);
    const bool nz = max_abs != 0.0f;
    uint32_t *q4 = reinterpret_cast<uint32_t *>(j.q);
    if (in_regs) {
#pragma unroll
        for (int k = 0; k < QJ_REGS; ++k) {
            const uint32_t i = threadIdx.x + (uint32_t)k * QUANT_THREADS;
            if (i < n4) q4[i] = quant_pack4(v[k], inv, nz);
        }
    } else {
        for (uint32_t i = threadIdx.x; i < n4; i += QUANT_THREADS) q4[i] = quant_pack4(x4[i], inv, nz);
    }
    if (threadIdx.x == 0) *j.scale = max_abs == 0.0f ? 1.0f : __fdiv_rn(max_abs, 127.0f);
}

// 2-D TMA tile load: box at (x bytes, y rows) of `map` into shared memory.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint32_t x,
                                            uint32_t y, uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// A warp's walk over (block, slice) boxes.  Block mode: blocks bi = first,
// first + STREAM_WARPS, ... below `end`, every slice 0 .. ceil(K/512)-1 of
// each.  Box mode (a CTA with few blocks): the CTA's boxes in order, `left`
// of them from (first, si).
// Each op's first block and box count per row, copied into shared memory at
// kernel start when there are at most STREAM_OPS_SMEM ops (the walk looks
// them up at every block; read from global memory they were a chain of
// dependent loads, 2-6 us before a CTA's first box).
constexpr uint32_t STREAM_OPS_SMEM = 512;
struct OpTab {
    const uint32_t *beg, *S;  // shared memory, or null
    const I2sStreamOp *ops;
    uint32_t n;
    __device__ __forceinline__ uint32_t begin(uint32_t j) const { return beg ? beg[j] : ops[j].block_begin; }
    __device__ __forceinline__ uint32_t boxes(uint32_t j) const { return S ? S[j] : (ops[j].K + 511u) / 512u; }
};

struct BoxWalk {
    uint32_t bi, end, j, si, S, step, left;

    __device__ __forceinline__ bool valid() const { return bi < end && left != 0u; }

    __device__ __forceinline__ void seek_op(const OpTab &t) {
        while (j + 1 < t.n && bi >= t.begin(j + 1)) ++j;
        S = t.boxes(j);
    }

    __device__ __forceinline__ void next(const OpTab &t) {
        --left;
        if (++si < S) return;
        si = 0;
        bi += step;
        if (bi < end) seek_op(t);
    }
};

// Op of block bi (binary search over the ops' first blocks).
__device__ __forceinline__ uint32_t stream_op_of(const OpTab &t, uint32_t bi) {
    uint32_t lo = 0, hi = t.n;
    while (lo + 1 < hi) {
        const uint32_t mid = (lo + hi) / 2;
        if (t.begin(mid) <= bi) lo = mid; else hi = mid;
    }
    return lo;
}

// A CTA with fewer blocks than this splits its boxes evenly over its warps,
// each warp a contiguous range (a block's rows then combine partial dots in
// shared memory); with more, each warp takes every STREAM_WARPS-th block, so
// that the warps stream neighbouring rows.  (A small row slice, e.g. one
// rank's share of a model split 8 ways, is about 11 blocks of 5 or 14 boxes
// per CTA: dealt whole blocks, one warp streamed 14 boxes while others had
// none.  Measured on the BitNet-2B sweep: the whole model, 72 blocks per CTA,
// 108 us in block mode and 123 us with contiguous ranges; a half, 36 per CTA,
// 67.5 and 65.8 us.  Dealing the boxes round robin instead of in contiguous
// ranges measured 114 / 64 / 41 / 29 us at 1 / 1/2 / 1/4 / 1/8 of the model,
// against 108 / 66 / 37 / 27: more op switches per warp.)
constexpr uint32_t STREAM_SPLIT_MAX_BLOCKS = 64;

template <bool C3>
__global__ void __launch_bounds__(STREAM_THREADS, 1)
    i2s_stream_kernel(const __grid_constant__ I2sStreamParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bars[STREAM_WARPS * STREAM_WSTAGES];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~(uintptr_t)1023);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *ring = smem + (size_t)warp * STREAM_WSTAGES * STREAM_BOX;
    uint64_t *bar = bars + warp * STREAM_WSTAGES;
    const uint32_t b0 = p.cta_blocks[blockIdx.x], b1 = p.cta_blocks[blockIdx.x + 1];
    // Box mode: a block shared by several warps adds its rows' partial dots
    // into part[slot] (slot = the first warp whose range reaches into the
    // block) and counts its boxes in cnt[slot]; the warp completing the count
    // finishes the rows.
    __shared__ int32_t part[STREAM_WARPS][STREAM_BOX_ROWS];
    __shared__ uint32_t cnt[STREAM_WARPS];
    __shared__ uint32_t s_beg[STREAM_OPS_SMEM], s_S[STREAM_OPS_SMEM];
    const bool tab_smem = p.n_ops <= STREAM_OPS_SMEM;
    if (tab_smem)
        for (uint32_t i = threadIdx.x; i < p.n_ops; i += STREAM_THREADS) {
            s_beg[i] = p.ops[i].block_begin;
            s_S[i] = (p.ops[i].K + 511u) / 512u;
        }
    const OpTab tab = {tab_smem ? s_beg : nullptr, tab_smem ? s_S : nullptr, p.ops, p.n_ops};
    // Block mode deals blocks dynamically: warp w starts with block b0 + w and
    // then claims the next unclaimed block of the CTA (next_blk) whenever its
    // issue cursor reaches the end of a block, so warps that drew short
    // blocks take more of them.  The claims go through a per-warp ring that
    // the warp's consumer side reads in the same order.  (Claiming the CTA's
    // longest blocks first, to end on short ones, measured slower: 108.7
    // against 105.3 us for the whole BitNet-2B sweep.)
    __shared__ uint32_t next_blk;
    __shared__ uint32_t claim[STREAM_WARPS][4];
    if (threadIdx.x == 0) next_blk = b0 + STREAM_WARPS;
    __syncthreads();  // the op table, next_blk
    const bool split = b1 - b0 < STREAM_SPLIT_MAX_BLOCKS;
    uint32_t T = 0;  // box mode: the CTA's boxes; warp w streams [rw(w), rw(w + 1))
    auto rw = [&](uint32_t w) { return (uint32_t)(((uint64_t)T * w) / STREAM_WARPS); };
    BoxWalk walk = {b0 + warp, b1, 0, 0, 1, STREAM_WARPS, 0xFFFFFFFFu};
    if (split) {
        for (uint32_t i = threadIdx.x; i < STREAM_WARPS * STREAM_BOX_ROWS; i += STREAM_THREADS)
            (&part[0][0])[i] = 0;
        if (threadIdx.x < STREAM_WARPS) cnt[threadIdx.x] = 0u;
        if (b1 > b0) {
            uint32_t j = stream_op_of(tab, b0);
            for (uint32_t bi = b0; bi < b1; ++bi) {
                while (j + 1 < tab.n && bi >= tab.begin(j + 1)) ++j;
                T += tab.boxes(j);
            }
        }
        // this warp's first box: block and slice of box rw(warp)
        walk = {b0, b1, 0, 0, 1, 1u, rw(warp + 1u) - rw(warp)};
        if (walk.valid()) {
            walk.j = stream_op_of(tab, b0);
            walk.seek_op(tab);
            uint32_t g = 0;
            while (g + walk.S <= rw(warp)) {
                g += walk.S;
                ++walk.bi;
                walk.seek_op(tab);
            }
            walk.si = rw(warp) - g;
        }
        __syncthreads();  // part and cnt cleared
    } else if (walk.valid()) {
        walk.j = stream_op_of(tab, walk.bi);
        walk.seek_op(tab);
    }
    // box index (within the CTA) of the current block's first box, box mode
    uint32_t gblk = split && walk.valid() ? rw(warp) - walk.si : 0u;
    uint32_t bstart = walk.si;  // first slice of the current block this warp streams
    BoxWalk ahead = walk;  // the issue cursor runs STREAM_WSTAGES boxes ahead
    const uint64_t policy = l2_policy_evict_first();
    if (lane == 0) {
        for (int s = 0; s < STREAM_WSTAGES; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    uint32_t issued = 0, claims = 0, taken = 0;
    auto issue = [&](uint32_t stage) {
        const I2sStreamOp &op = p.ops[ahead.j];
        mbar_arrive_expect_tx(&bar[stage], STREAM_BOX);
        tma_load_2d(ring + stage * STREAM_BOX, p.maps + ahead.j, ahead.si * STREAM_BOX_BYTES,
                    (ahead.bi - op.block_begin) * STREAM_BOX_ROWS, &bar[stage], policy);
        if (!split && ahead.si + 1 == ahead.S) {  // claim the next block
            uint32_t nb = atomicAdd(&next_blk, 1u);
            nb = nb < b1 ? nb : b1;
            claim[warp][claims++ & 3u] = nb;
            ahead.si = 0;
            ahead.bi = nb;
            if (nb < b1) ahead.seek_op(tab);
        } else {
            ahead.next(tab);
        }
        ++issued;
    };
    if (lane == 0)
        for (int s = 0; s < STREAM_WSTAGES && ahead.valid(); ++s) issue(s);
    __syncwarp();
    pdl_launch_dependents();
    pdl_wait();  // quantised inputs come from the previous kernel

    uint32_t cur = 0xFFFFFFFFu, P = 0;
    int32_t asum = 0;
    float combined = 0.0f;
    I2sAcc acc[STREAM_RPL];
    int32_t corr[STREAM_RPL];
#pragma unroll
    for (int r = 0; r < STREAM_RPL; ++r) {
        acc[r] = {0, 0, 0, 0};
        corr[r] = 0;
    }
    bool timeout = false;
    for (uint32_t k = 0; walk.valid(); ++k) {
        const uint32_t st = k % STREAM_WSTAGES;
        if (!__all_sync(0xffffffffu, mbar_wait(&bar[st], (k / STREAM_WSTAGES) & 1u))) {
            timeout = true;
            // Give the boxes still in flight a bounded chance to land before
            // this warp's shared memory is released.
            if (lane == 0)
                for (uint32_t kk = k + 1; kk < issued; ++kk)
                    (void)mbar_wait(&bar[kk % STREAM_WSTAGES], (kk / STREAM_WSTAGES) & 1u);
            break;
        }
        const I2sStreamOp &op = p.ops[walk.j];
        if (walk.j != cur) {  // op switch: sum of this op's activations
            cur = walk.j;
            P = op.K >> 6;
            // 8 loads in flight per lane (a plain loop waited for each in turn:
            // 14 round trips, about 6 us, for a 6912-element input).  The loop
            // also brings the activations into L1 for this op's boxes: the
            // sum formed by the quantiser instead, with the lines prefetched
            // (prefetch.global.L1) and not waited for, measured slower (113
            // against 108 us for the whole model, 28.7 against 26.7 for 1/8).
            int32_t s = 0;
            for (uint32_t i0 = lane * 16; i0 < op.K; i0 += 8 * 32 * 16) {
                uint4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const uint32_t i = i0 + (uint32_t)u * 32u * 16u;
                    v[u] = i < op.K ? __ldg(reinterpret_cast<const uint4 *>(op.q + i)) : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) s += sum_bytes(v[u]);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            asum = s;
            combined = __fmul_rn(op.w_scale, __ldg(op.act_scale));
        }
        const uint8_t *box = ring + st * STREAM_BOX;
        uint32_t c3[STREAM_RPL];
#pragma unroll
        for (int r = 0; r < STREAM_RPL; ++r) c3[r] = 0;
#pragma unroll
        for (uint32_t s = 0; s < 8; ++s) {
            const uint32_t pp = walk.si * 8 + s;
            if (pp < P) {
                const int8_t *qa = op.q + (pp >> 1) * 128u + (pp & 1u) * 16u;
                uint4 a[4];
#pragma unroll
                for (int o = 0; o < 4; ++o) a[o] = __ldg(reinterpret_cast<const uint4 *>(qa + 32 * o));
#pragma unroll
                for (int r = 0; r < STREAM_RPL; ++r) {
                    // row lane + 32r sits in 128-byte line lane + 32r; its swizzle
                    // phase is (lane + 32r) & 7 = lane & 7
                    const uint4 wv = *reinterpret_cast<const uint4 *>(
                        box + (lane + 32u * r) * STREAM_BOX_BYTES + ((s ^ (lane & 7u)) << 4));
                    i2s_slot<C3>(wv, a, acc[r], c3[r]);
                }
            }
        }
        if constexpr (C3) {
#pragma unroll
            for (int r = 0; r < STREAM_RPL; ++r) {
                if ((c3[r] & 0x55555555u) != 0u) {  // this row has code 0b11 in this box
                    const uint8_t *line = box + (lane + 32u * r) * STREAM_BOX_BYTES;
                    for (uint32_t s = 0; s < 8; ++s) {
                        const uint32_t pp = walk.si * 8 + s;
                        if (pp >= P) break;
                        const uint4 wv =
                            *reinterpret_cast<const uint4 *>(line + ((s ^ (lane & 7u)) << 4));
                        uint4 a[4];
                        i2s_load_act<false>(op.q, pp, 0u, a);
                        int32_t c = corr[r];
                        c = i2s_word_c3(wv.x, a[0].x, a[1].x, a[2].x, a[3].x, c);
                        c = i2s_word_c3(wv.y, a[0].y, a[1].y, a[2].y, a[3].y, c);
                        c = i2s_word_c3(wv.z, a[0].z, a[1].z, a[2].z, a[3].z, c);
                        c = i2s_word_c3(wv.w, a[0].w, a[1].w, a[2].w, a[3].w, c);
                        corr[r] = c;
                    }
                }
            }
        }
        __syncwarp();  // every lane is done with this stage
        if (lane == 0 && ahead.valid()) issue(st);
        const bool block_end = walk.si + 1 == walk.S;
        if (block_end || walk.left == 1u) {  // this warp's last box of the block
            bool finish = true;
            int32_t part_dot[STREAM_RPL];
#pragma unroll
            for (int r = 0; r < STREAM_RPL; ++r) part_dot[r] = i2s_acc_total(acc[r]) - 2 * corr[r];
            if (split && !(bstart == 0u && block_end)) {
                // shared block: add the partial dots, count this warp's boxes
                uint32_t slot = 0;
#pragma unroll
                for (uint32_t w = 1; w < (uint32_t)STREAM_WARPS; ++w)
                    if (rw(w) <= gblk) slot = w;
#pragma unroll
                for (int r = 0; r < STREAM_RPL; ++r) atomicAdd(&part[slot][lane + 32u * r], part_dot[r]);
                __syncwarp();
                uint32_t done = 0;
                if (lane == 0) {
                    __threadfence_block();
                    const uint32_t mine = walk.si + 1u - bstart;
                    done = atomicAdd(&cnt[slot], mine) + mine == walk.S ? 1u : 0u;
                    __threadfence_block();
                }
                finish = __shfl_sync(0xffffffffu, done, 0) != 0u;
                if (finish) {
#pragma unroll
                    for (int r = 0; r < STREAM_RPL; ++r) part_dot[r] = atomicAdd(&part[slot][lane + 32u * r], 0);
                }
            }
            if (finish) {
#pragma unroll
                for (int r = 0; r < STREAM_RPL; ++r) {
                    const uint32_t row = (walk.bi - op.block_begin) * STREAM_BOX_ROWS + lane + 32u * r;
                    if (row < op.N) {
                        const int32_t dot = part_dot[r] - asum;
                        const float yv = __fmul_rn(combined, __int2float_rn(dot));
                        if (p.tp.world) tp_store_all(p.tp, op.y + op.row_off + row, yv);
                        else op.y[op.row_off + row] = yv;
                        if (op.acc) op.acc[op.row_off + row] = dot;
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < STREAM_RPL; ++r) {
                acc[r] = {0, 0, 0, 0};
                corr[r] = 0;
            }
        }
        if (block_end) {
            gblk += walk.S;
            bstart = 0;
        }
        if (!split && walk.si + 1 == walk.S) {  // the block the issue cursor claimed
            walk.si = 0;
            walk.bi = reinterpret_cast<volatile uint32_t *>(claim[warp])[taken++ & 3u];
            if (walk.bi < walk.end) walk.seek_op(tab);
        } else {
            walk.next(tab);
        }
    }
    if (timeout && lane == 0) atomicOr(p.status, WL_DEV_ERR_TIMEOUT);
    if (p.tp.world) {  // count this CTA in every rank once all its stores are out
        __syncthreads();
        if (threadIdx.x == 0) tp_arrive(p.tp);
    }
}

}  // namespace wl
