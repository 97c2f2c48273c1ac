// i2s_gemm_ws.cuh -- prefill GEMM on tcgen05 tensor cores, warp-specialised
// and persistent, over weights expanded once to int8 ternary values.
//
// Reference arithmetic as in i2s_gemm.cuh: per token m, absmax int8
// activations q[m, :] (bitlinear_sse2.rs:285-304) and the exact int32 dot
// with the ternary weights t = code - 1 (code 0b11 -> 0, bitlinear.rs:43-50):
//   Y[m, n] = (w_scale * act_scale[m]) * (float)(sum_k q[m, k] * t[n, k]).
// With t expanded to signed bytes (i2s_expand_kernel) the tensor core does
// the whole dot: tcgen05.mma kind::i8, A = q (s8, M x K), B = t (s8, N x K),
// D = s32 in tensor memory.  Code 0b11 is handled by the expansion, so no
// weight needs a separate path.
//
// Roles (one CTA per SM, persistent over output tiles of 128 x BN):
//   warp 0     TMA producer: A and B k-blocks (128 bytes of K) into a
//              STAGES-deep ring, 128-byte swizzle, mbarrier complete_tx;
//   warp 1     allocates 2 x BN tensor-memory columns (two accumulators) and
//              issues the MMAs (one elected thread): 4 x K=32 per k-block,
//              tcgen05.commit frees the stage / publishes the accumulator;
//   warps 2-5  epilogue: tcgen05.ld of their 32 lanes, scale, store; the
//              next tile's MMAs run into the other accumulator meanwhile.
// Every wait is bounded (2 s); a timeout sets the status word, raises a
// shared abort flag that ends every role's loop, and the MMA thread drains
// its committed MMAs before tensor memory is released.
#pragma once

#include <cuda.h>

#include <cstdint>

#include "i2s_gemm.cuh"
#include "wl_ptx.cuh"

namespace wl {

constexpr int WS_STAGES = 4;
constexpr int WS_THREADS = 192;

template <int BN>
struct WsSmem {
    static constexpr uint32_t A_BYTES = GEMM_BM * GEMM_BK;  // 16 KB
    static constexpr uint32_t B_BYTES = BN * GEMM_BK;
    static constexpr uint32_t STAGE = A_BYTES + B_BYTES;
    static constexpr uint32_t OUT = 4u * 32u * 32u * 4u;  // one 32 x 32 f32 box per epilogue warp
    static constexpr uint32_t TOTAL = WS_STAGES * STAGE + OUT;
    static constexpr size_t DYN = TOTAL + 1024;  // + alignment slack
};

struct I2sGemmWsParams {
    CUtensorMap a_map;  // int8 activations [M][K], box {128 B, 128 rows}, 128B swizzle
    CUtensorMap b_map;  // int8 ternary weights [N][K], box {128 B, BN rows}, 128B swizzle
    CUtensorMap y_map;  // f32 output [M][N], box {32, 32}, 128B swizzle (when use_tma_store)
    uint32_t use_tma_store;
    const float *act_scale;  // [M]
    float w_scale;
    uint32_t M, N, K;
    float *y;      // [M][N]
    int32_t *acc;  // [M][N] or null
    uint32_t *status;
};

// D s32, A s8, B s8, both K-major, M = 128, N = BN.
template <int BN>
__device__ __forceinline__ uint32_t umma_idesc_s8s8() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
           ((uint32_t)(GEMM_BM >> 4) << 24);
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, uint32_t x,
                                             uint32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
        "r"(smem_u32(src)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until the bulk stores of all but the newest N groups have read their
// shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int BN>
__global__ void __launch_bounds__(WS_THREADS, 1)
    i2s_gemm_ws_kernel(const __grid_constant__ I2sGemmWsParams p) {
    using L = WsSmem<BN>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full[WS_STAGES], empty[WS_STAGES];
    __shared__ __align__(8) uint64_t tfull[2], tempty[2];
    __shared__ uint32_t tmem_base_s, s_abort;
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~(uintptr_t)1023);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t MT = (p.M + GEMM_BM - 1) / GEMM_BM, NT = (p.N + BN - 1) / BN;
    const uint32_t tiles = MT * NT, nkb = p.K / GEMM_BK;

    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&tmem_base_s)),
                     "r"((uint32_t)(2 * BN)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        for (int s = 0; s < WS_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);  // one arrival per epilogue warp
        }
        s_abort = 0;
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    pdl_launch_dependents();
    // Only A (the quantised activations) and act_scale come from the previous
    // kernel: the producer requests the first stages' weights before waiting
    // for it, the epilogue waits before reading act_scale.

    auto abort_now = [&]() {
        atomicOr(p.status, WL_DEV_ERR_TIMEOUT);
        atomicExch(&s_abort, 1u);
    };
    auto aborted = [&]() { return *(volatile uint32_t *)&s_abort != 0u; };

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            uint32_t it = 0;
            // weights of the first stages before the dependency wait
            const uint32_t pre = blockIdx.x < tiles ? min(nkb, (uint32_t)WS_STAGES) : 0u;
            {
                const uint32_t n0 = (blockIdx.x / MT) * BN;
                for (uint32_t kb = 0; kb < pre; ++kb) {
                    uint8_t *st = smem + kb * L::STAGE;
                    mbar_arrive_expect_tx(&full[kb], L::STAGE);
                    tma_load_2d_plain(st + L::A_BYTES, &p.b_map, kb * GEMM_BK, n0, &full[kb]);
                }
            }
            pdl_wait();
            for (uint32_t t = blockIdx.x; t < tiles && !aborted(); t += gridDim.x) {
                const uint32_t m0 = (t % MT) * GEMM_BM, n0 = (t / MT) * BN;
                for (uint32_t kb = 0; kb < nkb; ++kb, ++it) {
                    const uint32_t s = it % WS_STAGES;
                    uint8_t *st = smem + s * L::STAGE;
                    if (it < pre) {  // weights already requested
                        tma_load_2d_plain(st, &p.a_map, kb * GEMM_BK, m0, &full[s]);
                        continue;
                    }
                    if (it >= WS_STAGES && !mbar_wait(&empty[s], ((it / WS_STAGES) - 1u) & 1u)) {
                        abort_now();
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], L::STAGE);
                    tma_load_2d_plain(st, &p.a_map, kb * GEMM_BK, m0, &full[s]);
                    tma_load_2d_plain(st + L::A_BYTES, &p.b_map, kb * GEMM_BK, n0, &full[s]);
                }
            }
            // drain (bounded): the last stages' copies land before smem is released
            for (uint32_t k = it > WS_STAGES ? it - WS_STAGES : 0; k < it; ++k)
                (void)mbar_wait(&full[k % WS_STAGES], (k / WS_STAGES) & 1u);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            const uint32_t idesc = umma_idesc_s8s8<BN>();
            uint32_t it = 0, local = 0;
            uint32_t committed_tiles = 0;
            for (uint32_t t = blockIdx.x; t < tiles && !aborted(); t += gridDim.x, ++local) {
                const uint32_t a = local & 1u;
                // the epilogue has drained this accumulator (tile local - 2)
                if (local >= 2 && !mbar_wait(&tempty[a], ((local / 2) - 1u) & 1u)) {
                    abort_now();
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + a * (uint32_t)BN;
                bool ok = true;
                for (uint32_t kb = 0; kb < nkb; ++kb, ++it) {
                    const uint32_t s = it % WS_STAGES;
                    if (!mbar_wait(&full[s], (it / WS_STAGES) & 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + s * L::STAGE);
                    const uint32_t b_addr = a_addr + L::A_BYTES;
#pragma unroll
                    for (uint32_t j = 0; j < GEMM_BK / 32; ++j)
                        umma_i8(d, umma_desc_sw128(a_addr + 32u * j),
                                umma_desc_sw128(b_addr + 32u * j), idesc, (kb | j) != 0u ? 1u : 0u);
                    umma_commit(&empty[s]);  // the stage is free once these MMAs are done
                }
                if (!ok) {
                    abort_now();
                    break;
                }
                umma_commit(&tfull[a]);  // accumulator a holds tile t
                ++committed_tiles;
            }
            // drain (bounded): every committed MMA completes before dealloc
            for (uint32_t k = it > WS_STAGES ? it - WS_STAGES : 0; k < it; ++k)
                (void)mbar_wait(&empty[k % WS_STAGES], (k / WS_STAGES) & 1u);
            (void)committed_tiles;
        }
    } else {
        // epilogue warps 2..5: TMEM lanes 32*(warp % 4) .. +31
        pdl_wait();  // act_scale comes from the previous kernel
        const uint32_t lb = 32u * (warp & 3u);
        uint32_t local = 0;
        for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
            const uint32_t a = local & 1u;
            const bool ok = mbar_wait(&tfull[a], (local / 2) & 1u);
            if (!__all_sync(0xffffffffu, ok)) {
                if (lane == 0) abort_now();
                break;
            }
            tc_fence_after();
            const uint32_t m0 = (t % MT) * GEMM_BM, n0 = (t / MT) * BN;
            const uint32_t m = m0 + lb + lane;
            const bool mvalid = m < p.M;
            const float combined = mvalid ? __fmul_rn(p.w_scale, p.act_scale[m]) : 0.0f;
            float *yrow = p.y + (size_t)m * p.N;
            // this warp's 32 x 32 f32 staging box (128-byte swizzle: row r's
            // 16-byte chunk c at c ^ (r & 7))
            uint8_t *box = smem + WS_STAGES * L::STAGE + (warp & 3u) * 4096u;
#pragma unroll 1
            for (uint32_t c0 = 0; c0 < (uint32_t)BN; c0 += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem + (lb << 16) + a * (uint32_t)BN + c0, r);
                if (p.use_tma_store) {
                    if (m0 + lb < p.M && n0 + c0 < p.N) {
                        if (lane == 0) bulk_wait_group_read<0>();  // the box is free again
                        __syncwarp();
#pragma unroll
                        for (uint32_t c = 0; c < 8; ++c) {
                            float4 v;
                            v.x = __fmul_rn(combined, __int2float_rn((int32_t)r[4 * c]));
                            v.y = __fmul_rn(combined, __int2float_rn((int32_t)r[4 * c + 1]));
                            v.z = __fmul_rn(combined, __int2float_rn((int32_t)r[4 * c + 2]));
                            v.w = __fmul_rn(combined, __int2float_rn((int32_t)r[4 * c + 3]));
                            *reinterpret_cast<float4 *>(box + lane * 128u + ((c ^ (lane & 7u)) << 4)) = v;
                        }
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&p.y_map, box, n0 + c0, m0 + lb);
                            bulk_commit_group();
                        }
                    }
                    if (p.acc && mvalid) {
                        int32_t *arow = p.acc + (size_t)m * p.N;
#pragma unroll
                        for (uint32_t i = 0; i < 32; ++i)
                            if (n0 + c0 + i < p.N) arow[n0 + c0 + i] = (int32_t)r[i];
                    }
                    continue;
                }
                if (mvalid) {
                    const uint32_t nb = n0 + c0;
                    if (nb + 32u <= p.N && (p.N & 3u) == 0u) {
#pragma unroll
                        for (uint32_t i = 0; i < 32; i += 4) {
                            float4 v;
                            v.x = __fmul_rn(combined, __int2float_rn((int32_t)r[i]));
                            v.y = __fmul_rn(combined, __int2float_rn((int32_t)r[i + 1]));
                            v.z = __fmul_rn(combined, __int2float_rn((int32_t)r[i + 2]));
                            v.w = __fmul_rn(combined, __int2float_rn((int32_t)r[i + 3]));
                            *reinterpret_cast<float4 *>(yrow + nb + i) = v;
                        }
                    } else {
#pragma unroll
                        for (uint32_t i = 0; i < 32; ++i)
                            if (nb + i < p.N)
                                yrow[nb + i] = __fmul_rn(combined, __int2float_rn((int32_t)r[i]));
                    }
                    if (p.acc) {
                        int32_t *arow = p.acc + (size_t)m * p.N;
#pragma unroll
                        for (uint32_t i = 0; i < 32; ++i)
                            if (nb + i < p.N) arow[nb + i] = (int32_t)r[i];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[a]);  // accumulator a may be overwritten
        }
        if (lane == 0) bulk_wait_group_read<0>();  // stores have read the staging boxes
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"((uint32_t)(2 * BN)));
    }
}

// Packed I2_S rows -> int8 ternary rows in natural element order
// (t = code - 1, code 0b11 -> 0; bitlinear.rs:43-50, tensor.rs:86-105): one
// thread per 32-byte block (128 elements).
__global__ void i2s_expand_kernel(const uint8_t *__restrict__ packed, size_t n_blocks,
                                  int8_t *__restrict__ out) {
    for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < n_blocks;
         b += (size_t)gridDim.x * blockDim.x) {
        const uint4 lo = *reinterpret_cast<const uint4 *>(packed + b * 32u);
        const uint4 hi = *reinterpret_cast<const uint4 *>(packed + b * 32u + 16u);
        const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        int8_t *dst = out + b * 128u;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {  // element group 32*jj .. 32*jj+31 <- bits 7-2jj, 6-2jj
            const uint32_t sh = 6u - 2u * (uint32_t)jj;
            uint32_t o[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t c = (w[k] >> sh) & 0x03030303u;
                // t = c - 1 per byte, and 0 where c == 3: c3 = c & (c >> 1)
                const uint32_t c3 = c & (c >> 1) & 0x01010101u;
                const uint32_t v = (c | 0x80808080u) - 0x01010101u;  // c - 1 per byte (no borrow)
                const uint32_t t = (v ^ 0x80808080u) & ~(c3 * 0xFFu);
                o[k] = t;
            }
            *reinterpret_cast<uint4 *>(dst + 32 * jj) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4 *>(dst + 32 * jj + 16) = make_uint4(o[4], o[5], o[6], o[7]);
        }
    }
}

}  // namespace wl
