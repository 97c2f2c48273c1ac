// i2s_gemm.cuh -- I2_S BitLinear prefill GEMM on the 5th-generation tensor
// cores (tcgen05.mma kind::i8, accumulators in tensor memory).
//
// Reference: the reference prefills one token at a time
// (src/model/generate.rs:241-250, src/model/multi_forward.rs:106-110), i.e.
// per-token absmax int8 quantisation (bitlinear_sse2.rs:285-304) and an
// exact int32 ternary dot per (token, row) (bitlinear_sse2.rs:313-342).  The
// int32 sums are exact in any order, so one tensor-core GEMM gives the same
// bits:
//
//   Y[m, n] = (w_scale * act_scale[m]) * (float)(sum_k q[m,k] * t[n,k]),
//   t = code - 1  (codes 0b00/0b01/0b10 -> -1/0/+1; weights holding code 0b11
//                  take the exact matvec path instead)
//   sum_k q*t = sum_k q[m,k]*code[n,k] - rowsum(q[m,:]).
//
// So the tensor core multiplies signed int8 activations (A, M x K) by the
// UNSIGNED 2-bit codes (B, N x K): in the natural element order a 16-byte
// chunk of a 128-element k-block of B is (packed >> shift) & 0x03 over 16
// consecutive packed bytes -- two ALU ops per four weights to expand the
// packed weights into the MMA's operand layout, no lookup tables.
//
// Tile: 128 tokens (tensor-memory lanes) x BN weight rows (columns) per CTA,
// K in 128-byte blocks (one 128-byte swizzle atom).  A (quantised
// activations) and the packed weights arrive by 2-D TMA through a 4-stage
// ring; the 4 warps expand the packed weights into a double-buffered
// K-major, 128-byte-swizzled code tile; thread 0 issues 4 MMAs (K = 32 each)
// per k-block and commits them to the stage's mbarrier.  Epilogue: the 4
// warps read their 32 tensor-memory lanes with tcgen05.ld, subtract the
// token's activation row sum and apply the two scales.
#pragma once

#include <cuda.h>

#include <cstdint>

#include "wl_ptx.cuh"

namespace wl {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 128;  // int8 elements (bytes) of K per k-block
constexpr int GEMM_STAGES = 4;
constexpr int GEMM_THREADS = 128;

template <int BN>
struct GemmSmem {
    static constexpr uint32_t A_BYTES = GEMM_BM * GEMM_BK;  // 16 KB
    static constexpr uint32_t BP_BYTES = BN * (GEMM_BK / 4);
    static constexpr uint32_t B_BYTES = BN * GEMM_BK;
    static constexpr uint32_t A_OFF = 0;
    static constexpr uint32_t BP_OFF = A_OFF + GEMM_STAGES * A_BYTES;
    static constexpr uint32_t B_OFF = BP_OFF + GEMM_STAGES * BP_BYTES;
    static constexpr uint32_t TOTAL = B_OFF + 2 * B_BYTES;
    static constexpr size_t DYN = TOTAL + 1024;  // + alignment slack
};

struct I2sGemmParams {
    CUtensorMap a_map;   // int8 activations [M][K], box {128 B, 128 rows}, 128B swizzle
    CUtensorMap bp_map;  // packed weights [N][K/4], box {32 B, BN rows}, no swizzle
    const float *act_scale;  // [M]
    const int32_t *rowsum;   // [M]
    float w_scale;
    uint32_t M, N, K;
    float *y;      // [M][N]
    int32_t *acc;  // [M][N] or null
    uint32_t *status;
};

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
    return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) |
           ((uint64_t)(1024u >> 4) << 32) | ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor: D s32, A s8, B u8, both K-major, M = 128, N = BN.
template <int BN>
__device__ __forceinline__ uint32_t umma_idesc_i8() {
    return (2u << 4) | (1u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) |
           ((uint32_t)(GEMM_BM >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d_plain(void *dst, const CUtensorMap *map, uint32_t x,
                                                  uint32_t y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                     "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int BN>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    i2s_gemm_kernel(const __grid_constant__ I2sGemmParams p) {
    using L = GemmSmem<BN>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full[GEMM_STAGES];
    __shared__ __align__(8) uint64_t mma_done[GEMM_STAGES];
    __shared__ uint32_t tmem_base_s;
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~(uintptr_t)1023);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t n0 = blockIdx.x * BN, m0 = blockIdx.y * GEMM_BM;
    const uint32_t nkb = p.K / GEMM_BK;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&tmem_base_s)),
                     "r"((uint32_t)BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        for (int s = 0; s < GEMM_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&mma_done[s], 1);
        }
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    pdl_launch_dependents();
    pdl_wait();  // the quantised activations come from the previous kernel

    uint32_t issued = 0;  // k-blocks whose TMA thread 0 has issued
    auto issue = [&](uint32_t kb) {
        const uint32_t s = kb % GEMM_STAGES;
        ++issued;
        mbar_arrive_expect_tx(&full[s], L::A_BYTES + L::BP_BYTES);
        tma_load_2d_plain(smem + L::A_OFF + s * L::A_BYTES, &p.a_map, kb * GEMM_BK, m0, &full[s]);
        tma_load_2d_plain(smem + L::BP_OFF + s * L::BP_BYTES, &p.bp_map, kb * (GEMM_BK / 4), n0,
                          &full[s]);
    };
    if (tid == 0)
        for (uint32_t kb = 0; kb < min(nkb, (uint32_t)GEMM_STAGES); ++kb) issue(kb);

    const uint32_t idesc = umma_idesc_i8<BN>();
    bool ok = true;
    (void)ok;
    uint32_t committed = 0;  // MMA groups committed by thread 0
    for (uint32_t kb = 0; kb < nkb; ++kb) {
        const uint32_t s = kb % GEMM_STAGES;
        bool w = mbar_wait(&full[s], (kb / GEMM_STAGES) & 1u);
        if (kb >= 2)  // code buffer kb&1 was last read by the MMAs of kb-2
            w = w && mbar_wait(&mma_done[(kb - 2) % GEMM_STAGES], ((kb - 2) / GEMM_STAGES) & 1u);
        if (!__syncthreads_and(w)) {
            ok = false;
            break;
        }
        // Stage (kb+2) % 4 == (kb-2) % 4 held k-block kb-2: its MMAs are done
        // (awaited above) and its packed weights were expanded at kb-2, so it
        // takes k-block kb+2 now -- the TMA stays two k-blocks ahead.
        if (tid == 0 && kb >= 2 && kb + 2 < nkb) issue(kb + 2);
        // Expand packed weights of stage s into code tile kb&1 (K-major,
        // 128-byte swizzle: row n, 16-byte chunk c at c ^ (n & 7)).
        const uint8_t *bp = smem + L::BP_OFF + s * L::BP_BYTES;
        uint8_t *codes = smem + L::B_OFF + (kb & 1u) * L::B_BYTES;
        for (uint32_t item = tid; item < (uint32_t)BN * 2u; item += GEMM_THREADS) {
            const uint32_t n = item >> 1, h = item & 1u;
            const uint4 v = *reinterpret_cast<const uint4 *>(bp + n * 32u + h * 16u);
            uint8_t *row = codes + (n >> 3) * 1024u + (n & 7u) * 128u;
#pragma unroll
            for (uint32_t jj = 0; jj < 4; ++jj) {
                const uint32_t sh = 6u - 2u * jj;
                const uint32_t c = h + 2u * jj;  // elements 16c .. 16c+15 of the k-block
                uint4 o;
                o.x = (v.x >> sh) & 0x03030303u;
                o.y = (v.y >> sh) & 0x03030303u;
                o.z = (v.z >> sh) & 0x03030303u;
                o.w = (v.w >> sh) & 0x03030303u;
                *reinterpret_cast<uint4 *>(row + ((c ^ (n & 7u)) << 4)) = o;
            }
        }
        // Make the generic-proxy stores visible to the tensor core.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t a_addr = smem_u32(smem + L::A_OFF + s * L::A_BYTES);
            const uint32_t b_addr = smem_u32(codes);
#pragma unroll
            for (uint32_t j = 0; j < GEMM_BK / 32; ++j)
                umma_i8(tmem, umma_desc_sw128(a_addr + 32u * j), umma_desc_sw128(b_addr + 32u * j),
                        idesc, (kb | j) != 0u ? 1u : 0u);
            umma_commit(&mma_done[s]);
            ++committed;
        }
    }
    // Wait for the last MMAs (bounded), then read the accumulators.
    if (ok && nkb > 0) {
        const uint32_t last = nkb - 1;
        ok = mbar_wait(&mma_done[last % GEMM_STAGES], (last / GEMM_STAGES) & 1u);
    }
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (ok) {
        const uint32_t m = m0 + warp * 32u + lane;
        const bool mvalid = m < p.M;
        const float combined = mvalid ? __fmul_rn(p.w_scale, p.act_scale[m]) : 0.0f;
        const int32_t rs = mvalid ? p.rowsum[m] : 0;
#pragma unroll 1
        for (uint32_t c0 = 0; c0 < (uint32_t)BN; c0 += 32) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem + ((warp * 32u) << 16) + c0, r);
            if (mvalid) {
                float *yrow = p.y + (size_t)m * p.N;
                int32_t *arow = p.acc ? p.acc + (size_t)m * p.N : nullptr;
#pragma unroll
                for (uint32_t i = 0; i < 32; ++i) {
                    const uint32_t n = n0 + c0 + i;
                    if (n < p.N) {
                        const int32_t dot = (int32_t)r[i] - rs;
                        yrow[n] = __fmul_rn(combined, __int2float_rn(dot));
                        if (arow) arow[n] = dot;
                    }
                }
            }
        }
    } else if (tid == 0) {
        atomicOr(p.status, WL_DEV_ERR_TIMEOUT);
        // Let committed MMAs and issued copies drain (bounded) before tensor
        // and shared memory are released.
        for (uint32_t k = committed > GEMM_STAGES ? committed - GEMM_STAGES : 0; k < committed; ++k)
            (void)mbar_wait(&mma_done[k % GEMM_STAGES], (k / GEMM_STAGES) & 1u);
        for (uint32_t k = issued > GEMM_STAGES ? issued - GEMM_STAGES : 0; k < issued; ++k)
            (void)mbar_wait(&full[k % GEMM_STAGES], (k / GEMM_STAGES) & 1u);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"((uint32_t)BN));
    }
}

}  // namespace wl
