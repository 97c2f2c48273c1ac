// tp.cuh -- tensor-parallel exchange over NVLink peer memory.
//
// North star (multi-GPU): BitLinear output rows are split across the GPUs of
// one box and all-gathered; the lm-head is split by vocab rows and reduced
// with a (max, index) reduction.  Here the exchange is fused into the
// computing kernels instead of a separate collective:
//  * every rank maps every peer's symmetric block (CUDA IPC), so a kernel can
//    store straight into a peer's memory over NVLink;
//  * a matvec CTA writes each output row it computes to the same offset of
//    every rank's block (its own included) and releases them at system
//    scope; the grid's last CTA then adds 1 to its rank's arrival counter in
//    every rank's block (a system-scope release);
//  * a kernel that consumes a gathered vector first waits (bounded, on its
//    own memory) until every rank's counter has caught up with this rank's
//    own -- every rank has then finished every exchange op this rank has
//    finished, and all their stores are visible.  The target is read on the
//    device (this rank's own counter, complete because the previous kernel on
//    the stream has finished), so launches can be captured in a CUDA graph
//    and replayed without host bookkeeping.
// No TMA copy of any kind touches peer memory; peers are reached with plain
// stores and atomics only.
#pragma once

#include <cstdint>

#include "wl_ptx.cuh"

namespace wl {

constexpr int TP_MAX_WORLD = 8;
// Symmetric block header: [0, 32) arrival counters (one per source rank),
// [256, 260) this rank's CTA-done counter, [260, 264) its lm-head call
// counter, [1024, 9216) argmax key slots.
constexpr uint32_t TP_HEADER_BYTES = 16384;
constexpr uint32_t TP_DONE_OFF = 256;
constexpr uint32_t TP_LMCALL_OFF = 260;
constexpr uint32_t WL_DEV_ERR_PEER_TIMEOUT = 2u;

struct TpParams {
    int world;                          // 0: no exchange
    int rank;
    uint8_t *local_base;                // this rank's symmetric block
    uint8_t *peer_base[TP_MAX_WORLD];   // every rank's block as mapped here
    uint32_t wait;                      // wait for every rank before reading inputs
};

// The symmetric block starts with one arrival counter per source rank.
__device__ __forceinline__ uint32_t *tp_counter(uint8_t *base, int src) {
    return reinterpret_cast<uint32_t *>(base) + src;
}

// Translate a pointer into this rank's block to the same offset in rank r's.
template <typename T>
__device__ __forceinline__ T *tp_peer_ptr(const TpParams &tp, T *local, int r) {
    return reinterpret_cast<T *>(tp.peer_base[r] +
                                 (reinterpret_cast<uint8_t *>(local) - tp.local_base));
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_sys_add(uint32_t *p, uint32_t v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Store one f32 output to every rank (own block included).
__device__ __forceinline__ void tp_store_all(const TpParams &tp, float *local, float v) {
    for (int r = 0; r < tp.world; ++r) *tp_peer_ptr(tp, local, r) = v;
}

// Release / acquire fences (no sequentially consistent fence is needed for
// these message-passing patterns; `fence.sc.sys` measured about 3.7 us per
// CTA after its peer stores and again in the last CTA).
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// One arrival of this rank in every rank's block: a release at system scope
// by a thread that follows (CTA barrier) the stores it publishes, so the
// fence is cumulative over the CTA's stores.
__device__ __forceinline__ void tp_signal(const TpParams &tp) {
    fence_acq_rel_sys();
    for (int r = 0; r < tp.world; ++r) red_release_sys_add(tp_counter(tp.peer_base[r], tp.rank), 1u);
}

// Called by thread 0 of every CTA after a CTA barrier that follows all of the
// CTA's peer stores.  Each CTA releases its stores at system scope and counts
// itself; the last CTA of the grid acquires the other CTAs' counts (and with
// them everything they released), re-arms the counter and signals one
// arrival to every rank with a system-scope release -- one arrival per
// kernel, whatever its grid size.
__device__ __forceinline__ void tp_arrive(const TpParams &tp) {
    fence_acq_rel_sys();
    uint32_t *done = reinterpret_cast<uint32_t *>(tp.local_base + TP_DONE_OFF);
    const uint32_t ctas = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(done, 1u) == ctas - 1u) {
        fence_acq_rel_gpu();
        atomicExch(done, 0u);
        for (int r = 0; r < tp.world; ++r)
            red_release_sys_add(tp_counter(tp.peer_base[r], tp.rank), 1u);
    }
}

// Called by one thread once the previous kernel on the stream has finished:
// wait (bounded) until every rank's counter in this rank's block has reached
// this rank's own.  Returns false on timeout.
__device__ __forceinline__ bool tp_wait(const TpParams &tp) {
    const uint32_t target = ld_acquire_sys(tp_counter(tp.local_base, tp.rank));
    const uint64_t t0 = globaltimer_ns(), limit = wait_limit_ns();
    for (int s = 0; s < tp.world; ++s) {
        const uint32_t *c = tp_counter(tp.local_base, s);
        while ((int32_t)(ld_acquire_sys(c) - target) < 0) {
            if (globaltimer_ns() - t0 > limit) return false;
        }
    }
    return true;
}

// Stand-alone wait (one thread): used between steps and before a consumer
// that is not itself a library kernel.
__global__ void tp_wait_kernel(const TpParams tp, uint32_t *status) {
    if (threadIdx.x == 0 && !tp_wait(tp)) atomicOr(status, WL_DEV_ERR_PEER_TIMEOUT);
}

// Wait (one thread, bounded) until the word another agent writes -- a peer
// GPU, the host through mapped memory, or an earlier kernel on another
// stream -- reaches `target` (wrap-around compare); on timeout set
// WL_DEV_ERR_TIMEOUT and return, so later work on the stream still runs.
__global__ void wait_flag_kernel(const uint32_t *flag, uint32_t target, uint32_t *status) {
    if (threadIdx.x != 0) return;
    const uint64_t t0 = globaltimer_ns(), limit = wait_limit_ns();
    while ((int32_t)(ld_acquire_sys(flag) - target) < 0) {
        if (globaltimer_ns() - t0 > limit) {
            atomicOr(status, WL_DEV_ERR_TIMEOUT);
            return;
        }
    }
}

}  // namespace wl
