// willamette_b200.cu -- the C ABI (include/willamette_b200.h) and its host
// logic: validation that mirrors the reference's error behaviour, the device
// cache of host weights, staging buffers, and kernel launches.
//
// Built as one translation unit with the kernel headers so the whole library
// is a single sm_100a object (see project_willamette_b200/build.py).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/willamette_b200.h"
#include "argmax.cuh"
#include "bitnet_decode.cuh"
#include "bitnet_mega.cuh"
#include "i2s_f32act.cuh"
#include "i2s_matvec.cuh"
#include "i2s_stream.cuh"
#include "i2s_gemm.cuh"
#include "i2s_gemm_ws.cuh"
#include "q6k_lmhead.cuh"
#include "q8_0.cuh"
#include "q8_batch.cuh"
#include "attn_batch.cuh"
#include "gguf.h"

namespace {

using namespace wl;

// ------------------------------------------------------------------ errors
thread_local std::string g_last_error;
thread_local uint32_t g_last_type = 0;

int fail(int status, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

int fail_type(uint32_t raw) {
    g_last_type = raw;
    return fail(WL_ERR_UNSUPPORTED_TENSOR_TYPE, "Unsupported GGML tensor type: %u", raw);
}

#define WL_CUDA(call)                                                                   \
    do {                                                                                \
        cudaError_t e_ = (call);                                                        \
        if (e_ != cudaSuccess)                                                          \
            return fail(WL_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));   \
    } while (0)

const char *tname(const wl_tensor_view *t) { return t && t->name ? t->name : "<unnamed>"; }

// ------------------------------------------------------------------ state
struct DevBuf {
    void *p = nullptr;
    size_t cap = 0;
};

struct CachedWeight {
    void *dptr = nullptr;
    size_t bytes = 0;
    bool bad_scale = false;  // Q8_0: some block scale is not finite
    bool has_code3 = true;   // I2_S: some 2-bit code is 0b11 (scanned on upload)
    int8_t *ternary = nullptr;  // I2_S: int8 ternary copy for prefill, made on first use
};

using CacheKey = std::tuple<const void *, size_t, uint32_t, uint64_t, uint64_t>;

struct Ctx {
    std::mutex mu;
    bool inited = false;
    int device = 0;
    int sm_count = 0;
    cudaStream_t stream = nullptr;
    uint32_t *d_status = nullptr;
    uint32_t *h_status = nullptr;  // pinned
    void *pinned = nullptr;
    size_t pinned_cap = 0;
    DevBuf x, y, q, scale, acc, ids, scratch, rowsum;
    // plain host-buffer matvec calls: [device status word, 16 B][y], so one
    // copy returns both (zeroed on allocation; reset after a reported error)
    DevBuf ys;
    std::map<CacheKey, CachedWeight> cache;
};

Ctx &ctx() {
    static Ctx c;
    return c;
}

constexpr int WL_MAX_DYN_SMEM = 227 * 1024 - 1024;
// From this many tokens on, prefill runs as one tensor-core GEMM.
constexpr size_t I2S_GEMM_MIN_TOKENS = 16;

int launch_i2s_gemm(const uint8_t *packed, float w_scale, uint32_t K, uint32_t N, uint32_t M,
                    const int8_t *q, const float *act_scale, const int32_t *rowsum, float *y,
                    int32_t *acc, cudaStream_t s, bool pdl, uint32_t *status);

int launch_i2s_gemm_s8(const int8_t *t, float w_scale, uint32_t K, uint32_t N, uint32_t M,
                       const int8_t *q, const float *act_scale, float *y, int32_t *acc,
                       cudaStream_t s, bool pdl, uint32_t *status);
int launch_i2s_expand(const uint8_t *packed, uint32_t K, uint32_t N, int8_t *out, cudaStream_t s);

using I2sKernel = void (*)(I2sMatvecParams);
using I2sStreamKernel = void (*)(I2sStreamParams);

// The exact-mode decode kernels: the input transform's sum of squares with
// the reference's sequential bits, indexed [shape][c3] (fused input only).
const I2sKernel kI2sExact[2][2] = {
    {i2s_matvec_kernel<8, 5, true, false, true>, i2s_matvec_kernel<8, 5, true, true, true>},
    {i2s_matvec_kernel<32, 4, true, false, true>, i2s_matvec_kernel<32, 4, true, true, true>},
};

// Every I2_S per-op kernel variant, indexed [shape][fuse_q][c3]:
// shape 0 = 8 lanes/row x 5 slots (in_dim <= 2560), 1 = 32 x 4 (<= 8192),
// 2 = 32 lanes, activations re-read from L1 (larger; never fused).
const I2sKernel kI2s[3][2][2] = {
    {{i2s_matvec_kernel<8, 5, false, false>, i2s_matvec_kernel<8, 5, false, true>},
     {i2s_matvec_kernel<8, 5, true, false>, i2s_matvec_kernel<8, 5, true, true>}},
    {{i2s_matvec_kernel<32, 4, false, false>, i2s_matvec_kernel<32, 4, false, true>},
     {i2s_matvec_kernel<32, 4, true, false>, i2s_matvec_kernel<32, 4, true, true>}},
    {{i2s_matvec_kernel<32, 0, false, false>, i2s_matvec_kernel<32, 0, false, true>},
     {i2s_matvec_kernel<32, 0, false, false>, i2s_matvec_kernel<32, 0, false, true>}},
};
const I2sStreamKernel kStream[2] = {i2s_stream_kernel<false>, i2s_stream_kernel<true>};

// Dynamic shared memory a kernel can get: the per-block limit (227 KB on
// sm_100) minus its static shared memory, at most `want`.
size_t kernel_dyn_cap(const void *k, size_t want = (size_t)WL_MAX_DYN_SMEM) {
    cudaFuncAttributes a;
    if (cudaFuncGetAttributes(&a, k) != cudaSuccess) return 0;
    const size_t limit = (size_t)227 * 1024;
    const size_t cap = a.sharedSizeBytes < limit ? limit - a.sharedSizeBytes : 0;
    return std::min(want, cap);
}

// Raise the dynamic shared-memory limit of every kernel once, at init, so
// launches never call cudaFuncSetAttribute (they can be captured in graphs).
int configure_kernels() {
    for (auto &a : kI2s)
        for (auto &b : a)
            for (I2sKernel k : b)
                WL_CUDA(cudaFuncSetAttribute((const void *)k,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             WL_MAX_DYN_SMEM / 2));
    for (auto &a : kI2sExact)
        for (I2sKernel k : a)
            WL_CUDA(cudaFuncSetAttribute((const void *)k,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         WL_MAX_DYN_SMEM / 2));
    const void *others[] = {(const void *)i2s_gemm_kernel<64>, (const void *)i2s_gemm_kernel<128>,
                            (const void *)i2s_gemm_kernel<256>,
                            (const void *)kStream[0], (const void *)kStream[1],
                            (const void *)q6k_lmhead_kernel<1>, (const void *)q6k_lmhead_kernel<2>,
                            (const void *)q6k_lmhead_kernel<4>, (const void *)q6k_lmhead_kernel<8>,
                            (const void *)q8_0_matvec_kernel, (const void *)attn_decode_kernel<false>,
                            (const void *)attn_decode_kernel<true>,
                            (const void *)attn_exact_kernel, (const void *)rms_norm_kernel,
                            (const void *)softmax_kernel,
                            (const void *)bitnet_mega_kernel<false>,
                            (const void *)bitnet_mega_kernel<true>,
                            (const void *)i2s_gemm_ws_kernel<64>,
                            (const void *)i2s_gemm_ws_kernel<128>,
                            (const void *)i2s_gemm_ws_kernel<256>,
                            (const void *)q8_batch_kernel<1, false>,
                            (const void *)q8_batch_kernel<4, false>,
                            (const void *)q8_batch_kernel<8, false>,
                            (const void *)q8_batch_kernel<32, false>,
                            (const void *)q8_batch_kernel<1, true>,
                            (const void *)q8_batch_kernel<4, true>,
                            (const void *)q8_batch_kernel<8, true>,
                            (const void *)q8_batch_kernel<32, true>,
                            (const void *)attn_gqa_batch_kernel<64, 1>,
                            (const void *)attn_gqa_batch_kernel<64, 2>,
                            (const void *)attn_gqa_batch_kernel<64, 3>,
                            (const void *)attn_gqa_batch_kernel<64, 4>,
                            (const void *)attn_gqa_batch_kernel<128, 1>,
                            (const void *)attn_gqa_batch_kernel<128, 2>,
                            (const void *)attn_gqa_batch_kernel<128, 3>,
                            (const void *)attn_gqa_batch_kernel<128, 4>};
    for (const void *k : others)
        WL_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kernel_dyn_cap(k)));
    return WL_OK;
}

int init_locked(Ctx &c, int device) {
    if (c.inited) return WL_OK;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
        return fail(WL_ERR_NO_DEVICE, "no CUDA device visible");
    if (device < 0 || device >= n) return fail(WL_ERR_NO_DEVICE, "device %d out of range", device);
    cudaDeviceProp prop;
    WL_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(WL_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a",
                    device, prop.major, prop.minor);
    WL_CUDA(cudaSetDevice(device));
    c.device = device;
    c.sm_count = prop.multiProcessorCount;
    WL_CUDA(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
    WL_CUDA(cudaMalloc(&c.d_status, 64));
    WL_CUDA(cudaMemsetAsync(c.d_status, 0, 64, c.stream));
    WL_CUDA(cudaStreamSynchronize(c.stream));
    WL_CUDA(cudaMallocHost(&c.h_status, 64));
    int rc = configure_kernels();
    if (rc) return rc;
    c.inited = true;
    return WL_OK;
}

int ensure_init(Ctx &c) {
    if (c.inited) {
        cudaSetDevice(c.device);
        return WL_OK;
    }
    return init_locked(c, 0);
}

int grow(DevBuf &b, size_t bytes) {
    if (b.cap >= bytes) return WL_OK;
    if (b.p) cudaFree(b.p);
    b.p = nullptr;
    b.cap = 0;
    size_t cap = bytes < 4096 ? 4096 : bytes;
    WL_CUDA(cudaMalloc(&b.p, cap));
    // Zero on the library stream so the kernels that follow on it see zeros
    // (scratch words such as the argmax slots must start at zero).
    WL_CUDA(cudaMemsetAsync(b.p, 0, cap, ctx().stream));
    b.cap = cap;
    return WL_OK;
}

int grow_pinned(Ctx &c, size_t bytes) {
    if (c.pinned_cap >= bytes) return WL_OK;
    if (c.pinned) cudaFreeHost(c.pinned);
    c.pinned = nullptr;
    c.pinned_cap = 0;
    size_t cap = bytes < (1u << 20) ? (1u << 20) : bytes;
    WL_CUDA(cudaMallocHost(&c.pinned, cap));
    c.pinned_cap = cap;
    return WL_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------------------------ launches
template <typename Kern, typename... Args>
cudaError_t launch(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                   Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

int sm_count_for_launch() {
    Ctx &c = ctx();
    if (c.inited) return c.sm_count;
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        n = 148;
    return n;
}

uint32_t *status_ptr() {
    Ctx &c = ctx();
    if (!c.inited) {
        std::lock_guard<std::mutex> g(c.mu);
        if (init_locked(c, 0) != WL_OK) return nullptr;
    }
    return c.d_status;
}

int i2s_shape_index(uint32_t K, int *lpr) {
    const uint32_t P = K / 64u;
    if (P <= 40) {
        *lpr = 8;
        return 0;
    }
    *lpr = 32;
    return P <= 128 ? 1 : 2;
}

int launch_quantize(const float *x, uint32_t n, uint32_t m, int8_t *q, float *scale,
                    cudaStream_t s, bool pdl, int32_t *rowsum = nullptr) {
    if (m == 0 || n == 0) return WL_OK;
    WL_CUDA(launch(quantize_absmax_kernel, dim3(m), dim3(QUANT_THREADS), 0, s, pdl, x, n, q,
                   scale, rowsum));
    return WL_OK;
}

// One launch of the per-op I2_S kernel over up to four weights that share an
// input: either pre-quantised (q, act_scale) or f32 (x, quantised in-kernel,
// optional copies of q / scale to q_out / scale_out).
struct I2sLaunch {
    const wl_i2s_dev_weight *w = nullptr;
    uint32_t nw = 0, K = 0;
    const int8_t *q = nullptr;
    const float *act_scale = nullptr;
    const float *x = nullptr;
    int8_t *q_out = nullptr;
    float *scale_out = nullptr;
    const TpParams *tp = nullptr;      // tensor-parallel exchange, or null
    const uint32_t *row_offs = nullptr;  // per weight (tensor parallel)
    // decode-step fusions (fused-input kernels only)
    uint32_t pre = I2S_PRE_NONE;
    const float *norm_w = nullptr, *x2 = nullptr;
    float eps = 0.0f;
    uint32_t residual = 0, finite_flag = 0, exact_norm = 0;
};

bool weights_may_have_code3(const wl_i2s_dev_weight *w, uint32_t nw) {
    for (uint32_t j = 0; j < nw; ++j)
        if (!(w[j].flags & WL_I2S_NO_CODE3)) return true;
    return false;
}

int launch_i2s_with_status(const I2sLaunch &L, cudaStream_t s, bool pdl, uint32_t *status) {
    I2sMatvecParams p = {};
    uint32_t rows = 0;
    for (uint32_t j = 0; j < L.nw; ++j) {
        p.jobs[j].w = L.w[j].packed;
        p.jobs[j].w_scale = L.w[j].w_scale;
        p.jobs[j].out_dim = L.w[j].out_dim;
        p.jobs[j].row_begin = rows;
        p.jobs[j].y = L.w[j].y;
        p.jobs[j].acc = L.w[j].acc;
        p.jobs[j].row_off = L.row_offs ? L.row_offs[j] : 0u;
        rows += L.w[j].out_dim;
    }
    if (rows == 0 && !L.tp) return WL_OK;
    const uint32_t K = L.K;
    p.njobs = (int)L.nw;
    p.K = K;
    p.total_rows = rows;
    p.q = L.q;
    p.act_scale = L.act_scale;
    p.x = L.x;
    p.q_out = L.q_out;
    p.scale_out = L.scale_out;
    p.status = status;
    if (L.tp) p.tp = *L.tp;
    p.pre = L.pre;
    p.norm_w = L.norm_w;
    p.x2 = L.x2;
    p.eps = L.eps;
    p.residual = L.residual;
    p.finite_flag = L.finite_flag;
    p.exact_norm = L.exact_norm;
    const bool fuse = L.x != nullptr;
    int lpr = 32;
    const int shape = i2s_shape_index(K, &lpr);
    if (fuse && (shape == 2 || K > I2S_FUSE_Q_MAX_K))
        return fail(WL_ERR_INVALID_ARGUMENT, "fused quantisation needs in_dim <= %u",
                    I2S_FUSE_Q_MAX_K);
    const int c3 = weights_may_have_code3(L.w, L.nw) ? 1 : 0;
    I2sKernel k = (fuse && L.pre != I2S_PRE_NONE && L.exact_norm) ? kI2sExact[shape][c3]
                                                                  : kI2s[shape][fuse ? 1 : 0][c3];
    const uint32_t rpi = (uint32_t)I2S_WARPS * (32u / (uint32_t)lpr);
    // (a tensor-parallel rank with an empty slice still launches one CTA,
    // which only signals its arrival)
    const uint32_t G = std::max<uint32_t>(1u, std::min<uint32_t>((uint32_t)sm_count_for_launch(), rows));
    p.rows_per_cta = std::max<uint32_t>(1u, (rows + G - 1) / G);
    const uint32_t stage_bytes = rpi * (K / 4u);
    const uint32_t nchunks = (p.rows_per_cta + rpi - 1) / rpi;
    uint32_t nst = std::max<uint32_t>(1u, I2S_STAGE_BUDGET / stage_bytes);
    nst = std::min<uint32_t>(nst, (uint32_t)I2S_MAX_STAGES);
    nst = std::min<uint32_t>(nst, nchunks);
    p.nstages = nst;
    size_t smem = (size_t)nst * stage_bytes + (fuse ? (size_t)K * 5u + I2S_QS_PAD : 0u);
    if (fuse && L.pre == I2S_PRE_RELU2_RMSNORM && !L.exact_norm &&
        smem + (size_t)K * 4u <= (size_t)WL_MAX_DYN_SMEM / 2) {
        p.stage_up = 1;
        smem += (size_t)K * 4u;
    }
    if (fuse && L.pre != I2S_PRE_NONE && L.exact_norm)  // staged RMSNorm weights (exact mode)
        smem += (size_t)K * 4u;
    if (fuse && L.residual && smem + (size_t)p.rows_per_cta * 4u <= (size_t)WL_MAX_DYN_SMEM / 2) {
        p.stage_res = 1;
        smem += ((size_t)p.rows_per_cta * 4u + 15u) & ~(size_t)15u;
    }
    if (smem > (size_t)WL_MAX_DYN_SMEM / 2)
        return fail(WL_ERR_INVALID_ARGUMENT, "in_dim %u too large for one shared-memory stage", K);
    // Decode-engine matvecs (fused input transform): ask for the kernel's
    // whole shared-memory allowance so that two of this op's CTAs never share
    // an SM (the block scheduler otherwise doubled some up while other SMs
    // were left to the attention CTAs; token 1145 -> 1136 us at BitNet-2B).
    if (fuse && L.pre != I2S_PRE_NONE) smem = (size_t)WL_MAX_DYN_SMEM / 2;
    const uint32_t grid = std::max<uint32_t>(1u, (rows + p.rows_per_cta - 1) / p.rows_per_cta);
    WL_CUDA(launch(k, dim3(grid), dim3(I2S_THREADS), smem, s, pdl, p));
    return WL_OK;
}

int launch_i2s(const I2sLaunch &L, cudaStream_t s, bool pdl) {
    uint32_t *status = status_ptr();
    if (!status) return WL_ERR_NO_DEVICE;
    return launch_i2s_with_status(L, s, pdl, status);
}

int q6k_launch_cfg(uint32_t n_embd, int bg, uint32_t *nst, size_t *smem) {
    const uint32_t stride = q6k_row_stride(n_embd / 256u);
    const size_t chunk = (size_t)Q6K_ROWS_PER_CHUNK * stride;
    const size_t xs = (size_t)bg * (n_embd + n_embd / 8u) * sizeof(float);
    const size_t cap = (size_t)WL_MAX_DYN_SMEM;
    for (uint32_t n = Q6K_STAGES; n >= 2; --n) {
        if (n * chunk + xs <= cap) {
            *nst = n;
            *smem = n * chunk + xs;
            return WL_OK;
        }
    }
    return fail(WL_ERR_INVALID_ARGUMENT, "embedding_length %u too large for the Q6_K lm-head",
                n_embd);
}

// One launch for all `batch` hidden rows: groups of BG rows (the largest of
// 8, 4, 2, 1 that the batch fills and whose hidden rows plus two weight
// stages fit in shared memory) x vocab ranges, about one CTA per SM.
int launch_q6k_all(const uint8_t *packed, uint32_t n_embd, uint32_t vocab, uint32_t row_offset,
                   const float *hidden, uint32_t batch, float *logits, uint32_t *ids,
                   void *scratch, cudaStream_t s, bool pdl, const TpParams *tp) {
    uint32_t *status = status_ptr();
    if (!status) return WL_ERR_NO_DEVICE;
    int bg = batch >= 8 ? 8 : batch >= 4 ? 4 : batch >= 2 ? 2 : 1;
    uint32_t nst = 0;
    size_t smem = 0;
    while (q6k_launch_cfg(n_embd, bg, &nst, &smem) != WL_OK) {
        if (bg == 1) return WL_ERR_INVALID_ARGUMENT;  // message set by q6k_launch_cfg
        bg /= 2;
    }
    const uint32_t groups = (batch + (uint32_t)bg - 1) / (uint32_t)bg;
    const uint32_t v = std::max(vocab, 1u);
    const uint32_t sms = (uint32_t)sm_count_for_launch();
    const uint32_t ranges = std::min<uint32_t>(v, std::max<uint32_t>(1u, sms / groups));
    Q6kParams p = {};
    p.packed = packed;
    p.n_embd = n_embd;
    p.vocab = vocab;
    p.nb = n_embd / 256u;
    p.row_stride = q6k_row_stride(p.nb);
    p.rows_per_cta = (v + ranges - 1) / ranges;
    p.n_ranges = (v + p.rows_per_cta - 1) / p.rows_per_cta;
    p.batch = batch;
    p.nstages = nst;
    p.l2_keep = groups > 1 ? 1u : 0u;
    p.hidden = hidden;
    p.logits = logits;
    p.ids = ids;
    p.slots = reinterpret_cast<unsigned long long *>(scratch);
    p.counter = reinterpret_cast<uint32_t *>(p.slots + batch);
    p.status = status;
    p.row_offset = row_offset;
    if (tp) p.tp = *tp;
    const dim3 grid(p.n_ranges * groups);
    switch (bg) {
        case 8: WL_CUDA(launch(q6k_lmhead_kernel<8>, grid, dim3(Q6K_THREADS), smem, s, pdl, p)); break;
        case 4: WL_CUDA(launch(q6k_lmhead_kernel<4>, grid, dim3(Q6K_THREADS), smem, s, pdl, p)); break;
        case 2: WL_CUDA(launch(q6k_lmhead_kernel<2>, grid, dim3(Q6K_THREADS), smem, s, pdl, p)); break;
        default: WL_CUDA(launch(q6k_lmhead_kernel<1>, grid, dim3(Q6K_THREADS), smem, s, pdl, p)); break;
    }
    return WL_OK;
}

int launch_q6k(const uint8_t *packed, uint32_t n_embd, uint32_t vocab, const float *hidden,
               uint32_t batch, float *logits, uint32_t *ids, void *scratch, cudaStream_t s,
               bool pdl) {
    if (batch == 0 || vocab == 0) return WL_OK;
    return launch_q6k_all(packed, n_embd, vocab, 0, hidden, batch, logits, ids, scratch, s, pdl,
                          nullptr);
}

int launch_q8(const uint8_t *packed, uint32_t K, uint32_t N, const float *x, float *y,
              cudaStream_t s, bool pdl) {
    if (N == 0) return WL_OK;
    const uint32_t nb = K / 32u;
    const uint32_t R = nb >= (uint32_t)Q8_THREADS ? 1u : (uint32_t)Q8_THREADS / nb;
    const size_t smem = ((size_t)K + K / 8u + (size_t)R * nb) * sizeof(float);
    if (smem > (size_t)WL_MAX_DYN_SMEM)
        return fail(WL_ERR_INVALID_ARGUMENT, "in_dim %u too large for the Q8_0 kernel", K);
    const uint32_t tiles = (N + R - 1) / R;
    const uint32_t grid = std::min<uint32_t>(tiles, (uint32_t)sm_count_for_launch() * 4u);
    WL_CUDA(launch(q8_0_matvec_kernel, dim3(grid), dim3(Q8_THREADS), smem, s, pdl, packed, K, N, x,
                   y));
    return WL_OK;
}

// ------------------------------------------------------------------ validation
// bitlinear_sse2.rs:129-177 + tensor.rs:278-309 (the x86 dispatch target).
int validate_i2s(const wl_tensor_view *w, size_t input_len, size_t output_len, bool check_io,
                 uint32_t *in_dim, uint32_t *out_dim, float *scale) {
    if (!w) return fail(WL_ERR_INVALID_ARGUMENT, "weight is NULL");
    if (w->ggml_type != WL_GGML_I2_S) return fail_type(w->ggml_type);
    if (w->n_dims != 2 || !w->shape)
        return fail(WL_ERR_GGUF_PARSE, "bitlinear_i2s_matvec_f32: weight \"%s\" is not 2-D",
                    tname(w));
    const uint64_t K = w->shape[0], N = w->shape[1];
    if (check_io && input_len != K)
        return fail(WL_ERR_GGUF_PARSE, "bitlinear_i2s_matvec_f32: input.len()=%zu != in_dim=%llu",
                    input_len, (unsigned long long)K);
    if (check_io && output_len != N)
        return fail(WL_ERR_GGUF_PARSE,
                    "bitlinear_i2s_matvec_f32: output.len()=%zu != out_dim=%llu", output_len,
                    (unsigned long long)N);
    if (K == 0 || K % WL_I2S_ELEMENTS_PER_BLOCK != 0)
        return fail(WL_ERR_GGUF_PARSE,
                    "bitlinear_i2s_matvec_f32: in_dim %llu is not a positive multiple of 128",
                    (unsigned long long)K);
    if (K > WL_I2S_MAX_IN_DIM)
        return fail(WL_ERR_INVALID_ARGUMENT, "in_dim %llu exceeds WL_I2S_MAX_IN_DIM (%u)",
                    (unsigned long long)K, WL_I2S_MAX_IN_DIM);
    if (N > 0xFFFFFFFFull / 2)
        return fail(WL_ERR_INVALID_ARGUMENT, "out_dim %llu too large", (unsigned long long)N);
    const uint64_t expected = K / 4 * N;
    if (!w->data && expected > 0) return fail(WL_ERR_INVALID_ARGUMENT, "weight data is NULL");
    if (w->data_len < expected)
        return fail(WL_ERR_GGUF_PARSE,
                    "bitlinear_i2s_matvec_f32: weight data.len()=%zu < %llu (in_dim/4 x out_dim)",
                    w->data_len, (unsigned long long)expected);
    if (!w->scale_data)
        return fail(WL_ERR_GGUF_PARSE, "i2s_scale: tensor \"%s\" has no scale_data set", tname(w));
    if (w->scale_len < 4)
        return fail(WL_ERR_GGUF_PARSE,
                    "i2s_scale: scale_data for \"%s\" too short (%zu bytes, need >= 4)", tname(w),
                    w->scale_len);
    float s;
    memcpy(&s, w->scale_data, 4);
    if (!std::isfinite(s))
        return fail(WL_ERR_GGUF_PARSE, "i2s_scale: non-finite scale (%g) for tensor \"%s\"", s,
                    tname(w));
    *in_dim = (uint32_t)K;
    *out_dim = (uint32_t)N;
    *scale = s;
    return WL_OK;
}

// Row byte length for the quantized lm-head / linear arms
// (tensor.rs q6k_expected_byte_len / q8_0_expected_byte_len).
int row_bytes_for(uint32_t type, uint64_t row_elems, uint64_t *row_bytes) {
    if (type == WL_GGML_Q6_K) {
        if (row_elems % WL_Q6K_ELEMENTS_PER_BLOCK)
            return fail(WL_ERR_GGUF_PARSE, "Q6_K row length %llu is not a multiple of QK_K=256",
                        (unsigned long long)row_elems);
        *row_bytes = row_elems / WL_Q6K_ELEMENTS_PER_BLOCK * WL_Q6K_BYTES_PER_BLOCK;
        return WL_OK;
    }
    if (type == WL_GGML_Q8_0) {
        if (row_elems % WL_Q8_0_ELEMENTS_PER_BLOCK)
            return fail(WL_ERR_GGUF_PARSE, "Q8_0 row length %llu is not a multiple of QK8_0=32",
                        (unsigned long long)row_elems);
        *row_bytes = row_elems / WL_Q8_0_ELEMENTS_PER_BLOCK * WL_Q8_0_BYTES_PER_BLOCK;
        return WL_OK;
    }
    return fail_type(type);
}

float h2f(uint16_t h) {
    const uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0x1F) bits = (sign << 31) | (0xFFu << 23) | (man << 13);
    else if (exp == 0) return (sign ? -1.0f : 1.0f) * (float)man * (1.0f / 16777216.0f);
    else bits = (sign << 31) | ((exp + 112u) << 23) | (man << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// ------------------------------------------------------------------ weight cache
int get_weight(Ctx &c, const wl_tensor_view *w, uint64_t in_dim, uint64_t out_dim,
               size_t used_bytes, CachedWeight **out) {
    CacheKey key{w->data, w->data_len, w->ggml_type, in_dim, out_dim};
    auto it = c.cache.find(key);
    if (it != c.cache.end()) {
        *out = &it->second;
        return WL_OK;
    }
    CachedWeight cw;
    if (w->ggml_type == WL_GGML_I2_S) {
        cw.bytes = used_bytes;
        WL_CUDA(cudaMalloc(&cw.dptr, std::max<size_t>(cw.bytes, 16)));
        // Upload on the library stream: the kernels run on that non-blocking
        // stream, which does not order with the legacy default stream.
        if (cw.bytes)
            WL_CUDA(cudaMemcpyAsync(cw.dptr, w->data, cw.bytes, cudaMemcpyHostToDevice,
                                    c.stream));
        // One-time scan for code 0b11, so calls on code-3-free weights (all
        // weights the reference's quantiser writes) take the fast path.
        uint32_t *found = c.d_status + 8;
        WL_CUDA(cudaMemsetAsync(found, 0, 4, c.stream));
        if (cw.bytes >= 16) {
            const size_t n16 = cw.bytes / 16;
            const uint32_t grid = (uint32_t)std::min<size_t>((n16 + 255) / 256, 2048);
            i2s_scan_code3_kernel<<<grid, 256, 0, c.stream>>>((const uint4 *)cw.dptr, n16, found);
            WL_CUDA(cudaGetLastError());
        }
        uint32_t h_found = 0;
        WL_CUDA(cudaMemcpyAsync(c.h_status + 8, found, 4, cudaMemcpyDeviceToHost, c.stream));
        WL_CUDA(cudaStreamSynchronize(c.stream));
        h_found = c.h_status[8];
        cw.has_code3 = h_found != 0;
    } else if (w->ggml_type == WL_GGML_Q6_K || w->ggml_type == WL_GGML_Q8_0) {
        const bool q6 = w->ggml_type == WL_GGML_Q6_K;
        cw.bytes = q6 ? wl_q6k_packed_bytes((uint32_t)in_dim, (uint32_t)out_dim)
                      : wl_q8_0_packed_bytes((uint32_t)in_dim, (uint32_t)out_dim);
        if (!q6) {
            const size_t nblk = used_bytes / WL_Q8_0_BYTES_PER_BLOCK;
            for (size_t b = 0; b < nblk; ++b) {
                uint16_t h;
                memcpy(&h, w->data + b * WL_Q8_0_BYTES_PER_BLOCK, 2);
                if (!std::isfinite(h2f(h))) {
                    cw.bad_scale = true;
                    break;
                }
            }
        }
        void *raw = nullptr;
        WL_CUDA(cudaMalloc(&cw.dptr, std::max<size_t>(cw.bytes, 16)));
        if (used_bytes) {
            WL_CUDA(cudaMalloc(&raw, used_bytes));
            WL_CUDA(cudaMemcpyAsync(raw, w->data, used_bytes, cudaMemcpyHostToDevice, c.stream));
            int rc = q6 ? wl_dev_q6k_repack((const uint8_t *)raw, (uint32_t)in_dim,
                                            (uint32_t)out_dim, (uint8_t *)cw.dptr, c.stream)
                        : wl_dev_q8_0_repack((const uint8_t *)raw, (uint32_t)in_dim,
                                             (uint32_t)out_dim, (uint8_t *)cw.dptr, c.stream);
            cudaError_t e = cudaStreamSynchronize(c.stream);
            cudaFree(raw);
            if (rc) return rc;
            if (e != cudaSuccess) return fail(WL_ERR_CUDA, "repack: %s", cudaGetErrorString(e));
        }
    } else {
        return fail_type(w->ggml_type);
    }
    auto res = c.cache.emplace(key, cw);
    *out = &res.first->second;
    return WL_OK;
}

// Copy the library's device status word back with the results of a call;
// report a device-side timeout as an error.
int finish_call(Ctx &c) {
    cudaError_t e = cudaStreamSynchronize(c.stream);
    if (e != cudaSuccess) return fail(WL_ERR_CUDA, "kernel execution: %s", cudaGetErrorString(e));
    if (*c.h_status) {
        const uint32_t f = *c.h_status;
        *c.h_status = 0;
        cudaMemsetAsync(c.d_status, 0, 4, c.stream);
        cudaStreamSynchronize(c.stream);
        return fail(WL_ERR_DEVICE_TIMEOUT, "a device-side wait timed out (flags 0x%x)", f);
    }
    return WL_OK;
}

int stage_status(Ctx &c) {
    WL_CUDA(cudaMemcpyAsync(c.h_status, c.d_status, 4, cudaMemcpyDeviceToHost, c.stream));
    return WL_OK;
}

int i2s_host_call(const wl_tensor_view *weight, const float *input, size_t input_len,
                  float *output, size_t output_len, size_t m, int32_t *acc_out,
                  float *act_scale_out, int8_t *act_q_out) {
    uint32_t K = 0, N = 0;
    float w_scale = 0.f;
    int rc = validate_i2s(weight, input_len, output_len, m == 1, &K, &N, &w_scale);
    if (rc) return rc;
    if (m == 0 || N == 0) return WL_OK;
    if ((!input || !output)) return fail(WL_ERR_INVALID_ARGUMENT, "input/output is NULL");
    Ctx &c = ctx();
    std::lock_guard<std::mutex> g(c.mu);
    if ((rc = ensure_init(c))) return rc;
    CachedWeight *cw = nullptr;
    if ((rc = get_weight(c, weight, K, N, (size_t)K / 4 * N, &cw))) return rc;
    const size_t xin = m * (size_t)K * 4, yout = m * (size_t)N * 4;
    if ((rc = grow(c.x, xin)) || (rc = grow(c.y, yout)) || (rc = grow(c.q, m * (size_t)K)) ||
        (rc = grow(c.scale, m * 4)) || (rc = grow(c.acc, m * (size_t)N * 4)))
        return rc;
    if ((rc = grow_pinned(c, xin + 2 * yout + m * (size_t)K + m * 4 + 64))) return rc;
    uint8_t *pin = (uint8_t *)c.pinned;
    memcpy(pin, input, xin);
    WL_CUDA(cudaMemcpyAsync(c.x.p, pin, xin, cudaMemcpyHostToDevice, c.stream));
    // Prefill of many tokens: one tensor-core GEMM over the weight's int8
    // ternary copy (expanded once, kept with the cached upload; 4x the packed
    // bytes -- the memory-for-speed trade a 180 GB device affords).
    const bool gemm = m >= I2S_GEMM_MIN_TOKENS && m <= 0x7FFFFFFFu;
    const bool fuse = !gemm && K <= I2S_FUSE_Q_MAX_K;
    // no debug outputs: y and the status word come back in one copy
    const bool plain = !gemm && !acc_out && !act_q_out && !act_scale_out;
    if (plain && (rc = grow(c.ys, yout + 16))) return rc;
    float *ydev = plain ? (float *)((uint8_t *)c.ys.p + 16) : (float *)c.y.p;
    uint32_t *dstat = plain ? (uint32_t *)c.ys.p : c.d_status;
    if (gemm) {
        if (!cw->ternary) {
            void *tp = nullptr;
            WL_CUDA(cudaMalloc(&tp, (size_t)K * N));
            cw->ternary = (int8_t *)tp;
            if ((rc = launch_i2s_expand((const uint8_t *)cw->dptr, K, N, cw->ternary, c.stream)))
                return rc;
        }
        if ((rc = launch_quantize((const float *)c.x.p, K, (uint32_t)m, (int8_t *)c.q.p,
                                  (float *)c.scale.p, c.stream, false)))
            return rc;
        if ((rc = launch_i2s_gemm_s8(cw->ternary, w_scale, K, N, (uint32_t)m,
                                     (const int8_t *)c.q.p, (const float *)c.scale.p,
                                     (float *)c.y.p, acc_out ? (int32_t *)c.acc.p : nullptr,
                                     c.stream, true, c.d_status)))
            return rc;
        m = 0;  // no per-token launches below
    } else if (!fuse && (rc = launch_quantize((const float *)c.x.p, K, (uint32_t)m,
                                              (int8_t *)c.q.p, (float *)c.scale.p, c.stream,
                                              false)))
        return rc;
    const size_t m_rows = gemm ? (yout / 4 / N) : m;
    for (size_t t = 0; t < m; ++t) {
        wl_i2s_dev_weight dw = {(const uint8_t *)cw->dptr, w_scale, N, ydev + t * N,
                                acc_out ? (int32_t *)c.acc.p + t * N : nullptr,
                                cw->has_code3 ? 0u : WL_I2S_NO_CODE3};
        I2sLaunch L;
        L.w = &dw;
        L.nw = 1;
        L.K = K;
        if (fuse) {
            L.x = (const float *)c.x.p + t * K;
            L.q_out = act_q_out ? (int8_t *)c.q.p + t * K : nullptr;
            L.scale_out = act_scale_out ? (float *)c.scale.p + t : nullptr;
        } else {
            L.q = (const int8_t *)c.q.p + t * K;
            L.act_scale = (const float *)c.scale.p + t;
        }
        if ((rc = launch_i2s_with_status(L, c.stream, t > 0 || !fuse, dstat))) return rc;
    }
    m = m_rows;
    if (plain) {
        uint8_t *pys = pin + xin;  // [status][y]
        WL_CUDA(cudaMemcpyAsync(pys, c.ys.p, yout + 16, cudaMemcpyDeviceToHost, c.stream));
        cudaError_t e = cudaStreamSynchronize(c.stream);
        if (e != cudaSuccess) return fail(WL_ERR_CUDA, "kernel execution: %s", cudaGetErrorString(e));
        uint32_t f;
        memcpy(&f, pys, 4);
        if (f) {
            WL_CUDA(cudaMemsetAsync(c.ys.p, 0, 4, c.stream));
            WL_CUDA(cudaStreamSynchronize(c.stream));
            return fail(WL_ERR_DEVICE_TIMEOUT, "a device-side wait timed out (flags 0x%x)", f);
        }
        memcpy(output, pys + 16, yout);
        return WL_OK;
    }
    uint8_t *py = pin + xin, *pacc = py + yout, *pq = pacc + yout, *ps = pq + m * (size_t)K;
    WL_CUDA(cudaMemcpyAsync(py, c.y.p, yout, cudaMemcpyDeviceToHost, c.stream));
    if (acc_out) WL_CUDA(cudaMemcpyAsync(pacc, c.acc.p, yout, cudaMemcpyDeviceToHost, c.stream));
    if (act_q_out) WL_CUDA(cudaMemcpyAsync(pq, c.q.p, m * (size_t)K, cudaMemcpyDeviceToHost, c.stream));
    if (act_scale_out) WL_CUDA(cudaMemcpyAsync(ps, c.scale.p, m * 4, cudaMemcpyDeviceToHost, c.stream));
    if ((rc = stage_status(c))) return rc;
    if ((rc = finish_call(c))) return rc;
    memcpy(output, py, yout);
    if (acc_out) memcpy(acc_out, pacc, yout);
    if (act_q_out) memcpy(act_q_out, pq, m * (size_t)K);
    if (act_scale_out) memcpy(act_scale_out, ps, m * 4);
    return WL_OK;
}

// The reference's f32-activation kernels (scalar, SSE2 f32, scalar LUT).
int launch_i2s_f32act(const uint8_t *packed, float w_scale, uint32_t K, uint32_t N,
                      const float *x, float *y, uint32_t kernel, cudaStream_t s, bool pdl) {
    if (N == 0) return WL_OK;
    const dim3 grid((N + I2S_F32ACT_THREADS - 1) / I2S_F32ACT_THREADS), block(I2S_F32ACT_THREADS);
    switch (kernel) {
        case I2S_KERNEL_SCALAR:
            WL_CUDA(launch(i2s_f32act_kernel<I2S_KERNEL_SCALAR>, grid, block, 0, s, pdl, packed,
                           w_scale, K, N, x, y));
            break;
        case I2S_KERNEL_SSE2_F32:
            WL_CUDA(launch(i2s_f32act_kernel<I2S_KERNEL_SSE2_F32>, grid, block, 0, s, pdl, packed,
                           w_scale, K, N, x, y));
            break;
        case I2S_KERNEL_SCALAR_LUT:
            WL_CUDA(launch(i2s_f32act_kernel<I2S_KERNEL_SCALAR_LUT>, grid, block, 0, s, pdl,
                           packed, w_scale, K, N, x, y));
            break;
        default:
            return fail(WL_ERR_INVALID_ARGUMENT, "unknown I2_S kernel %u", kernel);
    }
    return WL_OK;
}

// Host-buffer call of an f32-activation kernel: validation as that kernel
// (the scalar and LUT kernels want the packed length exactly, bitlinear.rs:192,
// bitlinear_lut.rs:174; the SSE2 kernels accept longer data), cached upload,
// one kernel, y and the status word back in one copy.
int i2s_f32act_host_call(const wl_tensor_view *weight, const float *input, size_t input_len,
                         float *output, size_t output_len, uint32_t kernel) {
    uint32_t K = 0, N = 0;
    float w_scale = 0.f;
    int rc = validate_i2s(weight, input_len, output_len, true, &K, &N, &w_scale);
    if (rc) return rc;
    const uint64_t expected = (uint64_t)K / 4 * N;
    if (kernel != I2S_KERNEL_SSE2_F32 && weight->data_len != expected)
        return fail(WL_ERR_GGUF_PARSE,
                    "bitlinear_i2s_matvec_f32: weight \"%s\" data.len()=%zu != expected packed "
                    "%llu (= in_dim/4 x out_dim)",
                    tname(weight), weight->data_len, (unsigned long long)expected);
    if (N == 0) return WL_OK;
    if (!input || !output) return fail(WL_ERR_INVALID_ARGUMENT, "input/output is NULL");
    Ctx &c = ctx();
    std::lock_guard<std::mutex> g(c.mu);
    if ((rc = ensure_init(c))) return rc;
    CachedWeight *cw = nullptr;
    if ((rc = get_weight(c, weight, K, N, (size_t)K / 4 * N, &cw))) return rc;
    const size_t xin = (size_t)K * 4, yout = (size_t)N * 4;
    if ((rc = grow(c.x, xin)) || (rc = grow(c.ys, yout + 16)) ||
        (rc = grow_pinned(c, xin + yout + 64)))
        return rc;
    uint8_t *pin = (uint8_t *)c.pinned;
    memcpy(pin, input, xin);
    WL_CUDA(cudaMemcpyAsync(c.x.p, pin, xin, cudaMemcpyHostToDevice, c.stream));
    if ((rc = launch_i2s_f32act((const uint8_t *)cw->dptr, w_scale, K, N, (const float *)c.x.p,
                                (float *)((uint8_t *)c.ys.p + 16), kernel, c.stream, false)))
        return rc;
    uint8_t *pys = pin + xin;  // [status][y]
    WL_CUDA(cudaMemcpyAsync(pys, c.ys.p, yout + 16, cudaMemcpyDeviceToHost, c.stream));
    cudaError_t e = cudaStreamSynchronize(c.stream);
    if (e != cudaSuccess) return fail(WL_ERR_CUDA, "kernel execution: %s", cudaGetErrorString(e));
    memcpy(output, pys + 16, yout);
    return WL_OK;
}

// lm_head.rs:35-85 validation for the Q6_K / Q8_0 arms.
int validate_lm_head(const float *hidden, size_t hidden_len, const wl_tensor_view *t,
                     uint32_t n_embd, uint32_t vocab, uint64_t *row_bytes) {
    if (!t) return fail(WL_ERR_INVALID_ARGUMENT, "token_embd is NULL");
    const uint32_t ty = t->ggml_type;
    if (ty != WL_GGML_F16 && ty != WL_GGML_Q4_0 && ty != WL_GGML_Q4_K && ty != WL_GGML_Q6_K &&
        ty != WL_GGML_Q8_0)
        return fail(WL_ERR_GGUF_PARSE,
                    "compute_logits: token_embd is raw type %u, expected F16, Q4_0, Q4_K, Q6_K, "
                    "or Q8_0",
                    ty);
    if (t->n_dims != 2 || !t->shape || t->shape[0] != n_embd || t->shape[1] != vocab)
        return fail(WL_ERR_GGUF_PARSE, "compute_logits: token_embd shape != [%u, %u]", n_embd,
                    vocab);
    if (hidden_len != n_embd)
        return fail(WL_ERR_GGUF_PARSE,
                    "compute_logits: final_hidden.len()=%zu != embedding_length=%u", hidden_len,
                    n_embd);
    if (ty != WL_GGML_Q6_K && ty != WL_GGML_Q8_0)
        return fail(WL_ERR_NOT_IMPLEMENTED,
                    "compute_logits: raw type %u rows are not on the B200 path", ty);
    int rc = row_bytes_for(ty, n_embd, row_bytes);
    if (rc) return rc;
    if (t->data_len != *row_bytes * vocab)
        return fail(WL_ERR_GGUF_PARSE, "compute_logits: token_embd.data.len()=%zu != expected %llu",
                    t->data_len, (unsigned long long)(*row_bytes * vocab));
    if (!t->data && t->data_len) return fail(WL_ERR_INVALID_ARGUMENT, "token_embd data is NULL");
    if (!hidden && hidden_len) return fail(WL_ERR_INVALID_ARGUMENT, "final_hidden is NULL");
    return WL_OK;
}

// Shared by compute_logits / lm_head_greedy / the quantized linear arms.
int rows_host_call(const wl_tensor_view *t, uint32_t n_embd, uint32_t vocab, uint64_t row_bytes,
                   const float *hidden, size_t batch, float *logits, uint32_t *ids) {
    if (batch == 0 || vocab == 0) return WL_OK;
    Ctx &c = ctx();
    std::lock_guard<std::mutex> g(c.mu);
    int rc = ensure_init(c);
    if (rc) return rc;
    CachedWeight *cw = nullptr;
    if ((rc = get_weight(c, t, n_embd, vocab, (size_t)(row_bytes * vocab), &cw))) return rc;
    if (cw->bad_scale) return fail(WL_ERR_GGUF_PARSE, "Q8_0 block has a non-finite scale");
    const size_t xin = batch * (size_t)n_embd * 4, lout = batch * (size_t)vocab * 4;
    if ((rc = grow(c.x, xin)) || (rc = grow(c.y, lout)) || (rc = grow(c.ids, batch * 4)) ||
        (rc = grow(c.scratch, wl_q6k_scratch_bytes((uint32_t)batch))))
        return rc;
    if ((rc = grow_pinned(c, xin + lout + batch * 4 + 64))) return rc;
    uint8_t *pin = (uint8_t *)c.pinned;
    memcpy(pin, hidden, xin);
    WL_CUDA(cudaMemcpyAsync(c.x.p, pin, xin, cudaMemcpyHostToDevice, c.stream));
    float *dlog = logits ? (float *)c.y.p : nullptr;
    if (t->ggml_type == WL_GGML_Q6_K) {
        rc = launch_q6k((const uint8_t *)cw->dptr, n_embd, vocab, (const float *)c.x.p,
                        (uint32_t)batch, dlog, ids ? (uint32_t *)c.ids.p : nullptr, c.scratch.p,
                        c.stream, false);
        if (rc) return rc;
    } else {
        for (size_t b = 0; b < batch; ++b) {
            rc = launch_q8((const uint8_t *)cw->dptr, n_embd, vocab,
                           (const float *)c.x.p + b * n_embd, (float *)c.y.p + b * vocab,
                           c.stream, false);
            if (rc) return rc;
            if (ids) {
                auto *slot = (unsigned long long *)c.scratch.p;
                WL_CUDA(launch(argmax_kernel, dim3(std::min<uint32_t>(vocab / ARGMAX_THREADS + 1, 148)),
                               dim3(ARGMAX_THREADS), 0, c.stream, true,
                               (const float *)c.y.p + b * vocab, vocab, slot,
                               (uint32_t *)(slot + 1), (uint32_t *)c.ids.p + b));
            }
        }
        dlog = logits ? (float *)c.y.p : nullptr;
    }
    uint8_t *pl = pin + xin, *pid = pl + lout;
    if (dlog) WL_CUDA(cudaMemcpyAsync(pl, dlog, lout, cudaMemcpyDeviceToHost, c.stream));
    if (ids) WL_CUDA(cudaMemcpyAsync(pid, c.ids.p, batch * 4, cudaMemcpyDeviceToHost, c.stream));
    if ((rc = stage_status(c))) return rc;
    if ((rc = finish_call(c))) return rc;
    if (logits) memcpy(logits, pl, lout);
    if (ids) memcpy(ids, pid, batch * 4);
    return WL_OK;
}

}  // namespace

// ------------------------------------------------------- no-allocation variant
// Scratch of wl_dev_i2s_matvec_f32_noalloc, in static device memory instead of
// caller- or library-allocated buffers: [0, 4) activation scale (f32),
// [4, 8) device status word, [256, 256 + WL_NOALLOC_MAX_IN_DIM) the int8
// activations.  Every GPU that loads this library holds these bytes until the
// process exits.  In host code the name is only a host-side stand-in; the
// device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_noalloc_scratch[256 + WL_NOALLOC_MAX_IN_DIM];

namespace {

struct NoAllocDevice {
    bool ready = false;
    void *ctx = nullptr;         // CUDA context the address was resolved in
    uint8_t *scratch = nullptr;  // device address of g_noalloc_scratch
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[64];

// The calling thread's current CUDA context (driver API through the runtime's
// entry-point table, so the library needs no -lcuda).  A module is loaded
// per context: after cudaDeviceReset, or in a caller that made another
// context current, g_noalloc_scratch has a new address.
int current_context(void **out) {
    using GetCtx = int (*)(void **);
    static GetCtx fn = nullptr;
    if (!fn) {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !f)
            return fail(WL_ERR_CUDA, "cuCtxGetCurrent entry point unavailable");
        fn = reinterpret_cast<GetCtx>(f);
    }
    *out = nullptr;
    if (fn(out) != 0) return fail(WL_ERR_CUDA, "cuCtxGetCurrent failed");
    return WL_OK;
}

// Once per (device, context), with that device current: resolve the array's
// device address and raise the kernels' shared-memory limit.  Allocates
// nothing.  With create = false, only reports an address resolved earlier
// in the current context (nullptr if none).
int noalloc_setup(uint8_t **scratch, bool create = true) {
    *scratch = nullptr;
    int dev = 0;
    WL_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(WL_ERR_INVALID_ARGUMENT, "device %d out of range", dev);
    void *cur = nullptr;
    int rc = current_context(&cur);
    if (rc) return rc;
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    NoAllocDevice &d = g_noalloc_dev[dev];
    if (d.ready && cur && d.ctx == cur) {
        *scratch = d.scratch;
        return WL_OK;
    }
    if (!create) return WL_OK;
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
        return fail(WL_ERR_CUDA, "cudaGetSymbolAddress(g_noalloc_scratch) on device %d: %s", dev,
                    cudaGetErrorString(e));
    if ((rc = configure_kernels())) return rc;
    if (!cur && (rc = current_context(&cur))) return rc;  // the runtime made its context now
    d.scratch = static_cast<uint8_t *>(p);
    d.ctx = cur;
    d.ready = true;
    *scratch = d.scratch;
    return WL_OK;
}

// Read and clear the allocation-free entry point's status word on the
// current device, if that entry point has run there in this context.
int noalloc_take_status(uint32_t *flags) {
    *flags = 0;
    uint8_t *scratch = nullptr;
    int rc = noalloc_setup(&scratch, false);
    if (rc || !scratch) return rc;
    WL_CUDA(cudaDeviceSynchronize());
    WL_CUDA(cudaMemcpyFromSymbol(flags, g_noalloc_scratch, 4, 4));
    if (*flags) {
        const uint32_t zero = 0;
        WL_CUDA(cudaMemcpyToSymbol(g_noalloc_scratch, &zero, 4, 4));
    }
    return WL_OK;
}

}  // namespace

// ------------------------------------------------------------- stream plans
struct wl_i2s_stream_plan {
    int device = 0;
    uint32_t n_ops = 0, n_quant = 0, grid = 0;
    bool c3 = true;
    void *d_block = nullptr;  // maps | ops | cta_blocks | quant jobs | scales | q buffers
    CUtensorMap *d_maps = nullptr;
    I2sStreamOp *d_ops = nullptr;
    uint32_t *d_cta_blocks = nullptr;
    QuantJob *d_qjobs = nullptr;
    uint32_t *status = nullptr;
    uintptr_t y_lo = 0, y_hi = 0;  // extent of the ops' outputs (tensor-parallel checks)
};

namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode_tiled(EncodeTiledFn *fn) {
    static EncodeTiledFn cached = nullptr;
    if (!cached) {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !f)
            return fail(WL_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
        cached = (EncodeTiledFn)f;
    }
    *fn = cached;
    return WL_OK;
}

// Tensor map of one packed I2_S weight: 2-D (row bytes, rows), 32-row x
// 128-byte boxes, 128-byte swizzle, zero fill out of bounds.
int encode_i2s_map(const uint8_t *packed, uint32_t K, uint32_t N, CUtensorMap *map) {
    EncodeTiledFn enc;
    int rc = get_encode_tiled(&enc);
    if (rc) return rc;
    const cuuint64_t dims[2] = {K / 4u, N};
    const cuuint64_t strides[1] = {K / 4u};
    const cuuint32_t box[2] = {STREAM_BOX_BYTES, STREAM_BOX_ROWS};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)packed, dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(WL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return WL_OK;
}

// ------------------------------------------------------------------ prefill GEMM
int encode_2d(EncodeTiledFn enc, CUtensorMap *map, const void *base, uint64_t inner_bytes,
              uint64_t rows, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    const cuuint64_t dims[2] = {inner_bytes, rows};
    const cuuint64_t strides[1] = {inner_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(WL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return WL_OK;
}

// Y[m][n] for m tokens from pre-quantised activations q [m][K] (with their
// scales and row sums) and code-3-free packed weights [N][K/4].
int launch_i2s_gemm(const uint8_t *packed, float w_scale, uint32_t K, uint32_t N, uint32_t M,
                    const int8_t *q, const float *act_scale, const int32_t *rowsum, float *y,
                    int32_t *acc, cudaStream_t s, bool pdl, uint32_t *status) {
    if (M == 0 || N == 0) return WL_OK;
    EncodeTiledFn enc;
    int rc = get_encode_tiled(&enc);
    if (rc) return rc;
    const uint32_t mt = (M + GEMM_BM - 1) / GEMM_BM;
    const uint32_t sms = (uint32_t)sm_count_for_launch();
    // widest tile that still gives every SM work
    int bn = 256;
    if ((uint64_t)mt * ((N + 255) / 256) < sms) bn = 128;
    if (bn == 128 && (uint64_t)mt * ((N + 127) / 128) < sms) bn = 64;
    I2sGemmParams p;
    memset(&p, 0, sizeof p);
    if ((rc = encode_2d(enc, &p.a_map, q, K, M, GEMM_BK, GEMM_BM, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = encode_2d(enc, &p.bp_map, packed, K / 4u, N, GEMM_BK / 4, (uint32_t)bn,
                        CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    p.act_scale = act_scale;
    p.rowsum = rowsum;
    p.w_scale = w_scale;
    p.M = M;
    p.N = N;
    p.K = K;
    p.y = y;
    p.acc = acc;
    p.status = status;
    const dim3 grid((N + bn - 1) / bn, mt);
    if (bn == 256)
        WL_CUDA(launch(i2s_gemm_kernel<256>, grid, dim3(GEMM_THREADS), GemmSmem<256>::DYN, s, pdl, p));
    else if (bn == 128)
        WL_CUDA(launch(i2s_gemm_kernel<128>, grid, dim3(GEMM_THREADS), GemmSmem<128>::DYN, s, pdl, p));
    else
        WL_CUDA(launch(i2s_gemm_kernel<64>, grid, dim3(GEMM_THREADS), GemmSmem<64>::DYN, s, pdl, p));
    return WL_OK;
}

// Y[m][n] from pre-quantised activations q [m][K] and int8 ternary weights
// t [N][K] (i2s_expand_kernel): the warp-specialised persistent GEMM.
int launch_i2s_gemm_s8(const int8_t *t, float w_scale, uint32_t K, uint32_t N, uint32_t M,
                       const int8_t *q, const float *act_scale, float *y, int32_t *acc,
                       cudaStream_t s, bool pdl, uint32_t *status) {
    if (M == 0 || N == 0) return WL_OK;
    EncodeTiledFn enc;
    int rc = get_encode_tiled(&enc);
    if (rc) return rc;
    const uint32_t mt = (M + GEMM_BM - 1) / GEMM_BM;
    const uint32_t sms = (uint32_t)sm_count_for_launch();
    // Tile width by estimated time: waves of persistent tiles x per-tile cost
    // (mainloop ~ BN columns, plus a fixed share for the epilogue and fill).
    int bn = 256;
    uint64_t best = ~0ull;
    for (int cand : {256, 128, 64}) {
        const uint64_t tiles = (uint64_t)mt * ((N + cand - 1) / cand);
        const uint64_t cost = ((tiles + sms - 1) / sms) * (uint64_t)(cand + 128);
        if (cost < best) {
            best = cost;
            bn = cand;
        }
    }
    I2sGemmWsParams p;
    memset(&p, 0, sizeof p);
    if ((rc = encode_2d(enc, &p.a_map, q, K, M, GEMM_BK, GEMM_BM, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = encode_2d(enc, &p.b_map, t, K, N, GEMM_BK, (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    // output boxes by TMA store when rows are 16-byte multiples
    if ((N % 4u) == 0 && aligned16(y)) {
        const cuuint64_t dims[2] = {N, M};
        const cuuint64_t strides[1] = {(cuuint64_t)N * 4u};
        const cuuint32_t box[2] = {32, 32};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&p.y_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)y, dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(WL_ERR_CUDA, "cuTensorMapEncodeTiled (y) failed (%d)", (int)r);
        p.use_tma_store = 1;
    }
    p.act_scale = act_scale;
    p.w_scale = w_scale;
    p.M = M;
    p.N = N;
    p.K = K;
    p.y = y;
    p.acc = acc;
    p.status = status;
    const uint32_t tiles = mt * ((N + bn - 1) / bn);
    const dim3 grid(std::min(tiles, sms));
    if (bn == 256)
        WL_CUDA(launch(i2s_gemm_ws_kernel<256>, grid, dim3(WS_THREADS), WsSmem<256>::DYN, s, pdl, p));
    else if (bn == 128)
        WL_CUDA(launch(i2s_gemm_ws_kernel<128>, grid, dim3(WS_THREADS), WsSmem<128>::DYN, s, pdl, p));
    else
        WL_CUDA(launch(i2s_gemm_ws_kernel<64>, grid, dim3(WS_THREADS), WsSmem<64>::DYN, s, pdl, p));
    return WL_OK;
}

int launch_i2s_expand(const uint8_t *packed, uint32_t K, uint32_t N, int8_t *out, cudaStream_t s) {
    const size_t blocks = (size_t)N * (K / 128u);
    if (!blocks) return WL_OK;
    const uint32_t grid = (uint32_t)std::min<size_t>((blocks + 255) / 256, 4u * 1184u);
    i2s_expand_kernel<<<grid, 256, 0, s>>>(packed, blocks, out);
    WL_CUDA(cudaGetLastError());
    return WL_OK;
}

int build_stream_plan(const wl_i2s_stream_op *ops, uint32_t n_ops, wl_i2s_stream_plan *plan) {
    // distinct inputs -> one quantisation each
    std::map<const float *, uint32_t> xid;
    std::vector<uint32_t> qK;
    std::vector<uint32_t> block_begin(n_ops);
    uint64_t total_blocks = 0;
    for (uint32_t j = 0; j < n_ops; ++j) {
        const wl_i2s_stream_op &o = ops[j];
        if (o.in_dim < STREAM_MIN_K || o.in_dim % 128 || o.in_dim > STREAM_MAX_K)
            return fail(WL_ERR_INVALID_ARGUMENT,
                        "op %u: in_dim %u must be a multiple of 128 in [%u, %u] for a stream plan",
                        j, o.in_dim, STREAM_MIN_K, STREAM_MAX_K);
        if (!o.packed || !aligned16(o.packed) || !o.x || !aligned16(o.x) || (!o.y && o.out_dim))
            return fail(WL_ERR_INVALID_ARGUMENT, "op %u: NULL or misaligned pointer", j);
        if (!std::isfinite(o.w_scale))
            return fail(WL_ERR_GGUF_PARSE, "op %u: i2s_scale: non-finite scale", j);
        auto it = xid.find(o.x);
        if (it == xid.end()) {
            xid.emplace(o.x, (uint32_t)qK.size());
            qK.push_back(o.in_dim);
        } else if (qK[it->second] != o.in_dim) {
            return fail(WL_ERR_INVALID_ARGUMENT, "op %u: input shared with a different in_dim", j);
        }
        block_begin[j] = (uint32_t)total_blocks;
        total_blocks += (o.out_dim + STREAM_BOX_ROWS - 1) / STREAM_BOX_ROWS;
    }
    if (total_blocks > 0x7FFFFFFFull) return fail(WL_ERR_INVALID_ARGUMENT, "too many rows");
    Ctx &c = ctx();
    std::lock_guard<std::mutex> g(c.mu);
    int rc = ensure_init(c);
    if (rc) return rc;
    const uint32_t G = (uint32_t)std::max(1, c.sm_count);
    const uint32_t nq = (uint32_t)qK.size();
    const size_t off_maps = 0;
    const size_t off_ops = align_up(off_maps + sizeof(CUtensorMap) * n_ops, 64);
    const size_t off_cta = align_up(off_ops + sizeof(I2sStreamOp) * n_ops, 16);
    const size_t off_q = align_up(off_cta + sizeof(uint32_t) * (G + 1), 16);
    const size_t off_sc = align_up(off_q + sizeof(QuantJob) * nq, 16);
    size_t bytes = align_up(off_sc + sizeof(float) * nq, 16);
    std::vector<size_t> qoff(nq);
    for (uint32_t i = 0; i < nq; ++i) {
        qoff[i] = bytes;
        bytes = align_up(bytes + qK[i], 16);
    }
    WL_CUDA(cudaMalloc(&plan->d_block, bytes));
    uint8_t *base = (uint8_t *)plan->d_block;
    std::vector<uint8_t> host(bytes, 0);
    std::vector<I2sStreamOp> hops(n_ops);
    bool any_c3 = false;
    uint32_t *found = c.d_status + 8;
    for (uint32_t j = 0; j < n_ops; ++j) {
        const wl_i2s_stream_op &o = ops[j];
        const uint32_t qi = xid[o.x];
        hops[j].q = (const int8_t *)(base + qoff[qi]);
        hops[j].act_scale = (const float *)(base + off_sc) + qi;
        hops[j].y = o.y;
        hops[j].acc = o.acc;
        hops[j].w_scale = o.w_scale;
        hops[j].K = o.in_dim;
        hops[j].N = o.out_dim;
        hops[j].block_begin = block_begin[j];
        hops[j].row_off = o.row_off;
        if (o.out_dim) {
            const uintptr_t lo = (uintptr_t)(o.y + o.row_off);
            const uintptr_t hi = lo + (uintptr_t)o.out_dim * sizeof(float);
            plan->y_lo = plan->y_lo ? std::min(plan->y_lo, lo) : lo;
            plan->y_hi = std::max(plan->y_hi, hi);
        }
        if (o.out_dim) {
            CUtensorMap m;
            if ((rc = encode_i2s_map(o.packed, o.in_dim, o.out_dim, &m))) return rc;
            memcpy(host.data() + off_maps + sizeof(CUtensorMap) * j, &m, sizeof m);
        }
        if (!(o.flags & WL_I2S_NO_CODE3) && !any_c3 && o.out_dim) {
            const size_t n16 = (size_t)o.out_dim * (o.in_dim / 4) / 16;
            WL_CUDA(cudaMemsetAsync(found, 0, 4, c.stream));
            const uint32_t grid = (uint32_t)std::min<size_t>((n16 + 255) / 256, 2048);
            i2s_scan_code3_kernel<<<grid, 256, 0, c.stream>>>((const uint4 *)o.packed, n16, found);
            WL_CUDA(cudaGetLastError());
            WL_CUDA(cudaMemcpyAsync(c.h_status + 8, found, 4, cudaMemcpyDeviceToHost, c.stream));
            WL_CUDA(cudaStreamSynchronize(c.stream));
            any_c3 = c.h_status[8] != 0;
        }
    }
    memcpy(host.data() + off_ops, hops.data(), sizeof(I2sStreamOp) * n_ops);
    // byte-balanced block boundaries per CTA
    std::vector<uint32_t> cb(G + 1, 0);
    {
        uint64_t total_bytes = 0;
        for (uint32_t j = 0; j < n_ops; ++j)
            total_bytes += (uint64_t)(ops[j].out_dim + STREAM_BOX_ROWS - 1) / STREAM_BOX_ROWS *
                           STREAM_BOX_ROWS * (ops[j].in_dim / 4);
        uint32_t j = 0, b = 1;
        uint64_t cum = 0;
        for (uint32_t blk = 0; blk < (uint32_t)total_blocks && b < G; ++blk) {
            while (j + 1 < n_ops && blk >= block_begin[j + 1]) ++j;
            cum += (uint64_t)STREAM_BOX_ROWS * (ops[j].in_dim / 4);
            while (b < G && cum >= total_bytes * b / G) cb[b++] = blk + 1;
        }
        for (; b < G; ++b) cb[b] = (uint32_t)total_blocks;
        cb[G] = (uint32_t)total_blocks;
    }
    memcpy(host.data() + off_cta, cb.data(), sizeof(uint32_t) * (G + 1));
    std::vector<QuantJob> qj(nq);
    for (auto &kv : xid) {
        const uint32_t i = kv.second;
        qj[i].x = kv.first;
        qj[i].q = (int8_t *)(base + qoff[i]);
        qj[i].scale = (float *)(base + off_sc) + i;
        qj[i].n = qK[i];
    }
    memcpy(host.data() + off_q, qj.data(), sizeof(QuantJob) * nq);
    WL_CUDA(cudaMemcpyAsync(base, host.data(), bytes, cudaMemcpyHostToDevice, c.stream));
    WL_CUDA(cudaStreamSynchronize(c.stream));
    plan->device = c.device;
    plan->n_ops = n_ops;
    plan->n_quant = nq;
    plan->grid = G;
    plan->c3 = any_c3;
    plan->d_maps = (CUtensorMap *)(base + off_maps);
    plan->d_ops = (I2sStreamOp *)(base + off_ops);
    plan->d_cta_blocks = (uint32_t *)(base + off_cta);
    plan->d_qjobs = (QuantJob *)(base + off_q);
    plan->status = c.d_status;
    return WL_OK;
}

}  // namespace

// ------------------------------------------------------- tensor-parallel group
struct wl_tp_group {
    int device = 0, rank = 0, world = 0;
    uint8_t *local = nullptr;  // header + caller region, cudaMalloc'd (IPC-exportable)
    size_t bytes = 0;
    uint8_t *peers[TP_MAX_WORLD] = {};
    bool connected = false;
};

namespace {

int tp_params(wl_tp_group *g, bool wait, TpParams *tp) {
    if (!g) return fail(WL_ERR_INVALID_ARGUMENT, "group is NULL");
    if (!g->connected) return fail(WL_ERR_COMM, "group is not connected (wl_tp_connect)");
    memset(tp, 0, sizeof *tp);
    tp->world = g->world;
    tp->rank = g->rank;
    tp->local_base = g->local;
    for (int r = 0; r < g->world; ++r) tp->peer_base[r] = g->peers[r];
    tp->wait = wait ? 1u : 0u;
    return WL_OK;
}

// Outputs written to peers are addressed by their offset in this rank's
// block, so they must lie inside the caller region of the block.
int check_sym_range(wl_tp_group *g, const float *y, size_t n_floats) {
    const uintptr_t lo = (uintptr_t)y, hi = lo + n_floats * sizeof(float);
    if (!y || lo < (uintptr_t)(g->local + TP_HEADER_BYTES) || hi > (uintptr_t)(g->local + g->bytes) ||
        (lo & 3u))
        return fail(WL_ERR_INVALID_ARGUMENT,
                    "a gathered output must lie in the group's block (wl_tp_buffer)");
    return WL_OK;
}

int launch_q6k_tp(const uint8_t *packed, uint32_t n_embd, uint32_t vocab, uint32_t row_offset,
                  const float *hidden, uint32_t batch, uint32_t *ids, void *scratch,
                  cudaStream_t s, const TpParams *tp) {
    // (an empty shard still launches, so that its rank's keys and arrival exist)
    return launch_q6k_all(packed, n_embd, vocab, row_offset, hidden, batch, nullptr, ids, scratch,
                          s, true, tp);
}

}  // namespace

// ------------------------------------------------------- BitNet decode engine
// Device-resident single-token forward with the reference's i8 KV cache
// (cached_forward.rs:206-504) and greedy generation (generate.rs:111-190).
struct wl_bitnet {
    wl_bitnet_config cfg{};
    int device = 0;
    cudaStream_t stream = nullptr;
    uint8_t *wblock = nullptr;             // every packed I2_S weight
    std::vector<wl_i2s_dev_weight> mats;   // n_layers * 7 (y set per use)
    float *norms = nullptr, *out_norm = nullptr;
    uint8_t *q6k = nullptr;                // repacked tied embedding / lm-head
    float2 *rope = nullptr;
    int8_t *kq = nullptr, *vq = nullptr;
    float *ks = nullptr, *vs = nullptr;
    float *hidden = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr,
          *gate = nullptr, *up = nullptr, *final_h = nullptr;
    uint32_t *d_token = nullptr, *d_pos = nullptr, *d_step = nullptr, *d_ids = nullptr;
    uint32_t ids_cap = 0;
    uint32_t splits = 1;                   // attention CTAs per head (per-op path)
    bool gqa_attn = false;                 // fast mode: attn_gqa_batch_kernel (KV head x split CTAs)
    bool exact_attn = false;               // exact mode: attn_exact_kernel (history in shared memory)
    uint32_t attn_chunk = 0;               // its positions per CTA
    float *attn_partial = nullptr;
    uint32_t *attn_counters = nullptr;
    // persistent whole-forward kernel
    bool mega = false, mega_c3 = false;
    uint32_t mega_grid = 0, mega_splits = 1;
    size_t mega_smem = 0;
    MegaParams mp{};
    MegaLayer *d_layers = nullptr;
    void *mega_state = nullptr;             // arrivals (u64), launches, abort
    float *att_g = nullptr;                 // exact-mode attention output
    void *lm_scratch = nullptr;
    uint32_t *h_pinned = nullptr;          // token staging
    uint32_t pos = 0;                      // host mirror of the cache position
    bool have_hidden = false;              // final_h holds a forward's output
    cudaGraphExec_t g_forward = nullptr, g_step = nullptr, g_last = nullptr;
    // tensor parallel (world > 1): this rank's row slice of every BitLinear,
    // hidden / q|k|v / gate|up in the group's symmetric block (gathered by
    // the matvec kernels), a vocab shard of the lm-head
    wl_tp_group *tpg = nullptr;
    TpParams tp{};
    std::vector<uint32_t> row_offs;        // n_layers * 7: first global row of the slice
    uint32_t vocab_off = 0, vocab_shard = 0;
};

namespace {

constexpr int BN_MATS = 7;  // q, k, v, o, gate, up, down

using AttnKernel = void (*)(AttnParams);
// fast-mode batched attention for head_dim 64 / 128 and 1..4 q heads per KV head
AttnKernel gqa_attn_kernel(uint32_t hd, uint32_t group) {
    static const AttnKernel k64[4] = {attn_gqa_batch_kernel<64, 1>, attn_gqa_batch_kernel<64, 2>,
                                      attn_gqa_batch_kernel<64, 3>, attn_gqa_batch_kernel<64, 4>};
    static const AttnKernel k128[4] = {attn_gqa_batch_kernel<128, 1>, attn_gqa_batch_kernel<128, 2>,
                                       attn_gqa_batch_kernel<128, 3>, attn_gqa_batch_kernel<128, 4>};
    if (group < 1 || group > AB_MAX_GROUP) return nullptr;
    if (hd == 64) return k64[group - 1];
    if (hd == 128) return k128[group - 1];
    return nullptr;
}


uint32_t bn_kv(const wl_bitnet_config &c) { return c.n_kv_heads * c.head_dim; }

int bn_validate(const wl_bitnet_config *c) {
    if (!c) return fail(WL_ERR_INVALID_ARGUMENT, "config is NULL");
    const uint32_t E = c->n_embd, F = c->n_ff, HD = c->head_dim;
    if (!c->n_layers || !E || !F || !HD || !c->n_heads || !c->n_kv_heads || !c->vocab ||
        !c->max_seq)
        return fail(WL_ERR_GGUF_PARSE, "bitnet config: zero dimension");
    if (E % 256 || E > I2S_FUSE_Q_MAX_K)
        return fail(WL_ERR_GGUF_PARSE, "embedding_length %u must be a multiple of 256 <= %u", E,
                    I2S_FUSE_Q_MAX_K);
    if (F % 128 || F > I2S_FUSE_Q_MAX_K)
        return fail(WL_ERR_GGUF_PARSE, "feed_forward_length %u must be a multiple of 128 <= %u",
                    F, I2S_FUSE_Q_MAX_K);
    if (c->n_heads * HD != E || c->n_heads % c->n_kv_heads)
        return fail(WL_ERR_GGUF_PARSE, "heads %u x head_dim %u vs embedding %u / kv heads %u",
                    c->n_heads, HD, E, c->n_kv_heads);
    if (HD % 32 || HD > 256 || (bn_kv(*c)) % 128)
        return fail(WL_ERR_GGUF_PARSE, "head_dim %u must be a multiple of 32 <= 256 and kv_dim a "
                    "multiple of 128", HD);
    if (!c->n_rot || c->n_rot % 2 || c->n_rot > HD)
        return fail(WL_ERR_GGUF_PARSE, "rope_dimension_count %u", c->n_rot);
    if (c->kv_f16 > 1) return fail(WL_ERR_INVALID_ARGUMENT, "kv_f16 must be 0 or 1");
    if (attn_smem_bytes(bn_kv(*c), HD, c->max_seq, 1, c->kv_f16 != 0) > (size_t)WL_MAX_DYN_SMEM)
        return fail(WL_ERR_INVALID_ARGUMENT, "max_seq %u too long for the attention kernel",
                    c->max_seq);
    if (!std::isfinite(c->eps) || !std::isfinite(c->freq_base))
        return fail(WL_ERR_GGUF_PARSE, "non-finite eps / rope base");
    return WL_OK;
}

// The reference's RoPE angles (primitives.rs:316-340): theta = pos *
// freq_base^(-2j / n_rot) in f32 with the C library's powf, then sinf/cosf.
void bn_rope_table(const wl_bitnet_config &c, std::vector<float2> &t) {
    const uint32_t half = c.n_rot / 2;
    t.resize((size_t)c.max_seq * half);
    const float n_rot_f = (float)c.n_rot;
    for (uint32_t p = 0; p < c.max_seq; ++p) {
        const float pos = (float)p;
        for (uint32_t j = 0; j < half; ++j) {
            const float exponent = -2.0f * (float)j / n_rot_f;
            const float theta = pos * powf(c.freq_base, exponent);
            t[(size_t)p * half + j] = make_float2(cosf(theta), sinf(theta));
        }
    }
}

// Tensor parallel: this rank's row slices, outputs stored to every rank;
// tp_wait: the input x was gathered, wait for every rank's stores first.
int bn_matvec(wl_bitnet *m, uint32_t l, int first, int count, uint32_t K, const float *x,
              float *const *ys, uint32_t pre, const float *norm_w, const float *x2,
              uint32_t residual, uint32_t finite_flag, cudaStream_t s, bool tp_wait = false) {
    wl_i2s_dev_weight w[3];
    for (int j = 0; j < count; ++j) {
        w[j] = m->mats[(size_t)l * BN_MATS + first + j];
        w[j].y = ys[j];
        w[j].acc = nullptr;
    }
    I2sLaunch L;
    TpParams tp = m->tp;
    if (m->tpg) {
        tp.wait = tp_wait ? 1u : 0u;
        L.tp = &tp;
        L.row_offs = m->row_offs.data() + (size_t)l * BN_MATS + first;
    }
    L.w = w;
    L.nw = (uint32_t)count;
    L.K = K;
    L.x = x;
    L.pre = pre;
    L.norm_w = norm_w;
    L.x2 = x2;
    L.eps = m->cfg.eps;
    L.residual = residual;
    L.finite_flag = finite_flag;
    L.exact_norm = m->cfg.exact;
    return launch_i2s(L, s, true);
}

// One token: embedding (of *d_token; appended to d_ids when commit), every
// layer, output norm; the device position advances by one.
// Shared-memory layout and parameters of the persistent kernel; it runs when
// one CTA fits on every SM (cooperative launch), else the per-op kernels do.
int bn_setup_mega(wl_bitnet *m) {
    const wl_bitnet_config &c = m->cfg;
    const uint32_t E = c.n_embd, F = c.n_ff, KV = bn_kv(c), HD = c.head_dim, G = m->mega_grid;
    auto up = [](size_t v, size_t a) { return (v + a - 1) / a * a; };
    const size_t rpc_qkv = (E + 2 * KV + G - 1) / G, rpc_gu = (2 * F + G - 1) / G,
                 rpc_e = (E + G - 1) / G;
    const size_t size_a = up(std::max(rpc_qkv, rpc_gu) * (E / 4), 1024);
    const size_t size_b = up(rpc_e * std::max(E / 4, F / 4), 1024);
    const size_t xq = up((size_t)std::max(E, F) * 4, 16) + up(std::max(E, F), 16);
    const uint32_t S = m->mega_splits, half = c.n_rot / 2;
    const size_t chunk = ((c.max_seq + S - 1) / S + 3) & ~3u;
    const size_t attn = (2 * KV + HD + MEGA_THREADS + 2 * chunk) * 4 + ((half + 1) & ~1u) * 8 +
                        2 * KV;
    const size_t region = up(std::max(xq, attn), 16);
    const size_t cmb = up(mega_cmb_floats(c.n_heads, S) * 4, 16);
    MegaParams &p = m->mp;
    p.buf_a = 0;
    p.norm_a = (uint32_t)size_a;
    p.buf_b = p.norm_a + (uint32_t)up((size_t)E * 4, 128);
    p.norm_b = p.buf_b + (uint32_t)size_b;
    p.xs_off = p.norm_b + (uint32_t)up((size_t)std::max(E, F) * 4, 128);
    p.qs_off = p.xs_off + (uint32_t)up((size_t)std::max(E, F) * 4, 16);
    p.att_off = p.xs_off;
    p.cmb_off = p.xs_off + (uint32_t)region;
    p.hloc_off = p.cmb_off + (uint32_t)cmb;
    m->mega_smem = p.hloc_off + up(rpc_e * 4, 16);
    if (m->mega_smem > (size_t)WL_MAX_DYN_SMEM) return WL_OK;  // per-op kernels
    bool c3 = false;
    for (auto &w : m->mats) c3 |= !(w.flags & WL_I2S_NO_CODE3);
    const void *k = c3 ? (const void *)bitnet_mega_kernel<true> : (const void *)bitnet_mega_kernel<false>;
    int per_sm = 0;
    WL_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, MEGA_THREADS, m->mega_smem));
    if (per_sm < 1) return WL_OK;
    std::vector<MegaLayer> hl(c.n_layers);
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        for (int j = 0; j < BN_MATS; ++j) {
            hl[l].w[j] = m->mats[(size_t)l * BN_MATS + j].packed;
            hl[l].scale[j] = m->mats[(size_t)l * BN_MATS + j].w_scale;
        }
        hl[l].norm = m->norms + (size_t)l * (3 * E + F);
    }
    WL_CUDA(cudaMalloc(&m->d_layers, hl.size() * sizeof(MegaLayer)));
    WL_CUDA(cudaMemcpy(m->d_layers, hl.data(), hl.size() * sizeof(MegaLayer), cudaMemcpyHostToDevice));
    WL_CUDA(cudaMemset(m->mega_state, 0, 64));
    uint32_t *status = status_ptr();
    if (!status) return WL_ERR_NO_DEVICE;
    p.layers = m->d_layers;
    p.n_layers = c.n_layers;
    p.E = E;
    p.F = F;
    p.KV = KV;
    p.HD = HD;
    p.n_heads = c.n_heads;
    p.group = c.n_heads / c.n_kv_heads;
    p.n_rot = c.n_rot;
    p.max_seq = c.max_seq;
    p.splits = S;
    p.eps = c.eps;
    p.scale = 1.0f / sqrtf((float)HD);  // attention_scale, primitives.rs:354
    p.exact = c.exact;
    p.q6k = m->q6k;
    p.nb = E / 256u;
    p.q6k_stride = q6k_row_stride(E / 256u);
    p.token = m->d_token;
    p.ids = nullptr;
    p.step = m->d_step;
    p.hidden = m->hidden;
    p.qkv = m->q;
    p.gu = m->gate;
    p.att = m->att_g;
    p.final_h = m->final_h;
    p.partial = m->attn_partial;
    p.out_norm = m->out_norm;
    p.kq = m->kq;
    p.vq = m->vq;
    p.ks = m->ks;
    p.vs = m->vs;
    p.rope = m->rope;
    p.pos = m->d_pos;
    p.arrivals = reinterpret_cast<unsigned long long *>(m->mega_state);
    p.launches = reinterpret_cast<uint32_t *>(m->mega_state) + 2;
    p.abort = reinterpret_cast<uint32_t *>(m->mega_state) + 3;
    p.status = status;
    m->mega_c3 = c3;
    m->mega = true;
    return WL_OK;
}

int bn_enqueue_mega(wl_bitnet *m, cudaStream_t s, bool commit) {
    MegaParams p = m->mp;
    p.ids = commit ? m->d_ids : nullptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m->mega_grid);
    cfg.blockDim = dim3(MEGA_THREADS);
    cfg.dynamicSmemBytes = m->mega_smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (m->mega_c3) WL_CUDA(cudaLaunchKernelEx(&cfg, bitnet_mega_kernel<true>, p));
    else WL_CUDA(cudaLaunchKernelEx(&cfg, bitnet_mega_kernel<false>, p));
    return WL_OK;
}

int bn_enqueue_forward(wl_bitnet *m, cudaStream_t s, bool commit) {
    if (m->mega) return bn_enqueue_mega(m, s, commit);
    const wl_bitnet_config &c = m->cfg;
    const uint32_t E = c.n_embd, F = c.n_ff, KV = bn_kv(c), nb = E / 256u;
    uint32_t *status = status_ptr();
    if (!status) return WL_ERR_NO_DEVICE;
    EmbedParams ep;
    ep.packed = m->q6k;
    ep.nb = nb;
    ep.row_stride = q6k_row_stride(nb);
    ep.token = m->d_token;
    ep.hidden = m->hidden;
    ep.ids = commit ? m->d_ids : nullptr;
    ep.step = m->d_step;
    WL_CUDA(launch(embed_q6k_kernel, dim3(nb), dim3(256), 0, s, true, ep));
    const uint32_t group = c.n_heads / c.n_kv_heads;
    const size_t attn_smem = m->gqa_attn     ? attn_gqa_smem_bytes(KV, c.head_dim, group, m->attn_chunk)
                             : m->exact_attn ? attn_exact_smem_bytes(KV, c.head_dim, c.max_seq)
                                             : attn_smem_bytes(KV, c.head_dim, c.max_seq, m->splits,
                                                               c.kv_f16 != 0);
    const float scale = 1.0f / sqrtf((float)c.head_dim);  // attention_scale, primitives.rs:354
    int rc;
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        const float *nrm = m->norms + (size_t)l * (3 * E + F);
        float *qkv[3] = {m->q, m->k, m->v};
        if ((rc = bn_matvec(m, l, 0, 3, E, m->hidden, qkv, I2S_PRE_RMSNORM, nrm, nullptr, 0, 0, s,
                            true)))
            return rc;
        AttnParams ap{};  // one sequence: no batch strides, NEOX pairs
        ap.q = m->q;
        ap.k = m->k;
        ap.v = m->v;
        ap.att = m->att;
        const size_t kv_esz = c.kv_f16 ? 2u : 1u;  // bytes per cached element
        ap.k_cache = m->kq + (size_t)l * c.max_seq * KV * kv_esz;
        ap.v_cache = m->vq + (size_t)l * c.max_seq * KV * kv_esz;
        ap.k_scale = m->ks + (size_t)l * c.max_seq;
        ap.v_scale = m->vs + (size_t)l * c.max_seq;
        ap.rope = m->rope;
        ap.pos = m->d_pos;
        ap.n_kv_heads = c.n_kv_heads;
        ap.head_dim = c.head_dim;
        ap.n_rot = c.n_rot;
        ap.max_seq = c.max_seq;
        ap.group = c.n_heads / c.n_kv_heads;
        ap.scale = scale;
        ap.splits = m->splits;
        ap.partial = m->attn_partial;
        ap.counters = m->attn_counters;
        ap.status = status;
        ap.exact = c.exact;
        if (m->tpg) {  // q / k / v were gathered from every rank
            ap.tp = m->tp;
            ap.tp.wait = 1u;
        }
        if (m->gqa_attn) {
            ap.chunk = m->attn_chunk;
            WL_CUDA(launch(gqa_attn_kernel(c.head_dim, group), dim3(c.n_kv_heads, 1, m->splits),
                           dim3(AB_THREADS), attn_smem, s, true, ap));
        } else if (m->exact_attn) {
            ap.pos_stable = 1u;  // the position advances only at the end of a step
            WL_CUDA(launch(attn_exact_kernel, dim3(c.n_heads, 1, 1), dim3(AX_THREADS), attn_smem, s,
                           true, ap));
        } else {
            WL_CUDA(launch(c.kv_f16 ? attn_decode_kernel<true> : attn_decode_kernel<false>,
                           dim3(c.n_heads, m->splits), dim3(ATTN_THREADS),
                           attn_smem, s, true, ap));
        }
        float *o[1] = {m->hidden};
        if ((rc = bn_matvec(m, l, 3, 1, E, m->att, o, I2S_PRE_RMSNORM, nrm + E, nullptr, 1, 0, s)))
            return rc;
        float *gu[2] = {m->gate, m->up};
        if ((rc = bn_matvec(m, l, 4, 2, E, m->hidden, gu, I2S_PRE_RMSNORM, nrm + 2 * E, nullptr, 0,
                            0, s, true)))
            return rc;
        if ((rc = bn_matvec(m, l, 6, 1, F, m->gate, o, I2S_PRE_RELU2_RMSNORM, nrm + 3 * E, m->up, 1,
                            WL_DEV_ERR_NONFINITE, s, true)))
            return rc;
    }
    if (m->tpg) {  // the final hidden was gathered by the last down projection
        TpParams tp = m->tp;
        tp.wait = 1u;
        tp_wait_kernel<<<1, 32, 0, s>>>(tp, status);
        WL_CUDA(cudaGetLastError());
    }
    OutNormParams op;
    op.hidden = m->hidden;
    op.w = m->out_norm;
    op.out = m->final_h;
    op.n = E;
    op.eps = c.eps;
    op.pos = m->d_pos;
    op.exact = c.exact;
    WL_CUDA(launch(out_norm_kernel, dim3(1), dim3(256), 0, s, true, op));
    return WL_OK;
}

// Greedy head on final_h -> *d_token (lm_head.rs:29-108 + :161-174).
int bn_enqueue_head(wl_bitnet *m, cudaStream_t s) {
    if (m->tpg) {  // this rank's vocab shard, keys reduced across ranks
        uint32_t *status = status_ptr();
        if (!status) return WL_ERR_NO_DEVICE;
        TpParams tp = m->tp;
        tp.wait = 0u;
        const uint8_t *shard = m->q6k + (size_t)m->vocab_off * q6k_row_stride(m->cfg.n_embd / 256u);
        int rc = launch_q6k_tp(shard, m->cfg.n_embd, m->vocab_shard, m->vocab_off, m->final_h, 1,
                               m->d_token, m->lm_scratch, s, &tp);
        if (rc) return rc;
        q6k_tp_finalize_kernel<<<1, 64, 0, s>>>(tp, 1, m->d_token, status);
        WL_CUDA(cudaGetLastError());
        return WL_OK;
    }
    return launch_q6k(m->q6k, m->cfg.n_embd, m->cfg.vocab, m->final_h, 1, nullptr, m->d_token,
                      m->lm_scratch, s, true);
}

int bn_capture(wl_bitnet *m, int which, cudaGraphExec_t *out) {
    cudaGraph_t g = nullptr;
    WL_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int rc = WL_OK;
    if (which == 0) {
        rc = bn_enqueue_forward(m, m->stream, false);
    } else if (which == 1) {
        rc = bn_enqueue_head(m, m->stream);
        if (!rc) rc = bn_enqueue_forward(m, m->stream, true);
    } else {
        rc = bn_enqueue_head(m, m->stream);
        if (!rc) {
            // commit the last id without running its forward: the embedding
            // kernel appends it (writing hidden, which nothing reads next)
            EmbedParams ep;
            const uint32_t nb = m->cfg.n_embd / 256u;
            ep.packed = m->q6k;
            ep.nb = nb;
            ep.row_stride = q6k_row_stride(nb);
            ep.token = m->d_token;
            ep.hidden = m->hidden;
            ep.ids = m->d_ids;
            ep.step = m->d_step;
            if (launch(embed_q6k_kernel, dim3(nb), dim3(256), 0, m->stream, true, ep) !=
                cudaSuccess)
                rc = fail(WL_ERR_CUDA, "embedding launch failed");
        }
    }
    cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return fail(WL_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(WL_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
    return WL_OK;
}

// Device status after a synchronised run: a non-finite hidden is the
// reference's GgufParse error (cached_forward.rs:507-517).
int bn_check_status(wl_bitnet *m) {
    Ctx &c = ctx();
    WL_CUDA(cudaStreamSynchronize(m->stream));
    uint32_t f = 0;
    WL_CUDA(cudaMemcpy(&f, c.d_status, 4, cudaMemcpyDeviceToHost));
    if (!f) return WL_OK;
    WL_CUDA(cudaMemset(c.d_status, 0, 4));
    if ((f & WL_DEV_ERR_MEGA) && m->mega_state)  // the grid stopped early: re-arm its barriers
        WL_CUDA(cudaMemset(m->mega_state, 0, 64));
    if (f & WL_DEV_ERR_NONFINITE)
        return fail(WL_ERR_GGUF_PARSE, "forward_with_cache: non-finite hidden after a layer");
    if (f & WL_DEV_ERR_POSITION) return fail(WL_ERR_GGUF_PARSE, "KV cache is full");
    return fail(WL_ERR_DEVICE_TIMEOUT, "device status %#x", f);
}

int bn_forward_token(wl_bitnet *m, uint32_t token) {
    *m->h_pinned = token;
    WL_CUDA(cudaMemcpyAsync(m->d_token, m->h_pinned, 4, cudaMemcpyHostToDevice, m->stream));
    if (!m->g_forward) {
        int rc = bn_capture(m, 0, &m->g_forward);
        if (rc) return rc;
    }
    WL_CUDA(cudaGraphLaunch(m->g_forward, m->stream));
    m->pos += 1;
    m->have_hidden = true;
    return WL_OK;
}

}  // namespace

// ===================================================================== C ABI
extern "C" {

const char *wl_version(void) { return "willamette_b200 0.1.0 (sm_100a)"; }

const char *wl_last_error(void) { return g_last_error.c_str(); }

uint32_t wl_last_error_tensor_type(void) { return g_last_type; }

int wl_init(int device) {
    Ctx &c = ctx();
    std::lock_guard<std::mutex> g(c.mu);
    if (c.inited && c.device != device)
        return fail(WL_ERR_INVALID_ARGUMENT, "already initialised on device %d", c.device);
    return init_locked(c, device);
}

int wl_release_weights(void) {
    Ctx &c = ctx();
    std::lock_guard<std::mutex> g(c.mu);
    for (auto &kv : c.cache) {
        cudaFree(kv.second.dptr);
        if (kv.second.ternary) cudaFree(kv.second.ternary);
    }
    c.cache.clear();
    return WL_OK;
}

int wl_device_status(uint32_t *flags) {
    // The allocation-free entry point keeps its status word in its static
    // array, on the caller's current device: read it first (no allocation),
    // and without initialising the library if only that entry point has run.
    uint32_t na = 0;
    int rc = noalloc_take_status(&na);
    if (rc) return rc;
    Ctx &c = ctx();
    std::lock_guard<std::mutex> g(c.mu);
    bool noalloc_used = false;
    {
        uint8_t *scratch = nullptr;
        noalloc_used = noalloc_setup(&scratch, false) == WL_OK && scratch != nullptr;
    }
    if (!c.inited && noalloc_used) {
        if (flags) *flags = na;
        return WL_OK;
    }
    rc = ensure_init(c);
    if (rc) return rc;
    uint32_t f = 0;
    // Kernels of every stream (library and caller streams) must have finished.
    WL_CUDA(cudaDeviceSynchronize());
    WL_CUDA(cudaMemcpy(&f, c.d_status, 4, cudaMemcpyDeviceToHost));
    WL_CUDA(cudaMemset(c.d_status, 0, 4));
    WL_CUDA(cudaDeviceSynchronize());
    if (flags) *flags = f | na;
    return WL_OK;
}

int wl_set_wait_limit_ns(uint64_t ns) {
    if (ns < 1000ull || ns > 600000000000ull)
        return fail(WL_ERR_INVALID_ARGUMENT, "wait limit %llu ns outside [1 us, 600 s]",
                    (unsigned long long)ns);
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
        return fail(WL_ERR_NO_DEVICE, "no CUDA device visible");
    WL_CUDA(cudaDeviceSynchronize());  // no kernel reads the old value mid-wait
    WL_CUDA(cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns)));
    return WL_OK;
}

int wl_dev_wait_flag(const uint32_t *flag, uint32_t target, void *stream) {
    if (!flag) return fail(WL_ERR_INVALID_ARGUMENT, "NULL flag");
    if (reinterpret_cast<uintptr_t>(flag) & 3u)
        return fail(WL_ERR_INVALID_ARGUMENT, "flag not 4-byte aligned");
    uint32_t *status = status_ptr();
    if (!status) return WL_ERR_NO_DEVICE;
    wait_flag_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(flag, target, status);
    WL_CUDA(cudaGetLastError());
    return WL_OK;
}

int wl_bitlinear_i2s_matvec_f32(const wl_tensor_view *weight, const float *input,
                                size_t input_len, float *output, size_t output_len) {
    return i2s_host_call(weight, input, input_len, output, output_len, 1, nullptr, nullptr,
                         nullptr);
}

int wl_bitlinear_i2s_matvec_f32_dbg(const wl_tensor_view *weight, const float *input,
                                    size_t input_len, float *output, size_t output_len,
                                    int32_t *acc_out, float *act_scale_out, int8_t *act_q_out) {
    return i2s_host_call(weight, input, input_len, output, output_len, 1, acc_out, act_scale_out,
                         act_q_out);
}

int wl_bitlinear_i2s_matvec_f32_kernel(const wl_tensor_view *weight, const float *input,
                                       size_t input_len, float *output, size_t output_len,
                                       uint32_t kernel) {
    switch (kernel) {
        case WL_I2S_KERNEL_SSE2_I8:
            return i2s_host_call(weight, input, input_len, output, output_len, 1, nullptr,
                                 nullptr, nullptr);
        case WL_I2S_KERNEL_SCALAR:
        case WL_I2S_KERNEL_SSE2_F32:
        case WL_I2S_KERNEL_SCALAR_LUT:
            return i2s_f32act_host_call(weight, input, input_len, output, output_len, kernel);
        case WL_I2S_KERNEL_NEON:
            return fail(WL_ERR_NOT_IMPLEMENTED,
                        "bitlinear_i2s_matvec_f32: the aarch64 NEON kernel has no GPU arm; keep "
                        "the CPU kernel");
        default:
            return fail(WL_ERR_INVALID_ARGUMENT, "unknown I2_S kernel %u", kernel);
    }
}

int wl_dev_i2s_matvec_f32act(const uint8_t *packed, float w_scale, uint32_t in_dim,
                             uint32_t out_dim, const float *x, float *y, uint32_t kernel,
                             void *stream) {
    if (in_dim == 0 || in_dim % 128)
        return fail(WL_ERR_GGUF_PARSE, "in_dim %u is not a positive multiple of 128", in_dim);
    if (!std::isfinite(w_scale))
        return fail(WL_ERR_GGUF_PARSE, "i2s_scale: non-finite scale (%g)", w_scale);
    if (kernel != WL_I2S_KERNEL_SCALAR && kernel != WL_I2S_KERNEL_SSE2_F32 &&
        kernel != WL_I2S_KERNEL_SCALAR_LUT)
        return fail(WL_ERR_INVALID_ARGUMENT, "kernel %u is not an f32-activation kernel", kernel);
    if (out_dim == 0) return WL_OK;
    if (!packed || !x || !y) return fail(WL_ERR_INVALID_ARGUMENT, "NULL pointer");
    if (!aligned16(packed) || !aligned16(x))
        return fail(WL_ERR_INVALID_ARGUMENT, "packed / x not 16-byte aligned");
    if (!status_ptr()) return WL_ERR_NO_DEVICE;
    return launch_i2s_f32act(packed, w_scale, in_dim, out_dim, x, y, kernel, (cudaStream_t)stream,
                             true);
}

int wl_bitlinear_i2s_gemm_f32(const wl_tensor_view *weight, const float *input, size_t m,
                              float *output, int32_t *acc_out) {
    return i2s_host_call(weight, input, 0, output, 0, m, acc_out, nullptr, nullptr);
}

int wl_linear_matvec_f32(const wl_tensor_view *weight, const float *input, size_t input_len,
                         float *output, size_t output_len) {
    if (!weight) return fail(WL_ERR_INVALID_ARGUMENT, "weight is NULL");
    const uint32_t ty = weight->ggml_type;
    if (ty == WL_GGML_I2_S)
        return wl_bitlinear_i2s_matvec_f32(weight, input, input_len, output, output_len);
    if (ty == WL_GGML_F16 || ty == WL_GGML_Q4_0 || ty == WL_GGML_Q4_K)
        return fail(WL_ERR_NOT_IMPLEMENTED, "linear_matvec_f32: raw type %u is not on the B200 path",
                    ty);
    if (ty != WL_GGML_Q6_K && ty != WL_GGML_Q8_0) return fail_type(ty);
    // quantized_matvec_f32 / q8_0_matvec_f32 validation (linear.rs:59-114, :171-213).
    const char *nm = ty == WL_GGML_Q6_K ? "Q6_K" : "Q8_0";
    if (weight->n_dims != 2 || !weight->shape)
        return fail(WL_ERR_GGUF_PARSE, "%s linear \"%s\": expected 2 dimensions", nm,
                    tname(weight));
    const uint64_t K = weight->shape[0], N = weight->shape[1];
    if (input_len != K || output_len != N)
        return fail(WL_ERR_GGUF_PARSE, "%s linear \"%s\": input/output lengths %zu/%zu != %llu/%llu",
                    nm, tname(weight), input_len, output_len, (unsigned long long)K,
                    (unsigned long long)N);
    uint64_t row_bytes = 0;
    if (K != 0) {
        int rc = row_bytes_for(ty, K, &row_bytes);
        if (rc) return rc;
    }
    if (weight->data_len != row_bytes * N)
        return fail(WL_ERR_GGUF_PARSE, "%s linear \"%s\": data length %zu != expected %llu", nm,
                    tname(weight), weight->data_len, (unsigned long long)(row_bytes * N));
    if (N == 0) return WL_OK;
    if (K == 0) {
        for (uint64_t i = 0; i < N; ++i) output[i] = 0.0f;
        return WL_OK;
    }
    if (K > 0xFFFFFFFFull || N > 0xFFFFFFFFull)
        return fail(WL_ERR_INVALID_ARGUMENT, "tensor too large");
    return rows_host_call(weight, (uint32_t)K, (uint32_t)N, row_bytes, input, 1, output, nullptr);
}

int wl_compute_logits(const float *final_hidden, size_t hidden_len,
                      const wl_tensor_view *token_embd, uint32_t embedding_length,
                      uint32_t vocab_size, float *logits, size_t logits_len) {
    uint64_t row_bytes = 0;
    int rc = validate_lm_head(final_hidden, hidden_len, token_embd, embedding_length, vocab_size,
                              &row_bytes);
    if (rc) return rc;
    if (logits_len != vocab_size)
        return fail(WL_ERR_INVALID_ARGUMENT, "logits_len %zu != vocab_size %u", logits_len,
                    vocab_size);
    if (embedding_length == 0) {
        for (uint32_t v = 0; v < vocab_size; ++v) logits[v] = 0.0f;
        return WL_OK;
    }
    return rows_host_call(token_embd, embedding_length, vocab_size, row_bytes, final_hidden, 1,
                          logits, nullptr);
}

int wl_argmax(const float *logits, size_t len, int64_t *out_id) {
    if (!out_id) return fail(WL_ERR_INVALID_ARGUMENT, "out_id is NULL");
    if (len == 0) {
        *out_id = -1;
        return WL_OK;
    }
    if (!logits) return fail(WL_ERR_INVALID_ARGUMENT, "logits is NULL");
    if (len > 0xFFFFFFFEull) return fail(WL_ERR_INVALID_ARGUMENT, "logits too long");
    Ctx &c = ctx();
    std::lock_guard<std::mutex> g(c.mu);
    int rc = ensure_init(c);
    if (rc) return rc;
    if ((rc = grow(c.x, len * 4)) || (rc = grow(c.ids, 16)) ||
        (rc = grow(c.scratch, wl_q6k_scratch_bytes(1))) || (rc = grow_pinned(c, len * 4 + 64)))
        return rc;
    memcpy(c.pinned, logits, len * 4);
    WL_CUDA(cudaMemcpyAsync(c.x.p, c.pinned, len * 4, cudaMemcpyHostToDevice, c.stream));
    auto *slot = (unsigned long long *)c.scratch.p;
    const uint32_t n = (uint32_t)len;
    const uint32_t grid = std::min<uint32_t>((n + ARGMAX_THREADS - 1) / ARGMAX_THREADS,
                                             (uint32_t)c.sm_count * 2u);
    WL_CUDA(launch(argmax_kernel, dim3(grid), dim3(ARGMAX_THREADS), 0, c.stream, false,
                   (const float *)c.x.p, n, slot, (uint32_t *)(slot + 1), (uint32_t *)c.ids.p));
    uint32_t *pid = (uint32_t *)((uint8_t *)c.pinned + len * 4);
    WL_CUDA(cudaMemcpyAsync(pid, c.ids.p, 4, cudaMemcpyDeviceToHost, c.stream));
    if ((rc = stage_status(c))) return rc;
    if ((rc = finish_call(c))) return rc;
    *out_id = (int64_t)*pid;
    return WL_OK;
}

int wl_lm_head_greedy(const float *hidden, size_t batch, const wl_tensor_view *token_embd,
                      uint32_t embedding_length, uint32_t vocab_size, uint32_t *token_ids,
                      float *logits) {
    uint64_t row_bytes = 0;
    int rc = validate_lm_head(hidden, embedding_length, token_embd, embedding_length, vocab_size,
                              &row_bytes);
    if (rc) return rc;
    if (!token_ids && batch) return fail(WL_ERR_INVALID_ARGUMENT, "token_ids is NULL");
    if (vocab_size == 0) return fail(WL_ERR_INVALID_ARGUMENT, "vocab_size is 0 (argmax of nothing)");
    if (batch > 65535) return fail(WL_ERR_INVALID_ARGUMENT, "batch %zu > 65535", batch);
    if (embedding_length == 0) {
        for (size_t b = 0; b < batch; ++b) token_ids[b] = 0;
        if (logits)
            for (size_t i = 0; i < batch * (size_t)vocab_size; ++i) logits[i] = 0.0f;
        return WL_OK;
    }
    return rows_host_call(token_embd, embedding_length, vocab_size, row_bytes, hidden, batch,
                          logits, token_ids);
}

int wl_dev_rms_norm_f32(const float *x, const float *w, uint32_t n, float eps, float *out,
                        void *stream) {
    if (n == 0) return WL_OK;
    if (n % 4 != 0 || n > WL_RMS_NORM_MAX_N)
        return fail(WL_ERR_INVALID_ARGUMENT, "rms_norm: n %u must be a multiple of 4 <= %u", n,
                    WL_RMS_NORM_MAX_N);
    if (!x || !w || !out) return fail(WL_ERR_INVALID_ARGUMENT, "NULL pointer");
    if (!aligned16(x) || !aligned16(w) || !aligned16(out))
        return fail(WL_ERR_INVALID_ARGUMENT, "x / w / out not 16-byte aligned");
    if (!status_ptr()) return WL_ERR_NO_DEVICE;
    WL_CUDA(launch(rms_norm_kernel, dim3(1), dim3(256),
                   (size_t)n * 4u + exact_sum_scratch_bytes(256), (cudaStream_t)stream, true, x, w,
                   n, eps, out));
    return WL_OK;
}

int wl_dev_softmax_f32(float *x, uint32_t n, void *stream) {
    if (n == 0) return WL_OK;
    if (n > WL_SOFTMAX_MAX_N)
        return fail(WL_ERR_INVALID_ARGUMENT, "softmax: n %u exceeds %u", n, WL_SOFTMAX_MAX_N);
    if (!x) return fail(WL_ERR_INVALID_ARGUMENT, "NULL pointer");
    if (!aligned16(x)) return fail(WL_ERR_INVALID_ARGUMENT, "x not 16-byte aligned");
    if (!status_ptr()) return WL_ERR_NO_DEVICE;
    WL_CUDA(launch(softmax_kernel, dim3(1), dim3(512),
                   (size_t)((n + 3u) & ~3u) * 4u + exact_sum_scratch_bytes(512),
                   (cudaStream_t)stream, true, x, n));
    return WL_OK;
}

int wl_dev_quantize_absmax_i8(const float *x, uint32_t n, uint32_t m, int8_t *q, float *act_scale,
                              void *stream) {
    if (n % 4 != 0) return fail(WL_ERR_INVALID_ARGUMENT, "n must be a multiple of 4");
    if (!aligned16(x) || !aligned16(q)) return fail(WL_ERR_INVALID_ARGUMENT, "x/q not 16-byte aligned");
    if (!status_ptr()) return WL_ERR_NO_DEVICE;
    return launch_quantize(x, n, m, q, act_scale, (cudaStream_t)stream, true);
}

int wl_dev_i2s_matvec(const wl_i2s_dev_weight *weights, uint32_t n_weights, uint32_t in_dim,
                      const int8_t *q, const float *act_scale, void *stream) {
    if (!weights || n_weights == 0 || n_weights > WL_I2S_MAX_FUSED)
        return fail(WL_ERR_INVALID_ARGUMENT, "n_weights must be 1..%d", WL_I2S_MAX_FUSED);
    if (in_dim == 0 || in_dim % 128 || in_dim > WL_I2S_MAX_IN_DIM)
        return fail(WL_ERR_GGUF_PARSE, "in_dim %u is not a positive multiple of 128 <= %u", in_dim,
                    WL_I2S_MAX_IN_DIM);
    if (!aligned16(q)) return fail(WL_ERR_INVALID_ARGUMENT, "q not 16-byte aligned");
    uint64_t rows = 0;
    for (uint32_t j = 0; j < n_weights; ++j) {
        if (!aligned16(weights[j].packed))
            return fail(WL_ERR_INVALID_ARGUMENT, "weight %u not 16-byte aligned", j);
        rows += weights[j].out_dim;
    }
    if (rows > 0x7FFFFFFFull) return fail(WL_ERR_INVALID_ARGUMENT, "too many rows");
    I2sLaunch L;
    L.w = weights;
    L.nw = n_weights;
    L.K = in_dim;
    L.q = q;
    L.act_scale = act_scale;
    return launch_i2s(L, (cudaStream_t)stream, true);
}

int wl_dev_i2s_matvec_fused_f32(const wl_i2s_dev_weight *weights, uint32_t n_weights,
                                uint32_t in_dim, const float *x, void *stream) {
    if (!weights || n_weights == 0 || n_weights > WL_I2S_MAX_FUSED)
        return fail(WL_ERR_INVALID_ARGUMENT, "n_weights must be 1..%d", WL_I2S_MAX_FUSED);
    if (in_dim == 0 || in_dim % 128 || in_dim > I2S_FUSE_Q_MAX_K)
        return fail(WL_ERR_GGUF_PARSE, "in_dim %u is not a positive multiple of 128 <= %u", in_dim,
                    I2S_FUSE_Q_MAX_K);
    if (!aligned16(x)) return fail(WL_ERR_INVALID_ARGUMENT, "x not 16-byte aligned");
    for (uint32_t j = 0; j < n_weights; ++j) {
        if (!aligned16(weights[j].packed))
            return fail(WL_ERR_INVALID_ARGUMENT, "weight %u not 16-byte aligned", j);
        if (!std::isfinite(weights[j].w_scale))
            return fail(WL_ERR_GGUF_PARSE, "i2s_scale: non-finite scale for weight %u", j);
    }
    I2sLaunch L;
    L.w = weights;
    L.nw = n_weights;
    L.K = in_dim;
    L.x = x;
    return launch_i2s(L, (cudaStream_t)stream, true);
}

int wl_dev_i2s_scan_code3(const uint8_t *packed, size_t bytes, uint32_t *found, void *stream) {
    if (!aligned16(packed) || bytes % 16)
        return fail(WL_ERR_INVALID_ARGUMENT, "packed must be 16-byte aligned, bytes a multiple of 16");
    if (!status_ptr()) return WL_ERR_NO_DEVICE;
    cudaStream_t s = (cudaStream_t)stream;
    WL_CUDA(cudaMemsetAsync(found, 0, 4, s));
    if (bytes == 0) return WL_OK;
    const size_t n16 = bytes / 16;
    const uint32_t grid = (uint32_t)std::min<size_t>((n16 + 255) / 256, 2048);
    i2s_scan_code3_kernel<<<grid, 256, 0, s>>>((const uint4 *)packed, n16, found);
    WL_CUDA(cudaGetLastError());
    return WL_OK;
}

int wl_dev_i2s_matvec_f32(const uint8_t *packed, float w_scale, uint32_t in_dim,
                          uint32_t out_dim, const float *x, float *y, int8_t *q_scratch,
                          float *scale_scratch, void *stream) {
    if (in_dim == 0 || in_dim % 128 || in_dim > WL_I2S_MAX_IN_DIM)
        return fail(WL_ERR_GGUF_PARSE, "in_dim %u is not a positive multiple of 128 <= %u", in_dim,
                    WL_I2S_MAX_IN_DIM);
    if (!std::isfinite(w_scale))
        return fail(WL_ERR_GGUF_PARSE, "i2s_scale: non-finite scale (%g)", w_scale);
    wl_i2s_dev_weight w = {packed, w_scale, out_dim, y, nullptr, 0};
    if (in_dim <= I2S_FUSE_Q_MAX_K) {
        if (!aligned16(x)) return fail(WL_ERR_INVALID_ARGUMENT, "x not 16-byte aligned");
        if (!aligned16(packed)) return fail(WL_ERR_INVALID_ARGUMENT, "packed not 16-byte aligned");
        if (q_scratch && !aligned16(q_scratch))
            return fail(WL_ERR_INVALID_ARGUMENT, "q_scratch not 16-byte aligned");
        I2sLaunch L;
        L.w = &w;
        L.nw = 1;
        L.K = in_dim;
        L.x = x;
        L.q_out = q_scratch;
        L.scale_out = scale_scratch;
        return launch_i2s(L, (cudaStream_t)stream, true);
    }
    int rc = wl_dev_quantize_absmax_i8(x, in_dim, 1, q_scratch, scale_scratch, stream);
    if (rc) return rc;
    return wl_dev_i2s_matvec(&w, 1, in_dim, q_scratch, scale_scratch, stream);
}

size_t wl_q6k_packed_bytes(uint32_t n_embd, uint32_t vocab) {
    return (size_t)q6k_row_stride(n_embd / 256u) * vocab;
}

int wl_dev_q6k_repack(const uint8_t *raw, uint32_t n_embd, uint32_t vocab, uint8_t *packed,
                      void *stream) {
    if (n_embd == 0 || n_embd % 256) return fail(WL_ERR_GGUF_PARSE, "Q6_K row length %u", n_embd);
    const size_t total = (size_t)vocab * (n_embd / 256u);
    if (total == 0) return WL_OK;
    const uint32_t grid = (uint32_t)std::min<size_t>((total + 255) / 256, 4096);
    q6k_repack_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(raw, n_embd / 256u, vocab, packed);
    WL_CUDA(cudaGetLastError());
    return WL_OK;
}

size_t wl_q6k_scratch_bytes(uint32_t batch) { return (size_t)batch * 8u + 16u; }

int wl_dev_q6k_lm_head(const uint8_t *packed, uint32_t n_embd, uint32_t vocab, const float *hidden,
                       uint32_t batch, float *logits, uint32_t *ids, void *scratch,
                       void *stream) {
    if (n_embd == 0 || n_embd % 256) return fail(WL_ERR_GGUF_PARSE, "Q6_K row length %u", n_embd);
    if (!aligned16(packed) || !scratch || ((uintptr_t)scratch & 7u))
        return fail(WL_ERR_INVALID_ARGUMENT, "packed must be 16-byte and scratch 8-byte aligned");
    return launch_q6k(packed, n_embd, vocab, hidden, batch, logits, ids, scratch,
                      (cudaStream_t)stream, true);
}

size_t wl_q8_0_packed_bytes(uint32_t in_dim, uint32_t out_dim) {
    return (size_t)q8_row_stride(in_dim) * out_dim;
}

int wl_dev_q8_0_repack(const uint8_t *raw, uint32_t in_dim, uint32_t out_dim, uint8_t *packed,
                       void *stream) {
    if (in_dim == 0 || in_dim % 32) return fail(WL_ERR_GGUF_PARSE, "Q8_0 row length %u", in_dim);
    const size_t total = (size_t)out_dim * (in_dim / 32u);
    if (total == 0) return WL_OK;
    const uint32_t grid = (uint32_t)std::min<size_t>((total + 255) / 256, 4096);
    q8_0_repack_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(raw, in_dim, out_dim, packed);
    WL_CUDA(cudaGetLastError());
    return WL_OK;
}

int wl_dev_q8_0_matvec(const uint8_t *packed, uint32_t in_dim, uint32_t out_dim, const float *x,
                       float *y, void *stream) {
    if (in_dim == 0 || in_dim % 32) return fail(WL_ERR_GGUF_PARSE, "Q8_0 row length %u", in_dim);
    if (!aligned16(packed)) return fail(WL_ERR_INVALID_ARGUMENT, "packed not 16-byte aligned");
    if (!status_ptr()) return WL_ERR_NO_DEVICE;
    return launch_q8(packed, in_dim, out_dim, x, y, (cudaStream_t)stream, true);
}

int wl_dev_i2s_matvec_f32_noalloc(const uint8_t *packed, float w_scale, uint32_t in_dim,
                                  uint32_t out_dim, const float *x, float *y, void *stream) {
    if (in_dim == 0 || in_dim % 128)
        return fail(WL_ERR_GGUF_PARSE, "in_dim %u is not a positive multiple of 128", in_dim);
    if (in_dim > WL_NOALLOC_MAX_IN_DIM)
        return fail(WL_ERR_INVALID_ARGUMENT,
                    "wl_dev_i2s_matvec_f32_noalloc: in_dim %u exceeds the static scratch "
                    "(WL_NOALLOC_MAX_IN_DIM = %u); use wl_dev_i2s_matvec_f32 with caller "
                    "buffers",
                    in_dim, WL_NOALLOC_MAX_IN_DIM);
    if (!std::isfinite(w_scale))
        return fail(WL_ERR_GGUF_PARSE, "i2s_scale: non-finite scale (%g)", w_scale);
    if (!x || !y || !packed) return fail(WL_ERR_INVALID_ARGUMENT, "NULL pointer");
    if (!aligned16(x) || !aligned16(packed))
        return fail(WL_ERR_INVALID_ARGUMENT, "x / packed not 16-byte aligned");
    if (out_dim == 0) return WL_OK;
    uint8_t *scratch = nullptr;
    int rc = noalloc_setup(&scratch);
    if (rc) return rc;
    float *act_scale = reinterpret_cast<float *>(scratch);
    uint32_t *status = reinterpret_cast<uint32_t *>(scratch + 4);
    int8_t *q = reinterpret_cast<int8_t *>(scratch + 256);
    cudaStream_t s = (cudaStream_t)stream;
    if ((rc = launch_quantize(x, in_dim, 1, q, act_scale, s, true))) return rc;
    wl_i2s_dev_weight w = {packed, w_scale, out_dim, y, nullptr, 0};
    I2sLaunch L;
    L.w = &w;
    L.nw = 1;
    L.K = in_dim;
    L.q = q;
    L.act_scale = act_scale;
    return launch_i2s_with_status(L, s, true, status);
}

int wl_i2s_stream_plan_create(const wl_i2s_stream_op *ops, uint32_t n_ops,
                              wl_i2s_stream_plan **plan) {
    if (!plan || (!ops && n_ops)) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    *plan = nullptr;
    if (n_ops == 0) return fail(WL_ERR_INVALID_ARGUMENT, "a stream plan needs at least one op");
    auto *p = new wl_i2s_stream_plan();
    int rc = build_stream_plan(ops, n_ops, p);
    if (rc) {
        if (p->d_block) cudaFree(p->d_block);
        delete p;
        return rc;
    }
    *plan = p;
    return WL_OK;
}

int wl_dev_i2s_stream_run(wl_i2s_stream_plan *plan, void *stream) {
    if (!plan) return fail(WL_ERR_INVALID_ARGUMENT, "plan is NULL");
    cudaStream_t s = (cudaStream_t)stream;
    WL_CUDA(launch(quantize_jobs_kernel, dim3(plan->n_quant), dim3(QUANT_THREADS), 0, s, true,
                   (const QuantJob *)plan->d_qjobs));
    I2sStreamParams p;
    p.ops = plan->d_ops;
    p.maps = plan->d_maps;
    p.n_ops = plan->n_ops;
    p.cta_blocks = plan->d_cta_blocks;
    p.status = plan->status;
    WL_CUDA(launch(kStream[plan->c3 ? 1 : 0], dim3(plan->grid), dim3(STREAM_THREADS),
                   STREAM_SMEM, s, true, p));
    return WL_OK;
}

int wl_i2s_stream_plan_destroy(wl_i2s_stream_plan *plan) {
    if (!plan) return WL_OK;
    if (plan->d_block) cudaFree(plan->d_block);
    delete plan;
    return WL_OK;
}

size_t wl_i2s_gemm_workspace_bytes(uint32_t m, uint32_t in_dim) {
    return (size_t)m * in_dim + 2u * (((size_t)m * 4u + 15u) & ~(size_t)15u) + 16u;
}

int wl_dev_i2s_gemm_f32(const uint8_t *packed, float w_scale, uint32_t in_dim, uint32_t out_dim,
                        uint32_t m, const float *x, float *y, int32_t *acc, void *workspace,
                        uint32_t flags, void *stream) {
    if (in_dim == 0 || in_dim % 128 || in_dim > WL_I2S_MAX_IN_DIM)
        return fail(WL_ERR_GGUF_PARSE, "in_dim %u is not a positive multiple of 128 <= %u", in_dim,
                    WL_I2S_MAX_IN_DIM);
    if (!std::isfinite(w_scale)) return fail(WL_ERR_GGUF_PARSE, "i2s_scale: non-finite scale");
    if (!packed || !x || !y || !workspace || !aligned16(packed) || !aligned16(x) ||
        !aligned16(workspace))
        return fail(WL_ERR_INVALID_ARGUMENT, "NULL or misaligned pointer");
    if (m == 0 || out_dim == 0) return WL_OK;
    uint32_t *status = status_ptr();
    if (!status) return WL_ERR_NO_DEVICE;
    cudaStream_t s = (cudaStream_t)stream;
    int8_t *q = (int8_t *)workspace;
    float *scale = (float *)((uint8_t *)workspace + (size_t)m * in_dim);
    int32_t *rowsum = (int32_t *)((uint8_t *)scale + (((size_t)m * 4u + 15u) & ~(size_t)15u));
    int rc;
    if (flags & WL_I2S_NO_CODE3) {
        if ((rc = launch_quantize(x, in_dim, m, q, scale, s, true, rowsum))) return rc;
        return launch_i2s_gemm(packed, w_scale, in_dim, out_dim, m, q, scale, rowsum, y, acc, s,
                               true, status);
    }
    // Weights that may hold code 0b11: one exact matvec per token.
    if ((rc = launch_quantize(x, in_dim, m, q, scale, s, true))) return rc;
    for (uint32_t t = 0; t < m; ++t) {
        wl_i2s_dev_weight w = {packed, w_scale, out_dim, y + (size_t)t * out_dim,
                               acc ? acc + (size_t)t * out_dim : nullptr, 0};
        I2sLaunch L;
        L.w = &w;
        L.nw = 1;
        L.K = in_dim;
        L.q = q + (size_t)t * in_dim;
        L.act_scale = scale + t;
        if ((rc = launch_i2s(L, s, true))) return rc;
    }
    return WL_OK;
}

size_t wl_i2s_expanded_bytes(uint32_t in_dim, uint32_t out_dim) {
    return (size_t)in_dim * out_dim;
}

int wl_dev_i2s_expand(const uint8_t *packed, uint32_t in_dim, uint32_t out_dim, int8_t *ternary,
                      void *stream) {
    if (in_dim == 0 || in_dim % 128 || in_dim > WL_I2S_MAX_IN_DIM)
        return fail(WL_ERR_GGUF_PARSE, "in_dim %u is not a positive multiple of 128 <= %u", in_dim,
                    WL_I2S_MAX_IN_DIM);
    if (!packed || !ternary || !aligned16(packed) || !aligned16(ternary))
        return fail(WL_ERR_INVALID_ARGUMENT, "NULL or misaligned pointer");
    if (!status_ptr()) return WL_ERR_NO_DEVICE;
    return launch_i2s_expand(packed, in_dim, out_dim, ternary, (cudaStream_t)stream);
}

int wl_dev_i2s_gemm_s8_f32(const int8_t *ternary, float w_scale, uint32_t in_dim,
                           uint32_t out_dim, uint32_t m, const float *x, float *y, int32_t *acc,
                           void *workspace, void *stream) {
    if (in_dim == 0 || in_dim % 128 || in_dim > WL_I2S_MAX_IN_DIM)
        return fail(WL_ERR_GGUF_PARSE, "in_dim %u is not a positive multiple of 128 <= %u", in_dim,
                    WL_I2S_MAX_IN_DIM);
    if (!std::isfinite(w_scale)) return fail(WL_ERR_GGUF_PARSE, "i2s_scale: non-finite scale");
    if (!ternary || !x || !y || !workspace || !aligned16(ternary) || !aligned16(x) ||
        !aligned16(workspace))
        return fail(WL_ERR_INVALID_ARGUMENT, "NULL or misaligned pointer");
    if (m == 0 || out_dim == 0) return WL_OK;
    uint32_t *status = status_ptr();
    if (!status) return WL_ERR_NO_DEVICE;
    cudaStream_t s = (cudaStream_t)stream;
    int8_t *q = (int8_t *)workspace;
    float *scale = (float *)((uint8_t *)workspace + (size_t)m * in_dim);
    int rc;
    if ((rc = launch_quantize(x, in_dim, m, q, scale, s, true))) return rc;
    return launch_i2s_gemm_s8(ternary, w_scale, in_dim, out_dim, m, q, scale, y, acc, s, true,
                              status);
}

// ------------------------------------------------------------ tensor parallel
int wl_tp_create(int rank, int world, size_t sym_bytes, wl_tp_group **group,
                 uint8_t *handle_out) {
    if (!group || !handle_out) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    *group = nullptr;
    if (world < 1 || world > TP_MAX_WORLD || rank < 0 || rank >= world)
        return fail(WL_ERR_INVALID_ARGUMENT, "rank %d / world %d (world must be 1..%d)", rank,
                    world, TP_MAX_WORLD);
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    int rc = ensure_init(c);
    if (rc) return rc;
    auto *g = new wl_tp_group();
    g->device = c.device;
    g->rank = rank;
    g->world = world;
    g->bytes = TP_HEADER_BYTES + ((sym_bytes + 255) & ~(size_t)255);
    cudaError_t e = cudaMalloc(&g->local, g->bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(g->local, 0, g->bytes, c.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c.stream);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, g->local);
    if (e != cudaSuccess) {
        if (g->local) cudaFree(g->local);
        delete g;
        return fail(WL_ERR_COMM, "symmetric block: %s", cudaGetErrorString(e));
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == WL_TP_HANDLE_BYTES, "IPC handle size");
    memcpy(handle_out, &h, WL_TP_HANDLE_BYTES);
    *group = g;
    return WL_OK;
}

int wl_tp_connect(wl_tp_group *g, const uint8_t *handles) {
    if (!g || !handles) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    if (g->connected) return WL_OK;
    cudaSetDevice(g->device);
    for (int r = 0; r < g->world; ++r) {
        if (r == g->rank) {
            g->peers[r] = g->local;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, handles + (size_t)r * WL_TP_HANDLE_BYTES, WL_TP_HANDLE_BYTES);
        void *ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return fail(WL_ERR_COMM, "opening rank %d's block: %s", r, cudaGetErrorString(e));
        g->peers[r] = (uint8_t *)ptr;
    }
    g->connected = true;
    return WL_OK;
}

void *wl_tp_buffer(wl_tp_group *g, size_t offset) {
    if (!g || TP_HEADER_BYTES + offset >= g->bytes) return nullptr;
    return g->local + TP_HEADER_BYTES + offset;
}

int wl_tp_destroy(wl_tp_group *g) {
    if (!g) return WL_OK;
    cudaSetDevice(g->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < g->world; ++r)
        if (r != g->rank && g->peers[r]) cudaIpcCloseMemHandle(g->peers[r]);
    if (g->local) cudaFree(g->local);
    delete g;
    return WL_OK;
}

int wl_tp_wait(wl_tp_group *g, void *stream) {
    TpParams tp;
    int rc = tp_params(g, true, &tp);
    if (rc) return rc;
    uint32_t *status = status_ptr();
    if (!status) return WL_ERR_NO_DEVICE;
    tp_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(tp, status);
    WL_CUDA(cudaGetLastError());
    return WL_OK;
}

int wl_tp_i2s_matvec_fused_f32(wl_tp_group *g, const wl_i2s_dev_weight *weights,
                               const uint32_t *row_offsets, uint32_t n_weights, uint32_t in_dim,
                               const float *x, int wait_for_input, void *stream) {
    if (!weights || !row_offsets || n_weights == 0 || n_weights > WL_I2S_MAX_FUSED)
        return fail(WL_ERR_INVALID_ARGUMENT, "n_weights must be 1..%d", WL_I2S_MAX_FUSED);
    if (in_dim == 0 || in_dim % 128 || in_dim > I2S_FUSE_Q_MAX_K)
        return fail(WL_ERR_GGUF_PARSE, "in_dim %u is not a positive multiple of 128 <= %u", in_dim,
                    I2S_FUSE_Q_MAX_K);
    if (!x || !aligned16(x)) return fail(WL_ERR_INVALID_ARGUMENT, "x NULL or misaligned");
    TpParams tp;
    int rc = tp_params(g, wait_for_input != 0, &tp);
    if (rc) return rc;
    for (uint32_t j = 0; j < n_weights; ++j) {
        if (!aligned16(weights[j].packed))
            return fail(WL_ERR_INVALID_ARGUMENT, "weight %u not 16-byte aligned", j);
        if (!std::isfinite(weights[j].w_scale))
            return fail(WL_ERR_GGUF_PARSE, "i2s_scale: non-finite scale for weight %u", j);
        if ((rc = check_sym_range(g, weights[j].y, (size_t)row_offsets[j] + weights[j].out_dim)))
            return rc;
        if (weights[j].acc) return fail(WL_ERR_INVALID_ARGUMENT, "acc is not gathered; pass NULL");
    }
    I2sLaunch L;
    L.w = weights;
    L.nw = n_weights;
    L.K = in_dim;
    L.x = x;
    L.tp = &tp;
    L.row_offs = row_offsets;
    return launch_i2s(L, (cudaStream_t)stream, true);
}

int wl_tp_i2s_stream_run(wl_tp_group *g, wl_i2s_stream_plan *plan, void *stream) {
    if (!plan) return fail(WL_ERR_INVALID_ARGUMENT, "plan is NULL");
    TpParams tp;
    int rc = tp_params(g, false, &tp);
    if (rc) return rc;
    if (plan->y_lo < (uintptr_t)(g->local + TP_HEADER_BYTES) ||
        plan->y_hi > (uintptr_t)(g->local + g->bytes))
        return fail(WL_ERR_INVALID_ARGUMENT, "stream plan outputs are not in the group's block");
    cudaStream_t s = (cudaStream_t)stream;
    WL_CUDA(launch(quantize_jobs_kernel, dim3(plan->n_quant), dim3(QUANT_THREADS), 0, s, true,
                   (const QuantJob *)plan->d_qjobs));
    I2sStreamParams p;
    p.ops = plan->d_ops;
    p.maps = plan->d_maps;
    p.n_ops = plan->n_ops;
    p.cta_blocks = plan->d_cta_blocks;
    p.status = plan->status;
    p.tp = tp;
    WL_CUDA(launch(kStream[plan->c3 ? 1 : 0], dim3(plan->grid), dim3(STREAM_THREADS),
                   STREAM_SMEM, s, true, p));
    return WL_OK;
}

int wl_tp_q6k_lm_head_greedy(wl_tp_group *g, const uint8_t *packed_shard, uint32_t n_embd,
                             uint32_t vocab_shard, uint32_t row_offset, const float *hidden,
                             uint32_t batch, uint32_t *ids, void *scratch, void *stream) {
    if (n_embd == 0 || n_embd % 256) return fail(WL_ERR_GGUF_PARSE, "Q6_K row length %u", n_embd);
    if (batch == 0 || batch > TP_MAX_BATCH)
        return fail(WL_ERR_INVALID_ARGUMENT, "batch must be 1..%u", TP_MAX_BATCH);
    if (!ids || !hidden || !aligned16(packed_shard) || !scratch || ((uintptr_t)scratch & 7u))
        return fail(WL_ERR_INVALID_ARGUMENT, "NULL or misaligned pointer");
    TpParams tp;
    int rc = tp_params(g, false, &tp);
    if (rc) return rc;
    uint32_t *status = status_ptr();
    if (!status) return WL_ERR_NO_DEVICE;
    cudaStream_t s = (cudaStream_t)stream;
    // every rank launches the same batch groups, so arrivals stay in step
    if ((rc = launch_q6k_tp(packed_shard, n_embd, vocab_shard, row_offset, hidden, batch, ids,
                            scratch, s, &tp)))
        return rc;
    q6k_tp_finalize_kernel<<<1, 64, 0, s>>>(tp, batch, ids, status);
    WL_CUDA(cudaGetLastError());
    return WL_OK;
}

// ------------------------------------------------------- BitNet decode engine
}  // extern "C"

namespace {

// Caller-region bytes of a tensor-parallel engine's symmetric buffers:
// hidden (E), q | k | v (E + 2 KV), gate | up (2 F), each 256-byte aligned.
size_t bn_sym_layout(const wl_bitnet_config &c, size_t *off_q, size_t *off_g) {
    auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t E = c.n_embd, KV = bn_kv(c), F = c.n_ff;
    *off_q = up(E * 4);
    *off_g = *off_q + up((E + 2 * KV) * 4);
    return *off_g + up(2 * F * 4);
}

int bn_create(const wl_bitnet_config *cfg, const wl_bitnet_weights *w, wl_tp_group *tpg,
              wl_bitnet **out) {
    if (!out) return fail(WL_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    int rc = bn_validate(cfg);
    if (rc) return rc;
    TpParams tpp{};
    if (tpg) {
        if ((rc = tp_params(tpg, false, &tpp))) return rc;
        if (cfg->persistent)
            return fail(WL_ERR_INVALID_ARGUMENT, "the persistent engine runs on one GPU only");
        size_t oq, og;
        const size_t need = bn_sym_layout(*cfg, &oq, &og);
        if (TP_HEADER_BYTES + need > tpg->bytes)
            return fail(WL_ERR_INVALID_ARGUMENT, "symmetric block too small: %zu bytes needed",
                        need);
        if (tpg->device != ctx().device)
            return fail(WL_ERR_INVALID_ARGUMENT, "group is on device %d, library on %d", tpg->device,
                        ctx().device);
    }
    const uint32_t world = tpg ? (uint32_t)tpg->world : 1u, rank = tpg ? (uint32_t)tpg->rank : 0u;
    // rank's slice [lo, hi) of n rows
    auto slice_lo = [&](uint32_t n) { return (uint32_t)((uint64_t)n * rank / world); };
    auto slice_hi = [&](uint32_t n) { return (uint32_t)((uint64_t)n * (rank + 1) / world); };
    if (!w || !w->w || !w->w_scale || !w->norms || !w->output_norm || !w->token_embd)
        return fail(WL_ERR_INVALID_ARGUMENT, "weights: NULL pointer");
    const wl_bitnet_config c = *cfg;
    const uint32_t E = c.n_embd, F = c.n_ff, KV = bn_kv(c);
    const uint32_t outs[BN_MATS] = {E, KV, KV, E, F, F, E};
    const uint32_t ins[BN_MATS] = {E, E, E, E, E, E, F};
    for (uint32_t i = 0; i < c.n_layers * BN_MATS; ++i)
        if (!w->w[i] || !std::isfinite(w->w_scale[i]))
            return fail(WL_ERR_GGUF_PARSE, "layer %u tensor %u: missing data or non-finite scale",
                        i / BN_MATS, i % BN_MATS);
    Ctx &cx = ctx();
    std::lock_guard<std::mutex> lk(cx.mu);
    if ((rc = ensure_init(cx))) return rc;
    auto *m = new wl_bitnet();
    m->cfg = c;
    m->device = cx.device;
    auto cleanup = [&](int code) {
        wl_bitnet_destroy(m);
        return code;
    };
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
        return cleanup(fail(WL_ERR_CUDA, "stream"));
    // packed I2_S weights, 256-byte aligned each
    size_t total = 0;
    std::vector<size_t> off(c.n_layers * BN_MATS);
    for (uint32_t i = 0; i < c.n_layers * BN_MATS; ++i) {
        off[i] = total;
        const uint32_t N = outs[i % BN_MATS];
        total += ((size_t)ins[i % BN_MATS] / 4 * (slice_hi(N) - slice_lo(N)) + 255) & ~(size_t)255;
    }
    total = std::max<size_t>(total, 256);
    const size_t nrm = (size_t)c.n_layers * (3 * E + F);
    const size_t q6_raw = (size_t)c.vocab * (E / 256) * 210;
    const size_t q6_packed = (size_t)c.vocab * q6k_row_stride(E / 256);
    const size_t kv_bytes = (size_t)c.n_layers * c.max_seq * KV * (c.kv_f16 ? 2u : 1u);
    const size_t kvs = (size_t)c.n_layers * c.max_seq;
    m->ids_cap = 1u << 16;
    void *p = nullptr;
#define BN_ALLOC(ptr, bytes)                                                         \
    do {                                                                             \
        if (cudaMalloc(&p, (bytes)) != cudaSuccess)                                  \
            return cleanup(fail(WL_ERR_CUDA, "out of device memory (%s)", #ptr));    \
        ptr = reinterpret_cast<decltype(ptr)>(p);                                    \
    } while (0)
    BN_ALLOC(m->wblock, total);
    BN_ALLOC(m->norms, nrm * 4);
    BN_ALLOC(m->out_norm, (size_t)E * 4);
    BN_ALLOC(m->q6k, q6_packed);
    BN_ALLOC(m->rope, (size_t)c.max_seq * (c.n_rot / 2) * sizeof(float2));
    BN_ALLOC(m->kq, kv_bytes);
    BN_ALLOC(m->vq, kv_bytes);
    BN_ALLOC(m->ks, kvs * 4);
    BN_ALLOC(m->vs, kvs * 4);
    if (tpg) {  // gathered vectors live in the group's symmetric block
        size_t oq, og;
        bn_sym_layout(c, &oq, &og);
        uint8_t *base = reinterpret_cast<uint8_t *>(wl_tp_buffer(tpg, 0));
        m->tpg = tpg;
        m->tp = tpp;
        m->hidden = reinterpret_cast<float *>(base);
        m->q = reinterpret_cast<float *>(base + oq);
        m->gate = reinterpret_cast<float *>(base + og);
    } else {
        BN_ALLOC(m->hidden, (size_t)E * 4);
        BN_ALLOC(m->q, (size_t)(E + 2 * KV) * 4);  // q | k | v, contiguous
        BN_ALLOC(m->gate, (size_t)2 * F * 4);       // gate | up, contiguous
    }
    m->k = m->q + E;
    m->v = m->k + KV;
    BN_ALLOC(m->att, (size_t)E * 4);
    m->up = m->gate + F;
    m->vocab_off = slice_lo(c.vocab);
    m->vocab_shard = slice_hi(c.vocab) - m->vocab_off;
    BN_ALLOC(m->att_g, (size_t)E * 4);
    BN_ALLOC(m->mega_state, 64);
    BN_ALLOC(m->final_h, (size_t)E * 4);
    BN_ALLOC(m->d_token, 16);
    BN_ALLOC(m->d_pos, 16);
    BN_ALLOC(m->d_step, 16);
    BN_ALLOC(m->d_ids, (size_t)m->ids_cap * 4);
    BN_ALLOC(m->lm_scratch, 256);
    // attention splits: about 2 CTAs per SM over all heads, at least 32
    // positions per split
    m->splits = c.exact ? 1u
                        : std::max<uint32_t>(1u, std::min<uint32_t>((c.max_seq + 31) / 32,
                                                                    (uint32_t)(2 * cx.sm_count) /
                                                                        c.n_heads));
    {   // fast mode: one CTA per (KV head, split of `chunk` positions) for the
        // whole query group, when the group and head size have a kernel
        const uint32_t group = c.n_heads / c.n_kv_heads;
        if (!c.exact && !c.kv_f16 && gqa_attn_kernel(c.head_dim, group) && c.n_rot % 4 == 0) {
            // 64 positions per CTA measured fastest at BitNet-2B shapes with a
            // 640-position cache (1309 us per token; 1359 at 32, 1334 at 128)
            uint32_t chunk = 64;
            while ((uint64_t)((c.max_seq + chunk - 1) / chunk) * c.n_kv_heads > (uint64_t)cx.sm_count ||
                   (c.max_seq + chunk - 1) / chunk > AB_COMBINE / group)
                chunk += 32;
            if (attn_gqa_smem_bytes(KV, c.head_dim, group, chunk) <= (size_t)WL_MAX_DYN_SMEM) {
                m->gqa_attn = true;
                m->attn_chunk = chunk;
                m->splits = (c.max_seq + chunk - 1) / chunk;
            }
        }
    }
    // exact mode: the whole history of a head in shared memory, when it fits
    m->exact_attn = c.exact && !c.kv_f16 &&
                    attn_exact_smem_bytes(KV, c.head_dim, c.max_seq) <=
                        kernel_dyn_cap((const void *)attn_exact_kernel);
    m->mega_grid = (uint32_t)cx.sm_count;
    m->mega_splits = c.exact ? 1u : std::max<uint32_t>(1u, m->mega_grid / c.n_heads);
    BN_ALLOC(m->attn_partial, (size_t)c.n_heads * std::max(m->splits, m->mega_splits) *
                                  (4 + c.head_dim) * 4);
    BN_ALLOC(m->attn_counters, (size_t)c.n_heads * 4);
#undef BN_ALLOC
    if (cudaMallocHost(&p, 64) != cudaSuccess) return cleanup(fail(WL_ERR_CUDA, "pinned"));
    m->h_pinned = (uint32_t *)p;
    cudaStream_t s = m->stream;
    uint8_t *q6raw = nullptr;
    if (cudaMalloc(&q6raw, q6_raw) != cudaSuccess) return cleanup(fail(WL_ERR_CUDA, "q6k staging"));
    cudaError_t e = cudaMemcpyAsync(q6raw, w->token_embd, q6_raw, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        q6k_repack_kernel<<<1024, 256, 0, s>>>(q6raw, E / 256, c.vocab, m->q6k);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(q6raw);
    if (e != cudaSuccess) return cleanup(fail(WL_ERR_CUDA, "embedding upload: %s", cudaGetErrorString(e)));
    std::vector<float2> rope;
    bn_rope_table(c, rope);
    m->mats.resize((size_t)c.n_layers * BN_MATS);
    m->row_offs.resize((size_t)c.n_layers * BN_MATS);
    uint32_t *found = cx.d_status + 8;
    for (uint32_t i = 0; i < c.n_layers * BN_MATS && e == cudaSuccess; ++i) {
        const uint32_t K = ins[i % BN_MATS], N0 = outs[i % BN_MATS];
        const uint32_t r0 = slice_lo(N0), N = slice_hi(N0) - r0;  // this rank's rows
        m->row_offs[i] = r0;
        const size_t bytes = (size_t)K / 4 * N;
        uint8_t *dst = m->wblock + off[i];
        if (bytes) e = cudaMemcpyAsync(dst, w->w[i] + (size_t)r0 * (K / 4), bytes, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaMemsetAsync(found, 0, 4, s);
        if (e == cudaSuccess && bytes >= 16) {
            const size_t n16 = bytes / 16;
            i2s_scan_code3_kernel<<<(unsigned)std::min<size_t>((n16 + 255) / 256, 2048), 256, 0, s>>>(
                (const uint4 *)dst, n16, found);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaMemcpyAsync(m->h_pinned, found, 4, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        wl_i2s_dev_weight &mw = m->mats[i];
        mw.packed = dst;
        mw.w_scale = w->w_scale[i];
        mw.out_dim = N;
        mw.y = nullptr;
        mw.acc = nullptr;
        mw.flags = *m->h_pinned ? 0u : WL_I2S_NO_CODE3;
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->norms, w->norms, nrm * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->out_norm, w->output_norm, (size_t)E * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->rope, rope.data(), rope.size() * sizeof(float2),
                            cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->lm_scratch, 0, 256, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->attn_counters, 0, (size_t)c.n_heads * 4, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->d_pos, 0, 16, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->d_step, 0, 16, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cleanup(fail(WL_ERR_CUDA, "weight upload: %s", cudaGetErrorString(e)));
    if (c.persistent && !c.kv_f16 && (rc = bn_setup_mega(m))) return cleanup(rc);
    *out = m;
    return WL_OK;
}

}  // namespace

extern "C" {

int wl_bitnet_create(const wl_bitnet_config *cfg, const wl_bitnet_weights *w, wl_bitnet **out) {
    return bn_create(cfg, w, nullptr, out);
}

int wl_bitnet_create_tp(const wl_bitnet_config *cfg, const wl_bitnet_weights *w,
                        wl_tp_group *group, wl_bitnet **out) {
    if (!group) return fail(WL_ERR_INVALID_ARGUMENT, "group is NULL");
    return bn_create(cfg, w, group, out);
}

size_t wl_bitnet_tp_sym_bytes(const wl_bitnet_config *cfg) {
    if (!cfg) return 0;
    size_t oq, og;
    return bn_sym_layout(*cfg, &oq, &og);
}

int wl_bitnet_destroy(wl_bitnet *m) {
    if (!m) return WL_OK;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->g_forward) cudaGraphExecDestroy(m->g_forward);
    if (m->g_step) cudaGraphExecDestroy(m->g_step);
    if (m->g_last) cudaGraphExecDestroy(m->g_last);
    if (m->tpg) {  // in the group's symmetric block, not ours
        m->hidden = nullptr;
        m->q = nullptr;
        m->gate = nullptr;
    }
    void *bufs[] = {m->wblock, m->norms, m->out_norm, m->q6k, m->rope, m->kq, m->vq, m->ks,
                    m->vs, m->hidden, m->q, m->att, m->gate, m->final_h, m->att_g,
                    m->mega_state, m->d_layers,
                    m->d_token, m->d_pos, m->d_step, m->d_ids, m->lm_scratch,
                    m->attn_partial, m->attn_counters};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (m->h_pinned) cudaFreeHost(m->h_pinned);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return WL_OK;
}

int wl_bitnet_reset(wl_bitnet *m) {
    if (!m) return fail(WL_ERR_INVALID_ARGUMENT, "model is NULL");
    cudaSetDevice(m->device);
    WL_CUDA(cudaMemsetAsync(m->d_pos, 0, 4, m->stream));
    WL_CUDA(cudaStreamSynchronize(m->stream));
    m->pos = 0;
    m->have_hidden = false;
    return WL_OK;
}

uint32_t wl_bitnet_position(const wl_bitnet *m) { return m ? m->pos : 0u; }

int wl_bitnet_uses_persistent_kernel(const wl_bitnet *m) { return m && m->mega ? 1 : 0; }


int wl_bitnet_forward(wl_bitnet *m, uint32_t token, uint32_t position, float *out_hidden) {
    if (!m) return fail(WL_ERR_INVALID_ARGUMENT, "model is NULL");
    if (m->pos != position)
        return fail(WL_ERR_GGUF_PARSE,
                    "forward_with_cache: cache.position()=%u != position=%u; tokens must be "
                    "processed in order", m->pos, position);
    if (position >= m->cfg.max_seq) return fail(WL_ERR_GGUF_PARSE, "KV cache is full");
    if (token >= m->cfg.vocab)
        return fail(WL_ERR_GGUF_PARSE, "forward_with_cache: token_id %u out of vocab range %u",
                    token, m->cfg.vocab);
    cudaSetDevice(m->device);
    int rc = bn_forward_token(m, token);
    if (rc) return rc;
    if ((rc = bn_check_status(m))) return rc;
    if (out_hidden)
        WL_CUDA(cudaMemcpy(out_hidden, m->final_h, (size_t)m->cfg.n_embd * 4, cudaMemcpyDeviceToHost));
    return WL_OK;
}

int wl_bitnet_prefill(wl_bitnet *m, const uint32_t *tokens, uint32_t n) {
    if (!m || (!tokens && n)) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    if ((uint64_t)m->pos + n > m->cfg.max_seq) return fail(WL_ERR_GGUF_PARSE, "KV cache is full");
    for (uint32_t i = 0; i < n; ++i)
        if (tokens[i] >= m->cfg.vocab)
            return fail(WL_ERR_GGUF_PARSE, "prompt token %u (idx %u) out of vocab range %u",
                        tokens[i], i, m->cfg.vocab);
    cudaSetDevice(m->device);
    for (uint32_t i = 0; i < n; ++i) {
        int rc = bn_forward_token(m, tokens[i]);
        if (rc) return rc;
        // the token staging word is reused: wait for its copy before the next
        WL_CUDA(cudaStreamSynchronize(m->stream));
    }
    return bn_check_status(m);
}

int wl_bitnet_decode(wl_bitnet *m, uint32_t n_new, uint32_t *out_ids, float *out_hiddens,
                     float *device_ms) {
    if (!m || (!out_ids && n_new)) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    if (!m->have_hidden) return fail(WL_ERR_INVALID_ARGUMENT, "decode needs a prefilled prompt");
    if (n_new == 0) return WL_OK;
    if (n_new > m->ids_cap) return fail(WL_ERR_INVALID_ARGUMENT, "n_new > %u", m->ids_cap);
    if ((uint64_t)m->pos + n_new - 1 > m->cfg.max_seq)
        return fail(WL_ERR_GGUF_PARSE, "KV cache is full");
    cudaSetDevice(m->device);
    int rc;
    if (!m->g_step && (rc = bn_capture(m, 1, &m->g_step))) return rc;
    if (!m->g_last && (rc = bn_capture(m, 2, &m->g_last))) return rc;
    const uint32_t E = m->cfg.n_embd;
    WL_CUDA(cudaMemsetAsync(m->d_step, 0, 4, m->stream));
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (device_ms) {
        WL_CUDA(cudaEventCreate(&e0));
        WL_CUDA(cudaEventCreate(&e1));
        WL_CUDA(cudaEventRecord(e0, m->stream));
    }
    for (uint32_t step = 0; step < n_new; ++step) {
        if (out_hiddens)  // the hidden this step's id is chosen from
            WL_CUDA(cudaMemcpyAsync(out_hiddens + (size_t)step * E, m->final_h, (size_t)E * 4,
                                    cudaMemcpyDeviceToHost, m->stream));
        WL_CUDA(cudaGraphLaunch(step + 1 < n_new ? m->g_step : m->g_last, m->stream));
    }
    if (device_ms) {
        WL_CUDA(cudaEventRecord(e1, m->stream));
        WL_CUDA(cudaEventSynchronize(e1));
        cudaEventElapsedTime(device_ms, e0, e1);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    m->pos += n_new - 1;
    if ((rc = bn_check_status(m))) return rc;
    WL_CUDA(cudaMemcpy(out_ids, m->d_ids, (size_t)n_new * 4, cudaMemcpyDeviceToHost));
    return WL_OK;
}

int wl_bitnet_generate(wl_bitnet *m, const uint32_t *prompt, uint32_t n_prompt, uint32_t n_new,
                       uint32_t *out_ids, float *out_hiddens) {
    if (!m) return fail(WL_ERR_INVALID_ARGUMENT, "model is NULL");
    if (n_prompt == 0 || !prompt)
        return fail(WL_ERR_GGUF_PARSE, "greedy_generate_with_cache: prompt_ids must not be empty");
    if ((uint64_t)n_prompt + n_new > m->cfg.max_seq)
        return fail(WL_ERR_GGUF_PARSE, "prompt %u + %u new tokens exceed the cache (%u)", n_prompt,
                    n_new, m->cfg.max_seq);
    int rc = wl_bitnet_reset(m);
    if (!rc) rc = wl_bitnet_prefill(m, prompt, n_prompt);
    if (!rc) rc = wl_bitnet_decode(m, n_new, out_ids, out_hiddens, nullptr);
    return rc;
}

}  // extern "C"

// ============================================ batched Q8_0 Llama decode engine
// Independent sequences decoded in lock step (one token per sequence per
// step), each with its own i8 KV cache and position; every step is one CUDA
// graph: embedding -> per layer [RMSNorm + QKV, attention, O + residual,
// RMSNorm + gate/up + silu * up, down + residual] -> final norm, and the
// decode step prepends the lm-head with its argmax.  The reference runs the
// sequences one after another through greedy_generate_with_cache
// (generate.rs:111-190) with the VanillaLlama branches of the cached forward
// (cached_forward.rs:308-504: no sub-norms, SiLU FFN, Norm RoPE).
struct wl_llama_batch {
    wl_bitnet_config cfg{};
    uint32_t n_seqs = 0;
    int device = 0, sm_count = 148;
    cudaStream_t stream = nullptr;
    uint8_t *wblock = nullptr;                // every repacked Q8_0 linear
    std::vector<const uint8_t *> mats;        // n_layers * 7
    float *attn_norm = nullptr, *ffn_norm = nullptr, *out_norm = nullptr;
    uint8_t *emb = nullptr;                   // repacked tied embedding / lm-head
    float2 *rope = nullptr;
    int8_t *kq = nullptr, *vq = nullptr;      // [layer][seq][max_seq][KV]
    float *ks = nullptr, *vs = nullptr;       // [layer][seq][max_seq]
    float *hidden = nullptr, *qkv = nullptr, *att = nullptr, *fused = nullptr,
          *final_h = nullptr;
    uint32_t *d_tokens = nullptr, *d_active = nullptr, *d_ones = nullptr, *d_pos = nullptr,
             *d_cur_pos = nullptr, *d_step = nullptr, *d_ids = nullptr, *d_status = nullptr,
             *d_counter = nullptr, *attn_counters = nullptr;
    unsigned long long *d_slots = nullptr;
    float *attn_partial = nullptr;
    uint32_t splits = 1, ids_cap_steps = 0;
    bool gqa_attn = false;                    // attn_gqa_batch_kernel (fast mode) or attn_decode_kernel
    bool exact_attn = false;                  // exact mode: attn_exact_kernel
    uint32_t attn_chunk = 0;                  // positions per attention CTA (gqa kernel)
    uint32_t fixed_tg = 0;                    // tokens per CTA of the linears, 0: chosen per launch
    std::vector<uint32_t> pos;                // host mirror of every position
    std::vector<uint8_t> have_hidden;
    cudaGraphExec_t g_forward = nullptr, g_step = nullptr, g_last = nullptr;
};

namespace {

constexpr int LB_MATS = 7;  // q, k, v, o, gate, up, down

using QbKernel = void (*)(Q8BatchParams);
// [FMA][TG index] for TG in {1, 4, 8, 32}
const QbKernel kQb[2][4] = {
    {q8_batch_kernel<1, false>, q8_batch_kernel<4, false>, q8_batch_kernel<8, false>,
     q8_batch_kernel<32, false>},
    {q8_batch_kernel<1, true>, q8_batch_kernel<4, true>, q8_batch_kernel<8, true>,
     q8_batch_kernel<32, true>}};
constexpr uint32_t kQbTg[4] = {1, 4, 8, 32};


int lb_validate(const wl_bitnet_config *c, uint32_t n_seqs) {
    if (!c) return fail(WL_ERR_INVALID_ARGUMENT, "config is NULL");
    const uint32_t E = c->n_embd, F = c->n_ff, HD = c->head_dim;
    if (!n_seqs || n_seqs > 1024) return fail(WL_ERR_INVALID_ARGUMENT, "n_seqs %u (1..1024)", n_seqs);
    if (c->kv_f16) return fail(WL_ERR_INVALID_ARGUMENT, "kv_f16: the Llama batch engine keeps the int8 cache");
    if (!c->n_layers || !E || !F || !HD || !c->n_heads || !c->n_kv_heads || !c->vocab ||
        !c->max_seq)
        return fail(WL_ERR_GGUF_PARSE, "llama config: zero dimension");
    if (E % 32 || F % 32 || E > 8192 || F > 16384)
        return fail(WL_ERR_GGUF_PARSE, "embedding %u / feed-forward %u: Q8_0 needs multiples of 32",
                    E, F);
    if (c->n_heads * HD != E || c->n_heads % c->n_kv_heads)
        return fail(WL_ERR_GGUF_PARSE, "heads %u x head_dim %u vs embedding %u / kv heads %u",
                    c->n_heads, HD, E, c->n_kv_heads);
    if (HD % 32 || HD > 256) return fail(WL_ERR_GGUF_PARSE, "head_dim %u must be a multiple of 32 <= 256", HD);
    if (!c->n_rot || c->n_rot % 2 || c->n_rot > HD)
        return fail(WL_ERR_GGUF_PARSE, "rope_dimension_count %u", c->n_rot);
    if (attn_smem_bytes(c->n_kv_heads * HD, HD, c->max_seq, 1) > (size_t)WL_MAX_DYN_SMEM)
        return fail(WL_ERR_INVALID_ARGUMENT, "max_seq %u too long for the attention kernel", c->max_seq);
    if (!std::isfinite(c->eps) || !std::isfinite(c->freq_base))
        return fail(WL_ERR_GGUF_PARSE, "non-finite eps / rope base");
    return WL_OK;
}

// One batched Q8_0 launch over the jobs' rows.  Paired (gate / up) CTAs hold
// 32 rows of each job, others 32 rows of one; the lm-head (argmax) uses
// 256-row CTAs with every block in one warp (no cross-warp block terms).
int lb_q8(wl_llama_batch *m, const Q8BatchJob *jobs, uint32_t n_jobs, uint32_t K, const float *x,
          uint32_t x_stride, float *y, uint32_t y_stride, uint32_t pre, const float *norm_w,
          uint32_t epi, const uint32_t *active, cudaStream_t s, uint32_t *ids = nullptr) {
    Q8BatchParams p{};
    const bool argmax = epi == QB_EPI_ARGMAX, paired = epi == QB_EPI_SILU_PAIR;
    p.rg = argmax ? 8u : 1u;
    p.stage_w = argmax ? 0u : 1u;
    const uint32_t RT = 32u * p.rg, R2 = paired ? 2u * RT : RT;
    const uint32_t phases = QB_WARPS / (R2 / 32u);
    uint32_t tiles = 0;
    for (uint32_t i = 0; i < n_jobs; ++i) {
        p.job[i] = jobs[i];
        p.job[i].tile0 = tiles;
        if (!paired || i == 0) tiles += (jobs[i].n + RT - 1) / RT;
    }
    p.n_jobs = n_jobs;
    p.K = K;
    p.n_tokens = m->n_seqs;
    p.x = x;
    p.x_stride = x_stride;
    p.y = y;
    p.y_stride = y_stride;
    p.pre = pre;
    p.norm_w = norm_w;
    p.eps = m->cfg.eps;
    p.exact_norm = m->cfg.exact;
    p.epi = epi;
    p.active = active;
    p.status = m->d_status;
    p.slots = m->d_slots;
    p.counter = m->d_counter;
    p.tokens = m->d_tokens;
    p.ids = ids;
    p.step = m->d_step;
    // Tokens per CTA: the fixed choice when set and feasible, else the rule below.
    const QbKernel *ks = kQb[m->cfg.exact ? 0 : 1];
    int ti = -1;
    for (int c = 0; c < 4; ++c) {
        const uint32_t tg = kQbTg[c];
        const size_t sm = q8_batch_smem_bytes(K, tg, R2, phases, p.stage_w != 0, pre == QB_PRE_RMSNORM);
        if (sm > (size_t)WL_MAX_DYN_SMEM) continue;
        if (m->fixed_tg) {
            if (tg == m->fixed_tg || ti < 0) ti = c;  // else the smallest feasible
            continue;
        }
        if (c > 0 && kQbTg[c - 1] >= m->n_seqs) break;  // a larger group only adds empty tokens
        // measured on the SmolLM shapes (32 sequences): about 8 token groups
        // (TG = sequences / 8) balance the per-CTA weight copy and conversion
        // against the number of CTAs, for the layers and the lm-head alike;
        // take the largest TG not above that
        if (ti < 0 || tg <= std::max<uint32_t>(1u, (m->n_seqs + 7u) / 8u)) ti = c;
    }
    if (ti < 0) return fail(WL_ERR_INVALID_ARGUMENT, "in_dim %u too large for the batched Q8_0 kernel", K);
    const uint32_t tg = kQbTg[ti];
    const size_t smem = q8_batch_smem_bytes(K, tg, R2, phases, p.stage_w != 0, pre == QB_PRE_RMSNORM);
    WL_CUDA(launch(ks[ti], dim3(tiles, (m->n_seqs + tg - 1) / tg), dim3(QB_THREADS), smem, s, true, p));
    return WL_OK;
}

int lb_enqueue_forward(wl_llama_batch *m, cudaStream_t s) {
    const wl_bitnet_config &c = m->cfg;
    const uint32_t E = c.n_embd, F = c.n_ff, HD = c.head_dim, KV = c.n_kv_heads * HD;
    const uint32_t S = m->n_seqs, QS = E + 2 * KV;
    EmbedQ8BatchParams ep;
    ep.packed = m->emb;
    ep.K = E;
    ep.tokens = m->d_tokens;
    ep.active = m->d_active;
    ep.hidden = m->hidden;
    ep.pos = m->d_pos;
    ep.cur_pos = m->d_cur_pos;
    WL_CUDA(launch(embed_q8_batch_kernel, dim3(S), dim3(256), 0, s, true, ep));
    const size_t attn_smem = m->gqa_attn ? attn_gqa_smem_bytes(KV, HD, c.n_heads / c.n_kv_heads,
                                                               m->attn_chunk)
                             : m->exact_attn ? attn_exact_smem_bytes(KV, HD, c.max_seq)
                                             : attn_smem_bytes(KV, HD, c.max_seq, m->splits);
    const float scale = 1.0f / sqrtf((float)HD);  // attention_scale (primitives.rs:354-357)
    int rc;
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        const uint8_t *const *w = m->mats.data() + (size_t)l * LB_MATS;
        Q8BatchJob qkv[3] = {{w[0], E, 0, 0}, {w[1], KV, E, 0}, {w[2], KV, E + KV, 0}};
        if ((rc = lb_q8(m, qkv, 3, E, m->hidden, E, m->qkv, QS, QB_PRE_RMSNORM,
                        m->attn_norm + (size_t)l * E, QB_EPI_STORE, m->d_active, s)))
            return rc;
        AttnParams ap{};
        ap.q = m->qkv;
        ap.k = m->qkv + E;
        ap.v = m->qkv + E + KV;
        ap.att = m->att;
        // cache layout [layer][sequence][position][KV]: one layer's caches of
        // every sequence are contiguous
        const size_t cache_l = (size_t)l * S * c.max_seq;
        ap.k_cache = m->kq + cache_l * KV;
        ap.v_cache = m->vq + cache_l * KV;
        ap.k_scale = m->ks + cache_l;
        ap.v_scale = m->vs + cache_l;
        ap.rope = m->rope;
        ap.pos = m->d_cur_pos;
        ap.n_kv_heads = c.n_kv_heads;
        ap.head_dim = HD;
        ap.n_rot = c.n_rot;
        ap.max_seq = c.max_seq;
        ap.group = c.n_heads / c.n_kv_heads;
        ap.splits = m->splits;
        ap.scale = scale;
        ap.partial = m->attn_partial;
        ap.counters = m->attn_counters;
        ap.status = m->d_status;
        ap.exact = c.exact;
        ap.qkv_stride = QS;
        ap.att_stride = E;
        ap.scale_stride = c.max_seq;
        ap.cache_stride = (size_t)c.max_seq * KV;
        ap.active = m->d_active;
        ap.rope_pairs = 1;  // RopeType::Norm for VanillaLlama (cached_forward.rs:505-509)
        ap.chunk = m->attn_chunk;
        if (m->gqa_attn) {
            WL_CUDA(launch(gqa_attn_kernel(HD, c.n_heads / c.n_kv_heads), dim3(c.n_kv_heads, S, m->splits),
                           dim3(AB_THREADS), attn_smem, s, true, ap));
        } else if (m->exact_attn) {
            // the positions were latched by this step's embedding kernel:
            // the history is staged after the dependency wait (pos_stable 0)
            WL_CUDA(launch(attn_exact_kernel, dim3(c.n_heads, 1, S), dim3(AX_THREADS), attn_smem, s,
                           true, ap));
        } else {
            WL_CUDA(launch(attn_decode_kernel<false>, dim3(c.n_heads, m->splits, S), dim3(ATTN_THREADS),
                           attn_smem, s, true, ap));
        }
        Q8BatchJob o[1] = {{w[3], E, 0, 0}};
        if ((rc = lb_q8(m, o, 1, E, m->att, E, m->hidden, E, QB_PRE_NONE, nullptr,
                        QB_EPI_RESIDUAL, m->d_active, s)))
            return rc;
        Q8BatchJob gu[2] = {{w[4], F, 0, 0}, {w[5], F, 0, 0}};
        if ((rc = lb_q8(m, gu, 2, E, m->hidden, E, m->fused, F, QB_PRE_RMSNORM,
                        m->ffn_norm + (size_t)l * E, QB_EPI_SILU_PAIR, m->d_active, s)))
            return rc;
        Q8BatchJob dn[1] = {{w[6], E, 0, 0}};
        if ((rc = lb_q8(m, dn, 1, F, m->fused, F, m->hidden, E, QB_PRE_NONE, nullptr,
                        QB_EPI_RESIDUAL, m->d_active, s)))
            return rc;
    }
    OutNormBatchParams op;
    op.hidden = m->hidden;
    op.w = m->out_norm;
    op.out = m->final_h;
    op.n = E;
    op.eps = c.eps;
    op.exact = c.exact;
    WL_CUDA(launch(out_norm_batch_kernel, dim3(S), dim3(256), 0, s, true, op));
    return WL_OK;
}

// lm-head over every sequence's final hidden + argmax -> d_tokens and the
// id history row d_ids[*d_step].
int lb_enqueue_head(wl_llama_batch *m, cudaStream_t s) {
    Q8BatchJob lm[1] = {{m->emb, m->cfg.vocab, 0, 0}};
    return lb_q8(m, lm, 1, m->cfg.n_embd, m->final_h, m->cfg.n_embd, nullptr, 0, QB_PRE_NONE,
                 nullptr, QB_EPI_ARGMAX, nullptr, s, m->d_ids);
}

// which: 0 forward, 1 head + forward (a decode step), 2 head only (the last)
int lb_capture(wl_llama_batch *m, int which, cudaGraphExec_t *out) {
    cudaGraph_t g = nullptr;
    WL_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int rc = WL_OK;
    if (which != 0) rc = lb_enqueue_head(m, m->stream);
    if (!rc && which != 2) rc = lb_enqueue_forward(m, m->stream);
    cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return fail(WL_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(WL_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
    return WL_OK;
}

int lb_check_status(wl_llama_batch *m) {
    WL_CUDA(cudaStreamSynchronize(m->stream));
    uint32_t f = 0;
    WL_CUDA(cudaMemcpy(&f, m->d_status, 4, cudaMemcpyDeviceToHost));
    if (!f) return WL_OK;
    WL_CUDA(cudaMemset(m->d_status, 0, 4));
    if (f & WL_DEV_ERR_NONFINITE)
        return fail(WL_ERR_GGUF_PARSE, "forward_with_cache: non-finite hidden after a layer");
    if (f & WL_DEV_ERR_POSITION) return fail(WL_ERR_GGUF_PARSE, "KV cache is full");
    return fail(WL_ERR_DEVICE_TIMEOUT, "device status %#x", f);
}

// Host-side validation of GGUF Q8_0 rows: every block scale finite (the
// reference's dot_row rejects a non-finite d, q8_0.rs:50-70).
int lb_check_q8_scales(const uint8_t *raw, size_t n_blocks, const char *what, uint32_t idx) {
    for (size_t b = 0; b < n_blocks; ++b) {
        const uint16_t h = (uint16_t)(raw[b * 34] | (raw[b * 34 + 1] << 8));
        if (((h >> 10) & 0x1Fu) == 0x1Fu)
            return fail(WL_ERR_GGUF_PARSE, "%s %u: Q8_0 block %zu has a non-finite scale", what, idx, b);
    }
    return WL_OK;
}

}  // namespace

extern "C" {

int wl_llama_batch_create(const wl_bitnet_config *cfg, const wl_llama_weights *w, uint32_t n_seqs,
                          wl_llama_batch **out) {
    if (!out) return fail(WL_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    int rc = lb_validate(cfg, n_seqs);
    if (rc) return rc;
    if (!w || !w->w || !w->attn_norm || !w->ffn_norm || !w->output_norm || !w->token_embd)
        return fail(WL_ERR_INVALID_ARGUMENT, "weights: NULL pointer");
    const wl_bitnet_config c = *cfg;
    const uint32_t E = c.n_embd, F = c.n_ff, KV = c.n_kv_heads * c.head_dim, S = n_seqs;
    const uint32_t outs[LB_MATS] = {E, KV, KV, E, F, F, E};
    const uint32_t ins[LB_MATS] = {E, E, E, E, E, E, F};
    for (uint32_t i = 0; i < c.n_layers * LB_MATS; ++i) {
        if (!w->w[i]) return fail(WL_ERR_GGUF_PARSE, "layer %u tensor %u: missing data", i / LB_MATS, i % LB_MATS);
        if ((rc = lb_check_q8_scales(w->w[i], (size_t)outs[i % LB_MATS] * (ins[i % LB_MATS] / 32),
                                     "linear", i)))
            return rc;
    }
    if ((rc = lb_check_q8_scales(w->token_embd, (size_t)c.vocab * (E / 32), "token_embd", 0)))
        return rc;
    Ctx &cx = ctx();
    std::lock_guard<std::mutex> lk(cx.mu);
    if ((rc = ensure_init(cx))) return rc;
    auto *m = new wl_llama_batch();
    m->cfg = c;
    m->n_seqs = S;
    m->device = cx.device;
    m->sm_count = cx.sm_count;
    m->pos.assign(S, 0u);
    m->have_hidden.assign(S, 0u);
    auto cleanup = [&](int code) {
        wl_llama_batch_destroy(m);
        return code;
    };
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
        return cleanup(fail(WL_ERR_CUDA, "stream"));
    size_t total = 0;
    std::vector<size_t> off(c.n_layers * LB_MATS);
    for (uint32_t i = 0; i < c.n_layers * LB_MATS; ++i) {
        off[i] = total;
        total += ((size_t)q8_row_stride(ins[i % LB_MATS]) * outs[i % LB_MATS] + 255) & ~(size_t)255;
    }
    const size_t kv_bytes = (size_t)S * c.n_layers * c.max_seq * KV;
    const size_t kvs = (size_t)S * c.n_layers * c.max_seq;
    m->ids_cap_steps = 4096;
    // Attention: exact mode one CTA per (head, sequence) summing in the
    // reference's order; fast mode one CTA per (KV head, sequence, split)
    // for groups of up to 4 q heads, splits filling about two CTAs per SM.
    const uint32_t group = c.n_heads / c.n_kv_heads;
    m->splits = 1;
    if (!c.exact && gqa_attn_kernel(c.head_dim, group) && c.n_rot % 4 == 0) {
        // splits of a fixed number of positions (a sequence uses as many as
        // its context needs, so CTAs are equally long whatever the context
        // mix); at most AB_COMBINE / group of them (the combine's table)
        uint32_t chunk = 256;
        while ((c.max_seq + chunk - 1) / chunk > AB_COMBINE / group) chunk *= 2;
        if (attn_gqa_smem_bytes(KV, c.head_dim, group, chunk) <= (size_t)WL_MAX_DYN_SMEM) {
            m->gqa_attn = true;
            m->attn_chunk = chunk;
            m->splits = (c.max_seq + chunk - 1) / chunk;
        }
    }
    m->exact_attn = c.exact && attn_exact_smem_bytes(KV, c.head_dim, c.max_seq) <=
                                   kernel_dyn_cap((const void *)attn_exact_kernel);
    if (!c.exact && !m->gqa_attn)
        m->splits = std::max<uint32_t>(1u, std::min<uint32_t>(
                                               (c.max_seq + 63) / 64,
                                               (2u * (uint32_t)cx.sm_count + c.n_heads * S - 1) /
                                                   (c.n_heads * S)));
    void *p = nullptr;
#define LB_ALLOC(ptr, bytes)                                                         \
    do {                                                                             \
        if (cudaMalloc(&p, (bytes)) != cudaSuccess)                                  \
            return cleanup(fail(WL_ERR_CUDA, "out of device memory (%s)", #ptr));    \
        ptr = reinterpret_cast<decltype(ptr)>(p);                                    \
    } while (0)
    LB_ALLOC(m->wblock, total);
    LB_ALLOC(m->attn_norm, (size_t)c.n_layers * E * 4);
    LB_ALLOC(m->ffn_norm, (size_t)c.n_layers * E * 4);
    LB_ALLOC(m->out_norm, (size_t)E * 4);
    LB_ALLOC(m->emb, (size_t)c.vocab * q8_row_stride(E));
    LB_ALLOC(m->rope, (size_t)c.max_seq * (c.n_rot / 2) * sizeof(float2));
    LB_ALLOC(m->kq, kv_bytes);
    LB_ALLOC(m->vq, kv_bytes);
    LB_ALLOC(m->ks, kvs * 4);
    LB_ALLOC(m->vs, kvs * 4);
    LB_ALLOC(m->hidden, (size_t)S * E * 4);
    LB_ALLOC(m->qkv, (size_t)S * (E + 2 * KV) * 4);
    LB_ALLOC(m->att, (size_t)S * E * 4);
    LB_ALLOC(m->fused, (size_t)S * F * 4);
    LB_ALLOC(m->final_h, (size_t)S * E * 4);
    LB_ALLOC(m->d_tokens, (size_t)S * 4);
    LB_ALLOC(m->d_active, (size_t)S * 4);
    LB_ALLOC(m->d_ones, (size_t)S * 4);
    LB_ALLOC(m->d_pos, (size_t)S * 4);
    LB_ALLOC(m->d_cur_pos, (size_t)S * 4);
    LB_ALLOC(m->d_step, 16);
    LB_ALLOC(m->d_status, 16);
    LB_ALLOC(m->d_counter, 16);
    LB_ALLOC(m->d_slots, (size_t)S * 8);
    LB_ALLOC(m->d_ids, (size_t)m->ids_cap_steps * S * 4);
    LB_ALLOC(m->attn_partial, (size_t)S * c.n_heads * m->splits * (4 + c.head_dim) * 4);
    LB_ALLOC(m->attn_counters, (size_t)S * c.n_heads * 4);
#undef LB_ALLOC
    cudaStream_t s = m->stream;
    cudaError_t e = cudaSuccess;
    // weights: GGUF rows staged through one device buffer, repacked in place
    size_t stage_bytes = (size_t)c.vocab * (E / 32) * 34;
    for (uint32_t i = 0; i < LB_MATS; ++i)
        stage_bytes = std::max(stage_bytes, (size_t)outs[i] * (ins[i] / 32) * 34);
    uint8_t *stage = nullptr;
    if (cudaMalloc(&stage, stage_bytes) != cudaSuccess) return cleanup(fail(WL_ERR_CUDA, "staging"));
    m->mats.resize((size_t)c.n_layers * LB_MATS);
    for (uint32_t i = 0; i <= c.n_layers * LB_MATS && e == cudaSuccess; ++i) {
        const bool is_emb = i == c.n_layers * LB_MATS;
        const uint32_t K = is_emb ? E : ins[i % LB_MATS], N = is_emb ? c.vocab : outs[i % LB_MATS];
        const uint8_t *src = is_emb ? w->token_embd : w->w[i];
        uint8_t *dst = is_emb ? m->emb : m->wblock + off[i];
        e = cudaMemcpyAsync(stage, src, (size_t)N * (K / 32) * 34, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) {
            q8_0_repack_kernel<<<1024, 256, 0, s>>>(stage, K, N, dst);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // the staging buffer is reused
        if (!is_emb) m->mats[i] = dst;
    }
    cudaFree(stage);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->attn_norm, w->attn_norm, (size_t)c.n_layers * E * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->ffn_norm, w->ffn_norm, (size_t)c.n_layers * E * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->out_norm, w->output_norm, (size_t)E * 4, cudaMemcpyHostToDevice, s);
    std::vector<float2> rope;
    bn_rope_table(c, rope);
    std::vector<uint32_t> ones(S, 1u);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->d_ones, ones.data(), (size_t)S * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->d_pos, 0, (size_t)S * 4, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->d_step, 0, 16, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->d_status, 0, 16, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->d_counter, 0, 16, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->d_slots, 0, (size_t)S * 8, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->attn_counters, 0, (size_t)S * c.n_heads * 4, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // the host vectors above go out of scope
    if (e != cudaSuccess) return cleanup(fail(WL_ERR_CUDA, "weight upload: %s", cudaGetErrorString(e)));
    *out = m;
    return WL_OK;
}

int wl_llama_batch_destroy(wl_llama_batch *m) {
    if (!m) return WL_OK;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (cudaGraphExec_t g : {m->g_forward, m->g_step, m->g_last})
        if (g) cudaGraphExecDestroy(g);
    void *bufs[] = {m->wblock, m->attn_norm, m->ffn_norm, m->out_norm, m->emb, m->rope, m->kq,
                    m->vq, m->ks, m->vs, m->hidden, m->qkv, m->att, m->fused, m->final_h,
                    m->d_tokens, m->d_active, m->d_ones, m->d_pos, m->d_cur_pos, m->d_step,
                    m->d_status, m->d_counter, m->d_slots, m->d_ids, m->attn_partial,
                    m->attn_counters};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return WL_OK;
}

int wl_llama_batch_reset(wl_llama_batch *m) {
    if (!m) return fail(WL_ERR_INVALID_ARGUMENT, "batch is NULL");
    cudaSetDevice(m->device);
    WL_CUDA(cudaMemsetAsync(m->d_pos, 0, (size_t)m->n_seqs * 4, m->stream));
    WL_CUDA(cudaStreamSynchronize(m->stream));
    std::fill(m->pos.begin(), m->pos.end(), 0u);
    std::fill(m->have_hidden.begin(), m->have_hidden.end(), 0u);
    return WL_OK;
}

uint32_t wl_llama_batch_position(const wl_llama_batch *m, uint32_t seq) {
    return m && seq < m->n_seqs ? m->pos[seq] : 0u;
}

uint32_t wl_llama_batch_attention_splits(const wl_llama_batch *m) { return m ? m->splits : 0u; }

int wl_llama_batch_set_tokens_per_cta(wl_llama_batch *m, uint32_t tg) {
    if (!m) return fail(WL_ERR_INVALID_ARGUMENT, "batch is NULL");
    bool ok = tg == 0;
    for (uint32_t t : kQbTg) ok = ok || t == tg;
    if (!ok) return fail(WL_ERR_INVALID_ARGUMENT, "tokens per CTA %u: 0 (auto), 1, 4, 8 or 32", tg);
    cudaSetDevice(m->device);
    WL_CUDA(cudaStreamSynchronize(m->stream));
    for (cudaGraphExec_t *g : {&m->g_forward, &m->g_step, &m->g_last})
        if (*g) {
            cudaGraphExecDestroy(*g);
            *g = nullptr;
        }
    m->fixed_tg = tg;
    return WL_OK;
}

int wl_llama_batch_prefill(wl_llama_batch *m, const uint32_t *tokens, const uint32_t *offsets) {
    if (!m || !offsets) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    const uint32_t S = m->n_seqs;
    uint32_t longest = 0;
    for (uint32_t b = 0; b < S; ++b) {
        if (offsets[b + 1] < offsets[b]) return fail(WL_ERR_INVALID_ARGUMENT, "offsets must not decrease");
        const uint32_t n = offsets[b + 1] - offsets[b];
        if ((uint64_t)m->pos[b] + n > m->cfg.max_seq) return fail(WL_ERR_GGUF_PARSE, "KV cache is full");
        if (n && !tokens) return fail(WL_ERR_INVALID_ARGUMENT, "tokens is NULL");
        for (uint32_t i = offsets[b]; i < offsets[b + 1]; ++i)
            if (tokens[i] >= m->cfg.vocab)
                return fail(WL_ERR_GGUF_PARSE, "prompt token %u (sequence %u) out of vocab range %u",
                            tokens[i], b, m->cfg.vocab);
        longest = std::max(longest, n);
    }
    if (!longest) return WL_OK;
    cudaSetDevice(m->device);
    // step-major token / activity matrices, uploaded once
    std::vector<uint32_t> tok((size_t)longest * S, 0u), act((size_t)longest * S, 0u);
    for (uint32_t b = 0; b < S; ++b)
        for (uint32_t i = 0; i < offsets[b + 1] - offsets[b]; ++i) {
            tok[(size_t)i * S + b] = tokens[offsets[b] + i];
            act[(size_t)i * S + b] = 1u;
        }
    uint32_t *d_mat = nullptr;
    WL_CUDA(cudaMalloc(&d_mat, tok.size() * 8));
    int rc = WL_OK;
    cudaError_t e = cudaMemcpyAsync(d_mat, tok.data(), tok.size() * 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d_mat + tok.size(), act.data(), act.size() * 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess && !m->g_forward) rc = lb_capture(m, 0, &m->g_forward);
    for (uint32_t i = 0; i < longest && e == cudaSuccess && !rc; ++i) {
        e = cudaMemcpyAsync(m->d_tokens, d_mat + (size_t)i * S, (size_t)S * 4, cudaMemcpyDeviceToDevice, m->stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(m->d_active, d_mat + tok.size() + (size_t)i * S, (size_t)S * 4,
                                cudaMemcpyDeviceToDevice, m->stream);
        if (e == cudaSuccess) e = cudaGraphLaunch(m->g_forward, m->stream);
    }
    const cudaError_t e2 = cudaStreamSynchronize(m->stream);  // the host matrices go out of scope
    if (e == cudaSuccess) e = e2;
    cudaFree(d_mat);
    if (rc) return rc;
    if (e != cudaSuccess) return fail(WL_ERR_CUDA, "prefill: %s", cudaGetErrorString(e));
    for (uint32_t b = 0; b < S; ++b) {
        const uint32_t n = offsets[b + 1] - offsets[b];
        m->pos[b] += n;
        if (n) m->have_hidden[b] = 1u;
    }
    return lb_check_status(m);
}

int wl_llama_batch_decode(wl_llama_batch *m, uint32_t n_new, uint32_t *out_ids, float *out_hiddens,
                          float *device_ms) {
    if (!m || (!out_ids && n_new)) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    const uint32_t S = m->n_seqs, E = m->cfg.n_embd;
    for (uint32_t b = 0; b < S; ++b) {
        if (!m->have_hidden[b])
            return fail(WL_ERR_INVALID_ARGUMENT, "decode needs every sequence prefilled (sequence %u)", b);
        if (n_new && (uint64_t)m->pos[b] + n_new - 1 > m->cfg.max_seq)
            return fail(WL_ERR_GGUF_PARSE, "KV cache is full");
    }
    if (n_new == 0) return WL_OK;
    if (n_new > m->ids_cap_steps) return fail(WL_ERR_INVALID_ARGUMENT, "n_new > %u", m->ids_cap_steps);
    cudaSetDevice(m->device);
    int rc;
    if (!m->g_step && (rc = lb_capture(m, 1, &m->g_step))) return rc;
    if (!m->g_last && (rc = lb_capture(m, 2, &m->g_last))) return rc;
    WL_CUDA(cudaMemsetAsync(m->d_step, 0, 4, m->stream));
    WL_CUDA(cudaMemcpyAsync(m->d_active, m->d_ones, (size_t)S * 4, cudaMemcpyDeviceToDevice, m->stream));
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (device_ms) {
        WL_CUDA(cudaEventCreate(&e0));
        WL_CUDA(cudaEventCreate(&e1));
        WL_CUDA(cudaEventRecord(e0, m->stream));
    }
    for (uint32_t step = 0; step < n_new; ++step) {
        if (out_hiddens)  // the hiddens this step's ids are chosen from
            WL_CUDA(cudaMemcpyAsync(out_hiddens + (size_t)step * S * E, m->final_h, (size_t)S * E * 4,
                                    cudaMemcpyDeviceToHost, m->stream));
        WL_CUDA(cudaGraphLaunch(step + 1 < n_new ? m->g_step : m->g_last, m->stream));
    }
    if (device_ms) {
        WL_CUDA(cudaEventRecord(e1, m->stream));
        WL_CUDA(cudaEventSynchronize(e1));
        cudaEventElapsedTime(device_ms, e0, e1);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    for (uint32_t b = 0; b < S; ++b) m->pos[b] += n_new - 1;
    if ((rc = lb_check_status(m))) return rc;
    WL_CUDA(cudaMemcpy(out_ids, m->d_ids, (size_t)n_new * S * 4, cudaMemcpyDeviceToHost));
    return WL_OK;
}

int wl_llama_batch_generate(wl_llama_batch *m, const uint32_t *tokens, const uint32_t *offsets,
                            uint32_t n_new, uint32_t *out_ids, float *out_hiddens) {
    if (!m || !offsets) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    for (uint32_t b = 0; b < m->n_seqs; ++b) {
        if (offsets[b + 1] < offsets[b] || offsets[b + 1] == offsets[b])
            return fail(WL_ERR_GGUF_PARSE, "greedy_generate_with_cache: prompt_ids must not be empty "
                        "(sequence %u)", b);
        const uint32_t n = offsets[b + 1] - offsets[b];
        if ((uint64_t)n + n_new > m->cfg.max_seq)
            return fail(WL_ERR_GGUF_PARSE, "prompt %u + %u new tokens exceed the cache (%u)", n, n_new,
                        m->cfg.max_seq);
    }
    int rc = wl_llama_batch_reset(m);
    if (!rc) rc = wl_llama_batch_prefill(m, tokens, offsets);
    if (!rc) rc = wl_llama_batch_decode(m, n_new, out_ids, out_hiddens, nullptr);
    return rc;
}

}  // extern "C"

// =============================================================== GGUF models
namespace {

using namespace wl_gguf_detail;

int gguf_missing(const std::string &what) {
    return fail(WL_ERR_MISSING_METADATA, "Missing required metadata key(s): %s", what.c_str());
}

const Value *gguf_meta(const wl_gguf *g, const std::string &key) {
    auto it = g->meta.find(key);
    return it == g->meta.end() ? nullptr : &it->second;
}

// required_u32 / optional_u32 / required_f32 / optional_f32 (config.rs:274-322)
int gguf_u32(const wl_gguf *g, const std::string &key, uint32_t *out, bool required, bool *present = nullptr) {
    const Value *v = gguf_meta(g, key);
    if (present) *present = v != nullptr;
    if (!v) return required ? gguf_missing(key + " (u32/u64)") : WL_OK;
    uint64_t u;
    if (!v->as_u64(&u)) return gguf_missing(key + " (u32/u64)");
    if (u > UINT32_MAX)
        return fail(WL_ERR_GGUF_PARSE, "metadata key %s value %llu does not fit in u32", key.c_str(),
                    (unsigned long long)u);
    *out = (uint32_t)u;
    return WL_OK;
}

int gguf_f32(const wl_gguf *g, const std::string &key, float *out, bool required, bool *present = nullptr) {
    const Value *v = gguf_meta(g, key);
    if (present) *present = v != nullptr;
    if (!v) return required ? gguf_missing(key + " (f32)") : WL_OK;
    if (!v->as_f32(out)) return gguf_missing(key + " (f32)");
    return WL_OK;
}

void gguf_view(const Tensor &t, wl_tensor_view *v) {
    v->name = t.name.c_str();
    v->shape = t.shape.data();
    v->n_dims = (uint32_t)t.shape.size();
    v->ggml_type = t.type;
    v->data = t.data;
    v->data_len = (size_t)t.byte_len;
    v->scale_data = t.scale;
    v->scale_len = t.scale ? (size_t)I2S_SCALE_BLOCK : 0;
}

// ModelConfig::from_gguf_metadata (config.rs:61-260) for the two families
// the engines run.  variant: 0 BitNetSubNorm, 1 VanillaLlama.
int gguf_config(const wl_gguf *g, wl_bitnet_config *c, uint32_t *variant) {
    const Value *a = gguf_meta(g, "general.architecture");
    if (!a || a->type != GV_STR) return gguf_missing("general.architecture (string)");
    const std::string arch = a->s;
    memset(c, 0, sizeof *c);
    int rc;
    if (arch == "bitnet-b1.58" || arch == "bitnet-25" || arch == "bitnet") {
        // from_gguf_metadata_with_prefix (config.rs:78-176), prefix = the architecture string
        auto k = [&](const char *s) { return arch + "." + s; };
        uint32_t rope_dim = 0;
        if ((rc = gguf_u32(g, k("block_count"), &c->n_layers, true)) ||
            (rc = gguf_u32(g, k("embedding_length"), &c->n_embd, true)) ||
            (rc = gguf_u32(g, k("feed_forward_length"), &c->n_ff, true)) ||
            (rc = gguf_u32(g, k("context_length"), &c->max_seq, true)) ||
            (rc = gguf_u32(g, k("attention.head_count"), &c->n_heads, true)) ||
            (rc = gguf_u32(g, k("attention.head_count_kv"), &c->n_kv_heads, true)) ||
            (rc = gguf_f32(g, k("attention.layer_norm_rms_epsilon"), &c->eps, true)) ||
            (rc = gguf_u32(g, k("rope.dimension_count"), &rope_dim, true)) ||
            (rc = gguf_f32(g, k("rope.freq_base"), &c->freq_base, true)) ||
            (rc = gguf_u32(g, k("vocab_size"), &c->vocab, true)))
            return rc;
        if (c->n_heads == 0) return fail(WL_ERR_GGUF_PARSE, "head_count must be > 0");
        if (c->n_embd % c->n_heads)
            return fail(WL_ERR_GGUF_PARSE, "embedding_length %u not divisible by head_count %u", c->n_embd,
                        c->n_heads);
        c->head_dim = c->n_embd / c->n_heads;
        if (c->n_kv_heads == 0) return fail(WL_ERR_GGUF_PARSE, "head_count_kv must be > 0");
        if (c->n_heads % c->n_kv_heads)
            return fail(WL_ERR_GGUF_PARSE, "head_count %u not divisible by head_count_kv %u (GQA ratio must be integer)",
                        c->n_heads, c->n_kv_heads);
        if (rope_dim != c->head_dim)
            return fail(WL_ERR_GGUF_PARSE, "rope.dimension_count (%u) must equal head_dim (%u)", rope_dim,
                        c->head_dim);
        if (c->n_layers == 0) return fail(WL_ERR_GGUF_PARSE, "block_count must be > 0");
        if (c->vocab == 0) return fail(WL_ERR_GGUF_PARSE, "vocab_size must be > 0");
        c->n_rot = rope_dim;
        *variant = 0;
        return WL_OK;
    }
    if (arch == "llama") {
        // from_llama_metadata_with_prefix (config.rs:178-260)
        auto k = [](const char *s) { return std::string("llama.") + s; };
        bool has_kv = false, has_rot = false, has_base = false;
        uint32_t rope_dim = 0;
        if ((rc = gguf_u32(g, k("block_count"), &c->n_layers, true)) ||
            (rc = gguf_u32(g, k("embedding_length"), &c->n_embd, true)) ||
            (rc = gguf_u32(g, k("feed_forward_length"), &c->n_ff, true)) ||
            (rc = gguf_u32(g, k("context_length"), &c->max_seq, true)) ||
            (rc = gguf_u32(g, k("attention.head_count"), &c->n_heads, true)) ||
            (rc = gguf_u32(g, k("attention.head_count_kv"), &c->n_kv_heads, false, &has_kv)) ||
            (rc = gguf_f32(g, k("attention.layer_norm_rms_epsilon"), &c->eps, true)))
            return rc;
        if (!has_kv) c->n_kv_heads = c->n_heads;
        if (c->n_heads == 0 || c->n_embd % c->n_heads)
            return fail(WL_ERR_GGUF_PARSE, "embedding_length %u must be divisible by non-zero head_count %u",
                        c->n_embd, c->n_heads);
        c->head_dim = c->n_embd / c->n_heads;
        if ((rc = gguf_u32(g, k("rope.dimension_count"), &rope_dim, false, &has_rot)) ||
            (rc = gguf_f32(g, k("rope.freq_base"), &c->freq_base, false, &has_base)))
            return rc;
        if (!has_rot) rope_dim = c->head_dim;
        if (!has_base) c->freq_base = 10000.0f;
        const Value *tok = gguf_meta(g, "tokenizer.ggml.tokens");
        bool strings = tok && tok->type == GV_ARR;
        if (strings)
            for (const Value &e : tok->arr) strings = strings && e.type == GV_STR;
        if (!strings) return gguf_missing("tokenizer.ggml.tokens (string array)");
        if (tok->arr.size() > UINT32_MAX) return fail(WL_ERR_GGUF_PARSE, "tokenizer vocabulary does not fit in u32");
        c->vocab = (uint32_t)tok->arr.size();
        if (c->n_kv_heads == 0 || c->n_heads % c->n_kv_heads)
            return fail(WL_ERR_GGUF_PARSE, "head_count %u must be divisible by non-zero head_count_kv %u",
                        c->n_heads, c->n_kv_heads);
        if (rope_dim != c->head_dim)
            return fail(WL_ERR_NOT_IMPLEMENTED, "Llama partial RoPE is not supported: rope.dimension_count=%u, head_dim=%u",
                        rope_dim, c->head_dim);
        if (rope_dim % 2) return fail(WL_ERR_GGUF_PARSE, "Llama rope.dimension_count must be even, got %u", rope_dim);
        std::vector<std::string> scaling;
        const std::string scaling_prefix = "llama.rope.scaling";
        for (auto &kv : g->meta)
            if (kv.first.compare(0, scaling_prefix.size(), scaling_prefix) == 0) scaling.push_back(kv.first);
        const bool unscaled = scaling.size() == 1 && scaling[0] == "llama.rope.scaling.type" &&
                              gguf_meta(g, scaling[0])->type == GV_STR && gguf_meta(g, scaling[0])->s == "none";
        if (!scaling.empty() && !unscaled) return fail(WL_ERR_NOT_IMPLEMENTED, "Llama RoPE scaling is not supported");
        if (!c->n_layers || !c->n_embd || !c->n_ff || !c->max_seq || !c->vocab)
            return fail(WL_ERR_GGUF_PARSE, "Llama dimensions and vocabulary must be non-zero");
        if (!std::isfinite(c->eps) || c->eps <= 0.0f)
            return fail(WL_ERR_GGUF_PARSE, "Llama RMS epsilon must be finite and positive");
        if (!std::isfinite(c->freq_base) || c->freq_base <= 0.0f)
            return fail(WL_ERR_GGUF_PARSE, "Llama RoPE frequency base must be finite and positive");
        c->n_rot = rope_dim;
        *variant = 1;
        return WL_OK;
    }
    if (arch == "qwen2")
        return fail(WL_ERR_NOT_IMPLEMENTED, "architecture qwen2 has no device engine here");
    return fail(WL_ERR_UNSUPPORTED_ARCHITECTURE, "Unsupported architecture: \"%s\"", arch.c_str());
}

// require_tensor / check_dtype / check_shape (graph.rs:440-520)
int gguf_tensor_checked(const wl_gguf *g, const std::string &name, uint32_t type, std::vector<uint64_t> shape,
                        const Tensor **out) {
    auto it = g->by_name.find(name);
    if (it == g->by_name.end()) return gguf_missing("tensor " + name);
    const Tensor &t = g->tensors[it->second];
    if (t.type != type)
        return fail(type == WL_GGML_I2_S || type == WL_GGML_F32 ? WL_ERR_GGUF_PARSE : WL_ERR_NOT_IMPLEMENTED,
                    "tensor \"%s\": expected dtype %u, got %u", name.c_str(), type, t.type);
    if (t.shape != shape) return fail(WL_ERR_GGUF_PARSE, "tensor \"%s\": unexpected shape", name.c_str());
    *out = &t;
    return WL_OK;
}

int gguf_check_unique(const wl_gguf *g) {
    if (g->by_name.size() != g->tensors.size())
        return fail(WL_ERR_GGUF_PARSE, "duplicate tensor names in GGUF tensor directory");
    return WL_OK;
}

const char *const kRoles[7] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"};

}  // namespace

extern "C" {

int wl_gguf_open(const uint8_t *data, size_t len, wl_gguf **out) {
    if (!out || (!data && len)) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    auto *g = new wl_gguf();
    Parser p;
    const Err e = parse(data, len, g, p);
    if (e != OK) {
        delete g;
        const int code = e == MAGIC ? WL_ERR_INVALID_MAGIC
                         : e == VERSION ? WL_ERR_UNSUPPORTED_VERSION
                         : e == OOB ? WL_ERR_TENSOR_OUT_OF_BOUNDS : WL_ERR_GGUF_PARSE;
        return fail(code, "%s", p.msg.c_str());
    }
    *out = g;
    return WL_OK;
}

int wl_gguf_close(wl_gguf *g) {
    delete g;
    return WL_OK;
}

uint32_t wl_gguf_version(const wl_gguf *g) { return g ? g->version : 0u; }
uint64_t wl_gguf_alignment(const wl_gguf *g) { return g ? g->alignment : 0u; }
uint64_t wl_gguf_tensor_count(const wl_gguf *g) { return g ? (uint64_t)g->tensors.size() : 0u; }

int wl_gguf_tensor(const wl_gguf *g, uint64_t i, wl_tensor_view *out) {
    if (!g || !out) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    if (i >= g->tensors.size()) return fail(WL_ERR_INVALID_ARGUMENT, "tensor index %llu out of range", (unsigned long long)i);
    gguf_view(g->tensors[i], out);
    return WL_OK;
}

int wl_gguf_find_tensor(const wl_gguf *g, const char *name, wl_tensor_view *out) {
    if (!g || !name || !out) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    auto it = g->by_name.find(name);
    if (it == g->by_name.end()) return gguf_missing(std::string("tensor ") + name);
    gguf_view(g->tensors[it->second], out);
    return WL_OK;
}

int wl_gguf_get_u64(const wl_gguf *g, const char *key, uint64_t *out) {
    if (!g || !key || !out) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    const Value *v = gguf_meta(g, key);
    if (!v || !v->as_u64(out)) return gguf_missing(std::string(key) + " (u32/u64)");
    return WL_OK;
}

int wl_gguf_get_f32(const wl_gguf *g, const char *key, float *out) {
    if (!g || !key || !out) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    const Value *v = gguf_meta(g, key);
    if (!v || !v->as_f32(out)) return gguf_missing(std::string(key) + " (f32)");
    return WL_OK;
}

int wl_gguf_get_str(const wl_gguf *g, const char *key, const char **out) {
    if (!g || !key || !out) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    const Value *v = gguf_meta(g, key);
    if (!v || v->type != GV_STR) return gguf_missing(std::string(key) + " (string)");
    *out = v->s.c_str();
    return WL_OK;
}

uint64_t wl_gguf_array_len(const wl_gguf *g, const char *key) {
    if (!g || !key) return 0;
    const Value *v = gguf_meta(g, key);
    return v && v->type == GV_ARR ? (uint64_t)v->arr.size() : 0u;
}

int wl_gguf_model_config(const wl_gguf *g, wl_bitnet_config *cfg, uint32_t *variant) {
    if (!g || !cfg) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    uint32_t v = 0;
    const int rc = gguf_config(g, cfg, &v);
    if (!rc && variant) *variant = v;
    return rc;
}

int wl_bitnet_create_from_gguf(const wl_gguf *g, uint32_t max_seq, uint32_t exact, uint32_t persistent,
                               wl_bitnet **out) {
    if (!g || !out) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    wl_bitnet_config c;
    uint32_t variant = 0;
    int rc = gguf_config(g, &c, &variant);
    if (rc) return rc;
    if (variant != 0) return fail(WL_ERR_INVALID_ARGUMENT, "not a BitNet-family model (use the Llama engine)");
    if ((rc = gguf_check_unique(g))) return rc;
    if (max_seq) c.max_seq = max_seq;
    c.exact = exact;
    c.persistent = persistent;
    c.kv_f16 = 0;
    const uint64_t E = c.n_embd, F = c.n_ff, KV = (uint64_t)c.head_dim * c.n_kv_heads, V = c.vocab;
    const std::vector<uint64_t> shapes[7] = {{E, E}, {E, KV}, {E, KV}, {E, E}, {E, F}, {E, F}, {F, E}};
    const Tensor *t;
    if ((rc = gguf_tensor_checked(g, "token_embd.weight", WL_GGML_Q6_K, {E, V}, &t))) {
        auto it = g->by_name.find("token_embd.weight");
        if (it != g->by_name.end() && g->tensors[it->second].type == WL_GGML_F16)
            return fail(WL_ERR_NOT_IMPLEMENTED, "token_embd.weight is F16: convert it with the reference's "
                        "embedding-q6-k link step first");
        return rc;
    }
    const uint8_t *emb = t->data;
    if ((rc = gguf_tensor_checked(g, "output_norm.weight", WL_GGML_F32, {E}, &t))) return rc;
    std::vector<float> out_norm(E);
    memcpy(out_norm.data(), t->data, E * 4);
    std::vector<const uint8_t *> w((size_t)c.n_layers * 7);
    std::vector<float> scales((size_t)c.n_layers * 7), norms((size_t)c.n_layers * (3 * E + F));
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        const std::string b = "blk." + std::to_string(l) + ".";
        const char *nn[4] = {"attn_norm", "attn_sub_norm", "ffn_norm", "ffn_sub_norm"};
        const uint64_t nlen[4] = {E, E, E, F};
        float *dst = norms.data() + (size_t)l * (3 * E + F);
        for (int k = 0; k < 4; ++k) {
            if ((rc = gguf_tensor_checked(g, b + nn[k] + ".weight", WL_GGML_F32, {nlen[k]}, &t))) return rc;
            memcpy(dst, t->data, nlen[k] * 4);
            dst += nlen[k];
        }
        for (int k = 0; k < 7; ++k) {
            if ((rc = gguf_tensor_checked(g, b + kRoles[k] + ".weight", WL_GGML_I2_S, shapes[k], &t))) return rc;
            float sc;
            memcpy(&sc, t->scale, 4);  // i2s_scale (tensor.rs:278-309)
            if (!std::isfinite(sc))
                return fail(WL_ERR_GGUF_PARSE, "i2s_scale: non-finite scale for tensor \"%s\"", t->name.c_str());
            w[(size_t)l * 7 + k] = t->data;
            scales[(size_t)l * 7 + k] = sc;
        }
    }
    wl_bitnet_weights wt;
    wt.w = w.data();
    wt.w_scale = scales.data();
    wt.norms = norms.data();
    wt.output_norm = out_norm.data();
    wt.token_embd = emb;
    return wl_bitnet_create(&c, &wt, out);
}

int wl_llama_batch_create_from_gguf(const wl_gguf *g, uint32_t n_seqs, uint32_t max_seq, uint32_t exact,
                                    wl_llama_batch **out) {
    if (!g || !out) return fail(WL_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    wl_bitnet_config c;
    uint32_t variant = 0;
    int rc = gguf_config(g, &c, &variant);
    if (rc) return rc;
    if (variant != 1) return fail(WL_ERR_INVALID_ARGUMENT, "not a llama model (use the BitNet engine)");
    if ((rc = gguf_check_unique(g))) return rc;
    if (max_seq) c.max_seq = max_seq;
    c.exact = exact;
    c.persistent = 0;
    c.kv_f16 = 0;
    const uint64_t E = c.n_embd, F = c.n_ff, KV = (uint64_t)c.head_dim * c.n_kv_heads, V = c.vocab;
    const std::vector<uint64_t> shapes[7] = {{E, E}, {E, KV}, {E, KV}, {E, E}, {E, F}, {E, F}, {F, E}};
    if (g->by_name.count("output.weight"))
        return fail(WL_ERR_NOT_IMPLEMENTED, "a separate output.weight lm-head is not supported (tied only)");
    const Tensor *t;
    if ((rc = gguf_tensor_checked(g, "token_embd.weight", WL_GGML_Q8_0, {E, V}, &t))) return rc;
    const uint8_t *emb = t->data;
    if ((rc = gguf_tensor_checked(g, "output_norm.weight", WL_GGML_F32, {E}, &t))) return rc;
    std::vector<float> out_norm(E), attn_norm((size_t)c.n_layers * E), ffn_norm((size_t)c.n_layers * E);
    memcpy(out_norm.data(), t->data, E * 4);
    std::vector<const uint8_t *> w((size_t)c.n_layers * 7);
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        const std::string b = "blk." + std::to_string(l) + ".";
        for (const char *bias : {"attn_q.bias", "attn_k.bias", "attn_v.bias", "attn_output.bias"})
            if (g->by_name.count(b + bias))
                return fail(WL_ERR_NOT_IMPLEMENTED, "tensor %s%s: Llama bias tensors are not supported",
                            b.c_str(), bias);
        if ((rc = gguf_tensor_checked(g, b + "attn_norm.weight", WL_GGML_F32, {E}, &t))) return rc;
        memcpy(attn_norm.data() + (size_t)l * E, t->data, E * 4);
        if ((rc = gguf_tensor_checked(g, b + "ffn_norm.weight", WL_GGML_F32, {E}, &t))) return rc;
        memcpy(ffn_norm.data() + (size_t)l * E, t->data, E * 4);
        for (int k = 0; k < 7; ++k) {
            if ((rc = gguf_tensor_checked(g, b + kRoles[k] + ".weight", WL_GGML_Q8_0, shapes[k], &t))) return rc;
            w[(size_t)l * 7 + k] = t->data;
        }
    }
    wl_llama_weights wt;
    wt.w = w.data();
    wt.attn_norm = attn_norm.data();
    wt.ffn_norm = ffn_norm.data();
    wt.output_norm = out_norm.data();
    wt.token_embd = emb;
    return wl_llama_batch_create(&c, &wt, n_seqs, out);
}

}  // extern "C"
