// host_core.cuh -- host logic shared by every entry point: error reporting
// (fail / last error, the reference's status codes), per-device state and
// staging buffers, kernel launch helpers (programmatic dependent launch),
// input validation that mirrors the reference's rejections, the device cache
// of host weights, the host-buffer call paths, and the no-allocation
// variant's static device block.
//
// Part of the library's single translation unit: included, in order, by
// willamette_b200.cu after the headers and the parts before it (it is not a
// standalone header).
#pragma once

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
    uint8_t *pinned_dev = nullptr;  // the same buffer as the device reaches it
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
    // mapped: the host-buffer matvec's kernel writes its output here directly
    WL_CUDA(cudaHostAlloc(&c.pinned, cap, cudaHostAllocMapped | cudaHostAllocPortable));
    void *dev = nullptr;
    cudaError_t e = cudaHostGetDevicePointer(&dev, c.pinned, 0);
    if (e != cudaSuccess) {
        cudaFreeHost(c.pinned);
        c.pinned = nullptr;
        return fail(WL_ERR_CUDA, "cudaHostGetDevicePointer: %s", cudaGetErrorString(e));
    }
    c.pinned_dev = (uint8_t *)dev;
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
    uint32_t *status_host = nullptr;   // host-mapped error word, or null
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
    p.status_host = L.status_host;
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
    // No debug outputs: the kernel writes y straight into the mapped pinned
    // buffer (no device-to-host copy to wait for: about 2 us of a call) and
    // sets a host-mapped word beside it if any status bit is raised; the
    // status bits themselves stay in device memory (c.ys).
    const bool plain = !gemm && !acc_out && !act_q_out && !act_scale_out;
    if (plain && (rc = grow(c.ys, 16))) return rc;
    volatile uint32_t *hflag = reinterpret_cast<volatile uint32_t *>(pin + xin);  // [flag][pad][y]
    if (plain) *hflag = 0u;
    float *ydev = plain ? (float *)(c.pinned_dev + xin + 16) : (float *)c.y.p;
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
        if (plain) L.status_host = (uint32_t *)(c.pinned_dev + xin);
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
        cudaError_t e = cudaStreamSynchronize(c.stream);
        if (e != cudaSuccess) return fail(WL_ERR_CUDA, "kernel execution: %s", cudaGetErrorString(e));
        if (*hflag) {
            uint32_t f = 0;
            WL_CUDA(cudaMemcpyAsync(c.h_status + 9, c.ys.p, 4, cudaMemcpyDeviceToHost, c.stream));
            WL_CUDA(cudaMemsetAsync(c.ys.p, 0, 4, c.stream));
            WL_CUDA(cudaStreamSynchronize(c.stream));
            f = c.h_status[9];
            return fail(WL_ERR_DEVICE_TIMEOUT, "a device-side wait timed out (flags 0x%x)", f);
        }
        memcpy(output, pin + xin + 16, yout);
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
