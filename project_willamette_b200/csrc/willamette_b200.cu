// willamette_b200.cu -- the C ABI (include/willamette_b200.h): this file holds
// the single-op entry points (matvecs, GEMM, lm-head, norms, stream plans,
// device status); the host logic they share and the engines live in the
// host_*.cuh parts it includes:
//   host_core.cuh    errors, device state, launch helpers, validation, weight cache
//   host_stream.cuh  stream plans, prefill GEMM host side
//   host_tp.cuh      tensor-parallel group and its entry points
//   host_bitnet.cuh  BitNet decode engine (wl_bitnet_*)
//   host_llama.cuh   batched Q8_0 Llama decode engine (wl_llama_batch_*)
//   host_gguf.cuh    GGUF model configuration and engine upload
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

#include "host_core.cuh"
#include "host_stream.cuh"
#include "host_tp.cuh"

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
    I2sStreamParams p = {};  // single GPU: tp.world = 0
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


}  // extern "C"

#include "host_bitnet.cuh"
#include "host_llama.cuh"
#include "host_gguf.cuh"
