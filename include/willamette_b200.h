/*
 * willamette_b200.h -- C ABI of the B200 (sm_100a) BitLinear hot-path library.
 *
 * A drop-in for project-willamette's BitLinear / lm-head call surface
 * (Rust crate project-willamette v0.14.0).  Each entry point names the
 * reference function it replaces.  The ABI uses plain pointers and sizes
 * only: no CUDA, torch or C++ types cross it (a cudaStream_t is passed as
 * `void *`).
 *
 * Two families of entry points:
 *   wl_*      synchronous, HOST buffers in and out -- the same contract as the
 *             reference functions (inputs borrowed, output caller-allocated
 *             and fully overwritten on success, never written with fake
 *             values on error).  Weights are uploaded to the GPU on first use
 *             and cached, keyed by (data pointer, length, type, shape); the
 *             reference's weights are an immutable mmap for the life of the
 *             process, which is what makes that cache valid.
 *   wl_dev_*  asynchronous on a caller stream, DEVICE pointers, no host sync.
 *
 * Every entry point returns a wl_status; on failure wl_last_error() (thread
 * local) holds the message.  No entry point ever falls back to a CPU
 * implementation: without a usable sm_100 device they return WL_ERR_CUDA or
 * WL_ERR_NO_DEVICE.
 */
#ifndef WILLAMETTE_B200_H
#define WILLAMETTE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status
 * Mirrors the variants of WillametteError (src/error.rs:9-57) that the hot
 * path can produce, plus the device-side failures a GPU adds. */
typedef enum wl_status {
    WL_OK = 0,
    WL_ERR_UNSUPPORTED_TENSOR_TYPE = 1, /* UnsupportedTensorType(u32), error.rs:29 */
    WL_ERR_GGUF_PARSE = 2,              /* GgufParse(String), error.rs:14: shape/length/scale */
    WL_ERR_NOT_IMPLEMENTED = 3,         /* NotImplemented(String), error.rs:35: arms left to the CPU */
    WL_ERR_INVALID_ARGUMENT = 4,        /* NULL / misaligned pointer, size beyond a stated limit */
    WL_ERR_CUDA = 5,                    /* CUDA runtime error */
    WL_ERR_NO_DEVICE = 6,               /* no sm_100 device visible */
    WL_ERR_DEVICE_TIMEOUT = 7,          /* a bounded device-side wait gave up */
    WL_ERR_COMM = 8,                    /* multi-GPU peer setup / exchange failure */
    WL_ERR_INVALID_MAGIC = 9,           /* InvalidMagic(u32), error.rs:16 */
    WL_ERR_UNSUPPORTED_VERSION = 10,    /* UnsupportedVersion(u32), error.rs:19 */
    WL_ERR_UNSUPPORTED_ARCHITECTURE = 11, /* UnsupportedArchitecture(String), error.rs:22 */
    WL_ERR_MISSING_METADATA = 12,       /* MissingMetadata(Vec<String>), error.rs:25 */
    WL_ERR_TENSOR_OUT_OF_BOUNDS = 13    /* TensorOutOfBounds{..}, error.rs:40 */
} wl_status;

/* GGML type ids (src/gguf/types.rs:66-99). */
#define WL_GGML_F32 0u
#define WL_GGML_F16 1u
#define WL_GGML_Q4_0 2u
#define WL_GGML_Q8_0 8u
#define WL_GGML_Q4_K 12u
#define WL_GGML_Q6_K 14u
#define WL_GGML_I2_S 36u

/* Layout constants (src/gguf/tensor.rs:86-105, :141-175). */
#define WL_I2S_ELEMENTS_PER_BLOCK 128u
#define WL_I2S_PACKED_BYTES_PER_BLOCK 32u
#define WL_Q6K_ELEMENTS_PER_BLOCK 256u
#define WL_Q6K_BYTES_PER_BLOCK 210u
#define WL_Q8_0_ELEMENTS_PER_BLOCK 32u
#define WL_Q8_0_BYTES_PER_BLOCK 34u

/* Largest in_dim the I2_S kernels accept (its int32 partial sums stay exact
 * far beyond this; the bound keeps activations register-resident). */
#define WL_I2S_MAX_IN_DIM 65536u

/* TensorView (src/gguf/tensor.rs:21-54) as plain C.  shape is GGUF order,
 * innermost first: [in_dim, out_dim] for a 2-D weight.  For I2_S, data is
 * the packed-codes area only and scale_data the 32-byte trailing block whose
 * first 4 bytes are the little-endian f32 per-tensor scale. */
typedef struct wl_tensor_view {
    const char *name;          /* may be NULL; used in error messages */
    const uint64_t *shape;
    uint32_t n_dims;
    uint32_t ggml_type;        /* raw GGML type id */
    const uint8_t *data;
    size_t data_len;
    const uint8_t *scale_data; /* I2_S only, else NULL */
    size_t scale_len;
} wl_tensor_view;

/* ------------------------------------------------------------------ library */
const char *wl_version(void);
/* Message of the last failure on this thread ("" if none). */
const char *wl_last_error(void);
/* Raw GGML type carried by the last WL_ERR_UNSUPPORTED_TENSOR_TYPE. */
uint32_t wl_last_error_tensor_type(void);
/* Select the CUDA device for this process (default: 0 on first use).
 * Fails with WL_ERR_NO_DEVICE unless the device is compute capability 10.x. */
int wl_init(int device);
/* Free every cached device copy of host weights. */
int wl_release_weights(void);
/* Device-side error word (bit 0: a bounded wait timed out; bit 1: a
 * tensor-parallel peer never arrived).  Synchronises the device, then reads
 * and clears it.  Includes the status word of wl_dev_i2s_matvec_f32_noalloc
 * on the calling thread's current device; when only that entry point has run
 * in the process, this call allocates nothing either. */
int wl_device_status(uint32_t *flags);
/* Limit of every bounded device-side wait (TMA stage waits, peer and flag
 * waits, grid barriers) on the current device, in ns; default 2 s, accepted
 * range [1 us, 600 s].  A wait that runs out sets bit 0 (or bit 1 for a peer
 * wait) of the device status word and its kernel returns; nothing hangs.
 * Synchronises the device; call it outside stream capture.  No counterpart
 * in the reference (its CPU path has no device waits). */
int wl_set_wait_limit_ns(uint64_t ns);
/* Enqueue on `stream` a bounded device-side wait until the 32-bit word at
 * `flag` (device or mapped host memory, 4-byte aligned) reaches `target`
 * (wrap-around compare).  Work queued after it runs once the word is there,
 * or once the wait limit ran out, which sets bit 0 of the device status word.
 * The same wait the tensor-parallel kernels use for their peers, exposed for
 * callers that order GPU work after a word another agent writes.  No
 * counterpart in the reference. */
int wl_dev_wait_flag(const uint32_t *flag, uint32_t target, void *stream);

/* ------------------------------------------------- host-buffer entry points */

/* bitlinear_i2s_matvec_f32 (src/model/bitlinear.rs:67), x86 dispatch
 * target bitlinear_i2s_matvec_f32_sse2_i8 (src/model/bitlinear_sse2.rs:313):
 * per-vector absmax int8 quantisation of input, exact int32 ternary dot per
 * row, output[j] = (w_scale * act_scale) * (float)acc[j].  Validation as
 * bitlinear_sse2.rs:129-177 (data_len >= in_dim/4*out_dim) and
 * tensor.rs:278-309 (finite scale). */
int wl_bitlinear_i2s_matvec_f32(const wl_tensor_view *weight, const float *input,
                                size_t input_len, float *output, size_t output_len);

/* As wl_bitlinear_i2s_matvec_f32, also returning the parity intermediates:
 * acc_out[out_dim] int32 row dots, act_scale_out[1], act_q_out[in_dim]
 * (each may be NULL). */
int wl_bitlinear_i2s_matvec_f32_dbg(const wl_tensor_view *weight, const float *input,
                                    size_t input_len, float *output, size_t output_len,
                                    int32_t *acc_out, float *act_scale_out, int8_t *act_q_out);

/* The reference's dispatch choice (src/model/dispatch.rs:47-71 Kernel) for
 * bitlinear_i2s_matvec_f32 (bitlinear.rs:67-142), for a caller whose host or
 * build does not take the x86 default:
 *   WL_I2S_KERNEL_SCALAR      Kernel::Scalar -> bitlinear_i2s_matvec_f32_scalar
 *                             (bitlinear.rs:146-242)
 *   WL_I2S_KERNEL_NEON        Kernel::AArch64Neon: no GPU arm, returns
 *                             WL_ERR_NOT_IMPLEMENTED (keep the CPU kernel)
 *   WL_I2S_KERNEL_SSE2_I8     Kernel::X86Sse2, the default build: same as
 *                             wl_bitlinear_i2s_matvec_f32
 *   WL_I2S_KERNEL_SCALAR_LUT  Kernel::X86Sse2ScalarLut -> bitlinear_i2s_matvec_f32_lut_scalar
 *                             (bitlinear_lut.rs:59-131)
 *   WL_I2S_KERNEL_SSE2_F32    Kernel::X86Sse2 in a --cfg willamette_sse2_f32 build ->
 *                             bitlinear_i2s_matvec_f32_sse2 (bitlinear_sse2.rs:89-124)
 * The f32-activation kernels reproduce that kernel's f32 summation order bit
 * for bit (results differ from the int8 default's); validation as that
 * kernel (scalar and LUT want data_len == in_dim/4 * out_dim). */
#define WL_I2S_KERNEL_SCALAR 0u
#define WL_I2S_KERNEL_NEON 1u
#define WL_I2S_KERNEL_SSE2_I8 2u
#define WL_I2S_KERNEL_SCALAR_LUT 3u
#define WL_I2S_KERNEL_SSE2_F32 4u
int wl_bitlinear_i2s_matvec_f32_kernel(const wl_tensor_view *weight, const float *input,
                                       size_t input_len, float *output, size_t output_len,
                                       uint32_t kernel);

/* Prefill over m tokens: the reference runs bitlinear_i2s_matvec_f32 once
 * per token (src/model/generate.rs:241-250, src/model/multi_forward.rs:106-110),
 * i.e. per-token absmax quantisation; here one int8 tensor-core GEMM.
 * input is m x in_dim, output m x out_dim, row-major.  acc_out optional. */
int wl_bitlinear_i2s_gemm_f32(const wl_tensor_view *weight, const float *input, size_t m,
                              float *output, int32_t *acc_out);

/* linear_matvec_f32 (src/model/linear.rs:11): I2_S, Q8_0 (linear.rs:171,
 * AVX2 row order q8_0_simd.rs:72) and Q6_K (linear.rs:43, SSE2 row order
 * q6_k_sse2.rs:46) arms.  F16 / Q4_0 / Q4_K return WL_ERR_NOT_IMPLEMENTED;
 * other types WL_ERR_UNSUPPORTED_TENSOR_TYPE (linear.rs:23). */
int wl_linear_matvec_f32(const wl_tensor_view *weight, const float *input, size_t input_len,
                         float *output, size_t output_len);

/* compute_logits (src/model/lm_head.rs:29) for Q6_K and Q8_0 tables:
 * logits[v] = dot_row(row_v, final_hidden), bit-identical to the
 * reference's x86 row dot.  F16 / Q4_0 / Q4_K tables return
 * WL_ERR_NOT_IMPLEMENTED. */
int wl_compute_logits(const float *final_hidden, size_t hidden_len,
                      const wl_tensor_view *token_embd, uint32_t embedding_length,
                      uint32_t vocab_size, float *logits, size_t logits_len);

/* argmax (src/model/lm_head.rs:161): first index of the maximum, strict
 * '>' scan (ties -> lowest id; NaN never wins unless at index 0).  *out_id
 * = -1 for an empty slice (the reference's None). */
int wl_argmax(const float *logits, size_t len, int64_t *out_id);

/* Greedy next token for a batch of hidden rows: compute_logits + argmax
 * fused (sampler.rs:133-136 greedy short-circuit, generate.rs:166-169).
 * hidden is batch x embedding_length; token_ids[batch]; logits (optional,
 * batch x vocab_size) receives the full logit rows. */
int wl_lm_head_greedy(const float *hidden, size_t batch, const wl_tensor_view *token_embd,
                      uint32_t embedding_length, uint32_t vocab_size, uint32_t *token_ids,
                      float *logits);

/* ------------------------------------------------ device-pointer entry points
 * All asynchronous on `stream` (a cudaStream_t; NULL = legacy default
 * stream).  Device buffers must be 16-byte aligned. */

/* One of the f32-activation kernels of wl_bitlinear_i2s_matvec_f32_kernel
 * (WL_I2S_KERNEL_SCALAR, _SSE2_F32 or _SCALAR_LUT) on device buffers:
 * y[out_dim] from x[in_dim] and the packed weight. */
int wl_dev_i2s_matvec_f32act(const uint8_t *packed, float w_scale, uint32_t in_dim,
                             uint32_t out_dim, const float *x, float *y, uint32_t kernel,
                             void *stream);

/* rms_norm_f32 (src/model/primitives.rs:227-255) of one f32 vector, bit
 * for bit: mean = sum(x[i] * x[i]) / n with the sum in the reference's
 * sequential order, out = (x * (1 / sqrt(mean + eps))) * w.  The norm in
 * front of every BitLinear of the decode step (exact mode) uses the same
 * arithmetic.  n a multiple of 4, at most WL_RMS_NORM_MAX_N; n == 0 does
 * nothing.  out must not overlap x. */
#define WL_RMS_NORM_MAX_N 16384u
int wl_dev_rms_norm_f32(const float *x, const float *w, uint32_t n, float eps, float *out,
                        void *stream);

/* softmax_inplace (src/model/attention.rs:45-73) of one f32 vector, in
 * place, bit for bit: exp is the reference's f32::exp (the C library's expf:
 * glibc's algorithm, restated), the sum in the reference's sequential order.
 * The attention of the decode step (exact mode) uses the same arithmetic.
 * n at most WL_SOFTMAX_MAX_N; n == 0 does nothing. */
#define WL_SOFTMAX_MAX_N 16384u
int wl_dev_softmax_f32(float *x, uint32_t n, void *stream);

/* Per-row absmax int8 quantisation (bitlinear_sse2.rs:285-304) of an
 * m x n f32 matrix: q (m x n int8), act_scale (m f32). */
int wl_dev_quantize_absmax_i8(const float *x, uint32_t n, uint32_t m, int8_t *q,
                              float *act_scale, void *stream);

/* Up to WL_I2S_MAX_FUSED weights of equal in_dim sharing one quantised
 * input (e.g. Q/K/V or gate/up), one launch: y_i[out_dim_i] =
 * (w_scale_i * act_scale[0]) * acc.  acc_i may be NULL. */
#define WL_I2S_MAX_FUSED 4
#define WL_I2S_NO_CODE3 1u /* flags: the weight holds no 0b11 code (wl_dev_i2s_scan_code3) */
typedef struct wl_i2s_dev_weight {
    const uint8_t *packed; /* out_dim x in_dim/4 bytes, device */
    float w_scale;
    uint32_t out_dim;
    float *y;              /* device, out_dim f32 */
    int32_t *acc;          /* device, out_dim i32, or NULL */
    uint32_t flags;        /* 0, or WL_I2S_NO_CODE3 (skips the per-row code-3 check) */
} wl_i2s_dev_weight;
int wl_dev_i2s_matvec(const wl_i2s_dev_weight *weights, uint32_t n_weights, uint32_t in_dim,
                      const int8_t *q, const float *act_scale, void *stream);

/* As wl_dev_i2s_matvec, but from the f32 input: every CTA quantises x itself
 * (bitlinear_sse2.rs:285-304, same IEEE steps), so one kernel per BitLinear
 * (or per fused Q/K/V or gate/up group).  in_dim <= 8192. */
int wl_dev_i2s_matvec_fused_f32(const wl_i2s_dev_weight *weights, uint32_t n_weights,
                                uint32_t in_dim, const float *x, void *stream);

/* Prefill GEMM from f32 activations: x is m x in_dim, y m x out_dim (acc
 * optional), row-major, device.  With WL_I2S_NO_CODE3 in flags it is one
 * tcgen05 int8 tensor-core GEMM (kind::i8, accumulators in tensor memory);
 * otherwise one exact matvec per token.  workspace: wl_i2s_gemm_workspace_bytes
 * bytes, 16-byte aligned (quantised activations, scales, row sums). */
size_t wl_i2s_gemm_workspace_bytes(uint32_t m, uint32_t in_dim);
int wl_dev_i2s_gemm_f32(const uint8_t *packed, float w_scale, uint32_t in_dim, uint32_t out_dim,
                        uint32_t m, const float *x, float *y, int32_t *acc, void *workspace,
                        uint32_t flags, void *stream);
/* Weights expanded once to int8 ternary values (t = code - 1, code 0b11 -> 0;
 * bitlinear.rs:43-50) in natural element order, out_dim x in_dim bytes -- 4x
 * the packed size, kept resident for prefill.  The GEMM over them is a
 * warp-specialised persistent tcgen05 kernel (TMA producer warp, MMA warp,
 * epilogue warps, double-buffered tensor-memory accumulators) and has no
 * code-0b11 restriction.  Same result as wl_dev_i2s_gemm_f32 (the reference's
 * per-token matvec, bit for bit). */
size_t wl_i2s_expanded_bytes(uint32_t in_dim, uint32_t out_dim);
int wl_dev_i2s_expand(const uint8_t *packed, uint32_t in_dim, uint32_t out_dim, int8_t *ternary,
                      void *stream);
/* workspace: wl_i2s_gemm_workspace_bytes(m, in_dim) bytes, 16-byte aligned. */
int wl_dev_i2s_gemm_s8_f32(const int8_t *ternary, float w_scale, uint32_t in_dim,
                           uint32_t out_dim, uint32_t m, const float *x, float *y, int32_t *acc,
                           void *workspace, void *stream);

/* *found (device u32) = 1 if the packed tensor contains a 0b11 code, else 0. */
int wl_dev_i2s_scan_code3(const uint8_t *packed, size_t bytes, uint32_t *found, void *stream);

/* Many independent BitLinear matvecs in one persistent launch (sustained HBM
 * streaming).  Ops sharing an input pointer share one quantisation.  The plan
 * holds the device-side descriptors and scratch; runs are asynchronous.
 * 512 <= in_dim <= 65536 per op. */
typedef struct wl_i2s_stream_op {
    const uint8_t *packed; /* device */
    float w_scale;
    uint32_t in_dim, out_dim;
    const float *x;        /* device f32 input */
    float *y;              /* device f32 output */
    int32_t *acc;          /* device, or NULL */
    uint32_t flags;        /* WL_I2S_NO_CODE3 or 0 */
    uint32_t row_off;      /* tensor parallel: this slice's first row in y (else 0) */
} wl_i2s_stream_op;
typedef struct wl_i2s_stream_plan wl_i2s_stream_plan;
int wl_i2s_stream_plan_create(const wl_i2s_stream_op *ops, uint32_t n_ops,
                              wl_i2s_stream_plan **plan);
int wl_dev_i2s_stream_run(wl_i2s_stream_plan *plan, void *stream);
int wl_i2s_stream_plan_destroy(wl_i2s_stream_plan *plan);

/* Quantise x then matvec (the two kernels chained with programmatic
 * dependent launch).  q_scratch: in_dim int8, scale_scratch: 1 f32. */
int wl_dev_i2s_matvec_f32(const uint8_t *packed, float w_scale, uint32_t in_dim,
                          uint32_t out_dim, const float *x, float *y, int8_t *q_scratch,
                          float *scale_scratch, void *stream);

/* Same result as wl_dev_i2s_matvec_f32, but the library allocates nothing
 * and the caller passes no scratch: the int8 activations and their scale live
 * in a static device array of the library (about 16 KB per GPU, held by every
 * GPU that loads the library until the process exits).  For callers that
 * cannot call cudaMalloc -- a serving engine that has already reserved the
 * device memory for its own pools, or a latency-critical decode loop where
 * cudaMalloc/cudaFree would synchronise the device.  No counterpart in the
 * reference (its CPU path needs no device memory).
 * - in_dim must be <= WL_NOALLOC_MAX_IN_DIM (else WL_ERR_INVALID_ARGUMENT).
 * - The first call on each device resolves the array's address and sets
 *   kernel attributes; make that first call before any stream capture.
 * - All calls share the one array: calls that overlap on the GPU (other
 *   streams, other host threads) race and must be serialised by the caller.
 * - A bounded wait that runs out inside the kernel is reported by
 *   wl_device_status on the same device (its status word sits in the same
 *   static array).
 * - The array's address belongs to the CUDA context current at the call;
 *   after cudaDeviceReset or under another current context it is resolved
 *   again (again allocating nothing). */
#define WL_NOALLOC_MAX_IN_DIM 16384u
int wl_dev_i2s_matvec_f32_noalloc(const uint8_t *packed, float w_scale, uint32_t in_dim,
                                  uint32_t out_dim, const float *x, float *y, void *stream);

/* ------------------------------------------------ tensor parallel (one GPU per process)
 * North star: BitLinear output rows split across the GPUs of one box with an
 * all-gather; the lm-head split by vocab rows with a (max, index) reduction.
 * Here the kernels themselves store their outputs into every rank's
 * symmetric block over NVLink (CUDA IPC) and signal arrival counters there
 * (system-scope release/acquire); the consumer's kernel waits, bounded, on
 * its own memory.  Every rank must issue the same sequence of wl_tp_* calls.
 * Wait targets and key-slot sets are read on the device (from this rank's own
 * counters), so a sequence of wl_tp_* launches can be captured in a CUDA graph
 * and replayed.  Setup: wl_tp_create on every rank, exchange the WL_TP_HANDLE_BYTES handles
 * (any host channel), wl_tp_connect with all world handles in rank order. */
#define WL_TP_HANDLE_BYTES 64
typedef struct wl_tp_group wl_tp_group;
int wl_tp_create(int rank, int world, size_t sym_bytes, wl_tp_group **group,
                 uint8_t *handle_out);
int wl_tp_connect(wl_tp_group *group, const uint8_t *handles);
/* Device pointer at `offset` in this rank's symmetric region (NULL past its end). */
void *wl_tp_buffer(wl_tp_group *group, size_t offset);
int wl_tp_destroy(wl_tp_group *group);
/* Enqueue a wait until every rank's outputs so far are visible here. */
int wl_tp_wait(wl_tp_group *group, void *stream);
/* Row slice of up to WL_I2S_MAX_FUSED BitLinears sharing x: weights[j] holds
 * rows [row_offsets[j], row_offsets[j] + out_dim) of the full weight and its
 * y is the FULL output vector in the symmetric region; every rank ends up
 * with the complete y.  wait_for_input: the kernel first waits until every
 * rank has finished every earlier wl_tp_* op -- needed when x was gathered by
 * one of them, or when y overwrites a vector a peer may still be reading. */
int wl_tp_i2s_matvec_fused_f32(wl_tp_group *group, const wl_i2s_dev_weight *weights,
                               const uint32_t *row_offsets, uint32_t n_weights, uint32_t in_dim,
                               const float *x, int wait_for_input, void *stream);
/* A stream plan whose ops are row slices (wl_i2s_stream_op.row_off) with y in
 * the symmetric region; outputs are gathered on every rank.  It does not wait:
 * precede it with wl_tp_wait when its inputs were gathered. */
int wl_tp_i2s_stream_run(wl_tp_group *group, wl_i2s_stream_plan *plan, void *stream);
/* Vocab-sharded greedy lm-head: this rank holds rows [row_offset, row_offset +
 * vocab_shard) (repacked, wl_dev_q6k_repack); ids (batch <= 64) are the
 * global argmax with the reference's tie / NaN rules, on every rank.
 * scratch: wl_q6k_scratch_bytes(batch) bytes, zero before the first use. */
int wl_tp_q6k_lm_head_greedy(wl_tp_group *group, const uint8_t *packed_shard, uint32_t n_embd,
                             uint32_t vocab_shard, uint32_t row_offset, const float *hidden,
                             uint32_t batch, uint32_t *ids, void *scratch, void *stream);

/* ------------------------------------------------ BitNet b1.58 decode engine
 * Device-resident single-token forward with the reference's i8 KV cache and
 * greedy generation: forward_with_cache (src/model/cached_forward.rs:206-504)
 * and greedy_generate_with_cache (src/model/generate.rs:111-190) for the
 * BitNetSubNorm variant (RMSNorm, NEOX RoPE, GQA attention, attn_sub_norm,
 * relu^2 * up, ffn_sub_norm, tied Q6_K embedding / lm-head).  Weights are
 * copied to the device at create time; the caller keeps no device memory.
 * A decode step (lm-head, argmax, next forward) is replayed from a CUDA graph
 * and reads the token and position on the device. */
typedef struct {
    uint32_t n_layers, n_embd, n_heads, n_kv_heads, head_dim, n_ff, vocab, n_rot, max_seq;
    float eps, freq_base;
    /* 0: sums (RMSNorm, softmax, attention-weighted V) as parallel trees;
     * 1: every sum in the reference's sequential order (slower).  Either way
     * the per-element arithmetic is the reference's. */
    uint32_t exact;
    /* 0: one kernel per operation (PDL chain, the faster engine today);
     * 1: the whole forward as one persistent cooperative kernel (grid
     * barriers between phases, weights prefetched into shared memory).
     * Same arithmetic. */
    uint32_t persistent;
    /* KV cache layout.  0: the reference's per-token absmax int8 rows with
     * one f32 scale each (kv_cache.rs:245-259), the layout every parity
     * claim is made on.  1: IEEE binary16 rows (round to nearest even from
     * the f32 K after RoPE and V; read back exactly), the f16 cache of
     * benchmark config 2 -- not a reference layout, so its results are
     * compared with the oracle's f16 variant only.  The BitNet engine only
     * (the Llama batch engine requires 0); runs per operation (`persistent`
     * is ignored). */
    uint32_t kv_f16;
} wl_bitnet_config;

typedef struct {
    const uint8_t *const *w;   /* n_layers * 7 host I2_S packed: q, k, v, o, gate, up, down */
    const float *w_scale;      /* n_layers * 7 per-tensor scales */
    const float *norms;        /* per layer: attn_norm[E], attn_sub_norm[E], ffn_norm[E],
                                  ffn_sub_norm[n_ff] */
    const float *output_norm;  /* E */
    const uint8_t *token_embd; /* vocab Q6_K rows (GGUF layout), tied lm-head */
} wl_bitnet_weights;

typedef struct wl_bitnet wl_bitnet;
int wl_bitnet_create(const wl_bitnet_config *cfg, const wl_bitnet_weights *weights,
                     wl_bitnet **out);
/* Tensor-parallel engine, one per rank of a connected group (every rank
 * passes the same config and full host weights): each BitLinear's output
 * rows are split evenly over the ranks and gathered by the matvec kernels
 * themselves (peer stores over NVLink, bounded in-kernel waits); norms,
 * RoPE, attention and the KV cache are replicated; the lm-head is split by
 * vocabulary rows and reduced with (max, lowest index) keys.  The engine
 * places its gathered vectors at the start of the group's caller region,
 * which must hold wl_bitnet_tp_sym_bytes(cfg) bytes and is the engine's
 * while it lives.  Results equal the single-GPU engine's bit for bit.
 * Every rank must make the same sequence of calls.  `persistent` must be 0. */
int wl_bitnet_create_tp(const wl_bitnet_config *cfg, const wl_bitnet_weights *weights,
                        wl_tp_group *group, wl_bitnet **out);
size_t wl_bitnet_tp_sym_bytes(const wl_bitnet_config *cfg);
int wl_bitnet_destroy(wl_bitnet *model);
/* Empty the KV cache (position 0). */
int wl_bitnet_reset(wl_bitnet *model);
uint32_t wl_bitnet_position(const wl_bitnet *model);
/* 1 when the forward runs as the persistent kernel (it needs one CTA's shared
 * memory on every SM), 0 when it runs per operation. */
int wl_bitnet_uses_persistent_kernel(const wl_bitnet *model);
/* forward_with_cache (cached_forward.rs:131-149): position must equal the
 * cache position; out_hidden (host, n_embd, may be NULL) = output_norm(hidden). */
int wl_bitnet_forward(wl_bitnet *model, uint32_t token, uint32_t position, float *out_hidden);
/* Forward each token in order from the current position (the prompt loop of
 * generate.rs:147-160). */
int wl_bitnet_prefill(wl_bitnet *model, const uint32_t *tokens, uint32_t n);
/* The decode loop of generate.rs:165-187 from the last forward's hidden:
 * n_new greedy ids (host); out_hiddens (host, n_new x n_embd, optional): the
 * hidden each id was chosen from; device_ms (optional): device time of the
 * loop (CUDA events on the engine's stream). */
int wl_bitnet_decode(wl_bitnet *model, uint32_t n_new, uint32_t *out_ids, float *out_hiddens,
                     float *device_ms);
/* greedy_generate_with_cache: reset, prefill, decode. */
int wl_bitnet_generate(wl_bitnet *model, const uint32_t *prompt, uint32_t n_prompt,
                       uint32_t n_new, uint32_t *out_ids, float *out_hiddens);

/* Q6_K lm-head.  The raw GGUF rows (vocab x n_embd/256 x 210 bytes) are
 * repacked once into the device layout (wl_q6k_packed_bytes bytes). */
size_t wl_q6k_packed_bytes(uint32_t n_embd, uint32_t vocab);
int wl_dev_q6k_repack(const uint8_t *raw, uint32_t n_embd, uint32_t vocab, uint8_t *packed,
                      void *stream);
/* Logits (optional, batch x vocab) and greedy ids (batch) for batch hidden
 * rows.  scratch: wl_q6k_scratch_bytes(batch) bytes, zero before the first
 * call; every call leaves it zero again. */
size_t wl_q6k_scratch_bytes(uint32_t batch);
int wl_dev_q6k_lm_head(const uint8_t *packed, uint32_t n_embd, uint32_t vocab,
                       const float *hidden, uint32_t batch, float *logits, uint32_t *ids,
                       void *scratch, void *stream);

/* Q8_0 matvec / lm-head rows (q8_0_simd.rs:72-104 order), after a one-time
 * repack (wl_q8_0_packed_bytes).  Non-finite block scales are rejected by
 * the host entry points before upload (q8_0.rs:25-33). */
size_t wl_q8_0_packed_bytes(uint32_t in_dim, uint32_t out_dim);
int wl_dev_q8_0_repack(const uint8_t *raw, uint32_t in_dim, uint32_t out_dim, uint8_t *packed,
                       void *stream);
int wl_dev_q8_0_matvec(const uint8_t *packed, uint32_t in_dim, uint32_t out_dim,
                       const float *x, float *y, void *stream);

/* ------------------------------------- batched Q8_0 Llama decode engine
 * n_seqs independent sequences decoded in lock step, one token per sequence
 * per step, each with its own i8 KV cache and position.  Per sequence this
 * is the reference's greedy_generate_with_cache (src/model/generate.rs:
 * 111-190) over forward_with_cache (src/model/cached_forward.rs:206-504) in
 * its VanillaLlama variant: RMSNorm, Norm RoPE (pairs 2j, 2j+1), GQA
 * attention, no sub-norms, silu(gate) * up, every linear Q8_0
 * (q8_0_matvec_f32, src/model/linear.rs:171-224) and a tied Q8_0 embedding /
 * lm-head (compute_logits, src/model/lm_head.rs:103; argmax :161-174).
 * The config's `exact` selects the reference's summation order everywhere
 * (bit-exact linears); 0 contracts the Q8_0 products into FMAs and sums
 * norms / softmax as trees.  `persistent` is ignored. */
typedef struct {
    const uint8_t *const *w;   /* n_layers * 7 GGUF Q8_0 rows (34-byte blocks):
                                  q, k, v, o, gate, up, down */
    const float *attn_norm;    /* n_layers * n_embd */
    const float *ffn_norm;     /* n_layers * n_embd */
    const float *output_norm;  /* n_embd */
    const uint8_t *token_embd; /* vocab GGUF Q8_0 rows, tied lm-head */
} wl_llama_weights;

typedef struct wl_llama_batch wl_llama_batch;
int wl_llama_batch_create(const wl_bitnet_config *cfg, const wl_llama_weights *weights,
                          uint32_t n_seqs, wl_llama_batch **out);
int wl_llama_batch_destroy(wl_llama_batch *batch);
/* Empty every sequence's KV cache. */
int wl_llama_batch_reset(wl_llama_batch *batch);
uint32_t wl_llama_batch_position(const wl_llama_batch *batch, uint32_t seq);
/* Attention CTAs per (head or KV head, sequence) the engine chose. */
uint32_t wl_llama_batch_attention_splits(const wl_llama_batch *batch);
/* Tokens each CTA of the batched Q8_0 linears covers (1, 4, 8 or 32; 0, the
 * default: chosen per launch from the row tiles and the SM count).  A tuning
 * knob; results do not depend on it. */
int wl_llama_batch_set_tokens_per_cta(wl_llama_batch *batch, uint32_t tokens);
/* Forward sequence b's tokens tokens[offsets[b] .. offsets[b+1]) from its
 * current position (the prompt loop of generate.rs:147-160), all sequences in
 * lock step; a sequence with no tokens idles. */
int wl_llama_batch_prefill(wl_llama_batch *batch, const uint32_t *tokens, const uint32_t *offsets);
/* n_new greedy steps for every sequence (each must have been prefilled):
 * out_ids[step * n_seqs + b]; out_hiddens (optional, [n_new][n_seqs][n_embd]):
 * the hiddens the ids were chosen from; device_ms (optional): device time of
 * the loop. */
int wl_llama_batch_decode(wl_llama_batch *batch, uint32_t n_new, uint32_t *out_ids,
                          float *out_hiddens, float *device_ms);
/* Reset, prefill every sequence's (non-empty) prompt, decode n_new. */
int wl_llama_batch_generate(wl_llama_batch *batch, const uint32_t *tokens, const uint32_t *offsets,
                            uint32_t n_new, uint32_t *out_ids, float *out_hiddens);

/* ------------------------------------------------------------ GGUF models
 * GgufFile::parse (src/gguf/reader.rs:120-415) over the caller's bytes -- the
 * reference maps the file and parses the mapping; pass that mapping here.
 * Zero-copy: tensor views point into `data`, which must outlive the handle.
 * Errors: WL_ERR_INVALID_MAGIC, WL_ERR_UNSUPPORTED_VERSION,
 * WL_ERR_TENSOR_OUT_OF_BOUNDS, else WL_ERR_GGUF_PARSE (same checks, same
 * order as the reference).  Host code only: no GPU is touched. */
typedef struct wl_gguf wl_gguf;
int wl_gguf_open(const uint8_t *data, size_t len, wl_gguf **out);
int wl_gguf_close(wl_gguf *gguf);
uint32_t wl_gguf_version(const wl_gguf *gguf);
uint64_t wl_gguf_alignment(const wl_gguf *gguf);
uint64_t wl_gguf_tensor_count(const wl_gguf *gguf);
/* Tensor i in directory order, or by name (WL_ERR_MISSING_METADATA if
 * absent), as a view valid while the handle lives: data = the packed bytes
 * (byte length of reader.rs:688-770), scale_data = the I2_S 32-byte trailing
 * block (NULL for other types). */
int wl_gguf_tensor(const wl_gguf *gguf, uint64_t index, wl_tensor_view *out);
int wl_gguf_find_tensor(const wl_gguf *gguf, const char *name, wl_tensor_view *out);
/* Metadata (GgufValue::as_u64 / as_f32 / as_str, reader.rs:46-90):
 * WL_ERR_MISSING_METADATA when the key is absent or of another kind.
 * wl_gguf_get_str's pointer lives as long as the handle. */
int wl_gguf_get_u64(const wl_gguf *gguf, const char *key, uint64_t *out);
int wl_gguf_get_f32(const wl_gguf *gguf, const char *key, float *out);
int wl_gguf_get_str(const wl_gguf *gguf, const char *key, const char **out);
/* Element count of an array value (0 if absent or not an array). */
uint64_t wl_gguf_array_len(const wl_gguf *gguf, const char *key);
/* ModelConfig::from_gguf_metadata (src/model/config.rs:61-260): the
 * architecture (general.architecture: bitnet-b1.58 / bitnet-25 / bitnet ->
 * variant 0, BitNetSubNorm; llama -> variant 1, VanillaLlama) and its
 * dimensions into a wl_bitnet_config; max_seq = context_length. */
int wl_gguf_model_config(const wl_gguf *gguf, wl_bitnet_config *cfg, uint32_t *variant);
/* ModelGraph::from_gguf (src/model/graph.rs:95-240) straight to the device:
 * the BitNet engine from a BitNet-family file (I2_S linears with their
 * trailing scales, F32 norms, the tied embedding as Q6_K -- the reference's
 * embedding-q6-k artifact; an F16 embedding is WL_ERR_NOT_IMPLEMENTED), or the
 * batched Llama engine from a llama file (Q8_0 linears and tied Q8_0
 * token_embd; other linear types or a separate output.weight are
 * WL_ERR_NOT_IMPLEMENTED).  max_seq 0 = context_length. */
int wl_bitnet_create_from_gguf(const wl_gguf *gguf, uint32_t max_seq, uint32_t exact,
                               uint32_t persistent, wl_bitnet **out);
int wl_llama_batch_create_from_gguf(const wl_gguf *gguf, uint32_t n_seqs, uint32_t max_seq,
                                    uint32_t exact, wl_llama_batch **out);

#ifdef __cplusplus
}
#endif

#endif /* WILLAMETTE_B200_H */
