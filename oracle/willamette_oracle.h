/*
 * willamette_oracle.h -- CPU oracle for the BitLinear hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the
 * reference's x86 code path (Rust crate project-willamette v0.14.0), used
 * as the parity checker for the CUDA library and as the timed CPU
 * baseline.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference leg may load it.  The product library
 * never links or calls it.
 *
 * Parity pin: the reference is Rust and no Rust toolchain exists on the
 * build or GPU machines, so it cannot be executed.  The restatement is
 * pinned by the reference's own known-answer unit tests (transcribed from
 * its test sources into tests/test_oracle_kats.py).
 *
 * Every function names the reference file:line it follows.  All f32
 * arithmetic is compiled with -ffp-contract=off (Rust never contracts a*b+c
 * into an FMA) and uses the same SSE2/AVX2 intrinsics, in the same
 * reduction order, as the reference's x86 kernels.
 *
 * Status codes: 0 = ok, negative = the reference would return Err(..).
 */
#ifndef WILLAMETTE_ORACLE_H
#define WILLAMETTE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* src/model/primitives.rs:61-88 */
float or_f16_to_f32(uint16_t bits);
/* IEEE binary32 -> binary16, round-to-nearest-even (half 2.7.1 f16::from_f32). */
uint16_t or_f32_to_f16(float value);

/* src/model/bitlinear.rs:43-50 */
int8_t or_ternary_from_code(uint8_t code);

/* src/model/bitlinear.rs:146-242 (scalar two-accumulator f32 reference). */
int or_i2s_matvec_scalar(const uint8_t *packed, size_t packed_len, float scale,
                         uint32_t in_dim, uint32_t out_dim, const float *x,
                         float *y);

/* src/model/bitlinear_sse2.rs:285-304 (per-vector absmax int8 quantiser).
 * Returns the activation scale (max_abs / 127, or 1.0 for an all-zero x). */
float or_quantize_absmax_i8(const float *x, size_t n, int8_t *q);

/* src/model/bitlinear_sse2.rs:313-342 (x86 default: int8 activations).
 * acc_out (out_dim i32), act_scale_out (1 f32) and act_q_out (in_dim i8)
 * are optional debug outputs (NULL to skip). */
int or_i2s_matvec_sse2_i8(const uint8_t *packed, size_t packed_len,
                          float w_scale, uint32_t in_dim, uint32_t out_dim,
                          const float *x, float *y, int32_t *acc_out,
                          float *act_scale_out, int8_t *act_q_out);

/* Prefill "GEMM" as the reference runs it: one sse2_i8 matvec per token
 * (src/model/generate.rs:241-250, src/model/multi_forward.rs:106-110).
 * X is m x in_dim row-major, Y is m x out_dim, acc_out optional m x out_dim,
 * act_scale_out optional m. */
int or_i2s_gemm_rows(const uint8_t *packed, size_t packed_len, float w_scale,
                     uint32_t in_dim, uint32_t out_dim, uint32_t m,
                     const float *x, float *y, int32_t *acc_out,
                     float *act_scale_out, int n_threads);

/* src/model/bitlinear_sse2.rs:89-124 + :206-255 (f32 mask-add kernel). */
int or_i2s_matvec_sse2_f32(const uint8_t *packed, size_t packed_len,
                           float scale, uint32_t in_dim, uint32_t out_dim,
                           const float *x, float *y);

/* src/model/bitlinear_lut.rs:59-131 (scalar 256-entry LUT kernel). */
int or_i2s_matvec_lut(const uint8_t *packed, size_t packed_len, float scale,
                      uint32_t in_dim, uint32_t out_dim, const float *x,
                      float *y);

/* src/model/bitlinear.rs:247-299 */
int or_i2s_unpack_row(const uint8_t *packed, size_t packed_len,
                      uint32_t in_dim, uint32_t out_dim, uint32_t row,
                      int8_t *out);

/* src/model/q6_k.rs:59-69 (for_each_weight :25-57). n = values. */
int or_q6k_dequantize_row(const uint8_t *row, size_t row_len, float *out,
                          size_t n);
/* src/model/q6_k.rs:84-96 */
int or_q6k_dot_row_scalar(const uint8_t *row, size_t row_len, const float *x,
                          size_t n, float *out);
/* src/model/q6_k_sse2.rs:46-116 (the x86 dispatch target, q6_k.rs:71-82) */
int or_q6k_dot_row_sse2(const uint8_t *row, size_t row_len, const float *x,
                        size_t n, float *out);
/* src/model/q6_k.rs:232-238 (offline quantiser; used only to rebuild the
 * reference's Q6_K unit-test fixtures). */
int or_q6k_quantize_row(const float *in, size_t n, uint8_t *out,
                        size_t out_len);

/* src/model/q8_0.rs:35-48 */
int or_q8_0_dequantize_row(const uint8_t *row, size_t row_len, float *out,
                           size_t n);
/* src/model/q8_0.rs:72-85 */
int or_q8_0_dot_row_scalar(const uint8_t *row, size_t row_len, const float *x,
                           size_t n, float *out);
/* src/model/q8_0_simd.rs:72-104 (x86 hosts with AVX2, q8_0.rs:59-62) */
int or_q8_0_dot_row_avx2(const uint8_t *row, size_t row_len, const float *x,
                         size_t n, float *out);
/* src/model/q8_0_simd.rs:108-141 */
int or_q8_0_dot_row_sse2(const uint8_t *row, size_t row_len, const float *x,
                         size_t n, float *out);

/* src/model/linear.rs:171-224 (rayon over rows -> OpenMP over rows). */
int or_q8_0_matvec(const uint8_t *w, size_t w_len, uint32_t in_dim,
                   uint32_t out_dim, const float *x, float *y, int n_threads);

/* src/model/lm_head.rs:29-108.  ggml_type: 1 = F16, 8 = Q8_0, 14 = Q6_K.
 * Rows are independent (rayon); n_threads <= 0 uses all cores. */
int or_compute_logits(const float *hidden, uint32_t n_embd,
                      const uint8_t *w, size_t w_len, uint32_t ggml_type,
                      uint32_t vocab, float *logits, int n_threads);

/* src/model/lm_head.rs:161-174.  Returns -1 for an empty slice. */
int64_t or_argmax(const float *logits, size_t n);

/* ---- single-token decode step with the i8 KV cache (bitnet_forward.c) ----
 * BitNet b1.58 (ForwardVariant::BitNetSubNorm): RMSNorm, Q/K/V BitLinears,
 * NEOX RoPE, KV append (per-token absmax i8), attention, attn_sub_norm, O,
 * residual, ffn_norm, gate/up, relu^2 * up, ffn_sub_norm, down, residual;
 * output_norm after the last layer (src/model/cached_forward.rs:206-504). */
typedef struct {
    uint32_t n_layers, n_embd, n_heads, n_kv_heads, head_dim, n_ff, vocab, n_rot, max_seq;
    float eps, freq_base;
    /* ForwardVariant: 0 = BitNetSubNorm (sub-norms, relu^2, NEOX RoPE),
     * 1 = VanillaLlama (no sub-norms, SiLU, "normal" RoPE); cached_forward.rs:373-504 */
    uint32_t variant;
    uint32_t linear_type;  /* 0 = I2_S (w_scale used), 8 = Q8_0 */
    uint32_t embd_type;    /* tied embedding / lm-head: 14 = Q6_K, 8 = Q8_0 */
    /* 0: the reference's i8 KV cache; 1: binary16 K / V rows (round to nearest
     * even, read back exactly) -- not a reference layout: the checker of the
     * library's kv_f16 engine option.  k_q / v_q then hold uint16 values. */
    uint32_t kv_f16;
} or_bitnet_config;

typedef struct {
    const uint8_t *const *w;  /* n_layers * 7 packed I2_S: q, k, v, o, gate, up, down */
    const float *w_scale;     /* n_layers * 7 */
    const float *norms;       /* per layer: attn_norm[E], attn_sub_norm[E], ffn_norm[E],
                                 ffn_sub_norm[F] */
    const float *output_norm; /* E */
    const uint8_t *token_embd; /* vocab Q6_K rows (tied embedding / lm-head) */
} or_bitnet_weights;

typedef struct { /* src/model/kv_cache.rs layout, one slab per layer */
    int8_t *k_q, *v_q; /* n_layers * max_seq * kv_dim (uint16 each with kv_f16) */
    float *k_s, *v_s;  /* n_layers * max_seq */
    uint32_t pos;
} or_kv_cache;

/* primitives.rs:227-254 */
void or_rms_norm(const float *x, const float *w, float eps, float *out, uint32_t n);
/* primitives.rs:283-345, RopeType::Neox on one head (head_dim >= n_rot) */
void or_rope_neox(float *x, uint32_t n_rot, uint32_t position, float freq_base);
/* primitives.rs:316-327, RopeType::Norm (pairs 2j, 2j+1) */
void or_rope_norm(float *x, uint32_t n_rot, uint32_t position, float freq_base);
/* ffn.rs:45-49 */
void or_silu_inplace(float *x, uint32_t n);
/* attention.rs:45-73 */
void or_softmax_inplace(float *x, uint32_t n);
/* kv_cache.rs:245-259 (one token's K or V) */
void or_kv_quantise(const float *x, uint32_t n, int8_t *q, float *scale);
/* forward_with_cache (cached_forward.rs:206-259): out = output_norm(hidden). */
int or_bitnet_forward(const or_bitnet_config *c, const or_bitnet_weights *w, or_kv_cache *kv,
                      uint32_t token, uint32_t position, float *out, int n_threads);
/* greedy_generate_with_cache (generate.rs:111-190): prefill the prompt token by
 * token, then n_new greedy ids.  hiddens (optional, n_new x E): the final
 * hidden each id was chosen from. */
int or_bitnet_generate(const or_bitnet_config *c, const or_bitnet_weights *w, or_kv_cache *kv,
                       const uint32_t *prompt, uint32_t n_prompt, uint32_t n_new,
                       uint32_t *out_ids, float *hiddens, int n_threads);

#ifdef __cplusplus
}
#endif

#endif /* WILLAMETTE_ORACLE_H */
