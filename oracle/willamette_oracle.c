/*
 * willamette_oracle.c -- CPU oracle for the BitLinear hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see willamette_oracle.h).  A plain-C
 * restatement of the reference's x86 kernels; every function cites the
 * Rust source it follows.  Build with -O3 -msse2 -ffp-contract=off and no
 * fast-math (oracle/Makefile).  The product CUDA library never links this.
 */
#include "willamette_oracle.h"

#include <emmintrin.h>
#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define QK_I2_S 128
#define I2S_BLOCK_BYTES 32
#define Q6K_VALUES 256
#define Q6K_BYTES 210
#define Q8_0_VALUES 32
#define Q8_0_BYTES 34

static float bits_to_f32(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t f32_to_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* ------------------------------------------------------------------ f16 */

/* primitives.rs:61-88 -- hand-rolled binary16 -> binary32. */
float or_f16_to_f32(uint16_t bits) {
    uint32_t sign = (bits >> 15) & 0x1u;
    uint32_t exp = (bits >> 10) & 0x1Fu;
    uint32_t mantissa = bits & 0x3FFu;
    if (exp == 0) {
        if (mantissa == 0) return bits_to_f32(sign << 31);
        float m = (float)mantissa;
        float val = m * (1.0f / (float)(1u << 24));
        return sign ? -val : val;
    }
    if (exp == 0x1F) {
        return bits_to_f32((sign << 31) | (0xFFu << 23) | (mantissa << 13));
    }
    return bits_to_f32((sign << 31) | ((exp + (127 - 15)) << 23) | (mantissa << 13));
}

/* binary32 -> binary16 with round-to-nearest-even (IEEE 754), the rounding
 * the half crate's f16::from_f32 performs.  Used by the Q6_K quantiser
 * (q6_k.rs:225). */
uint16_t or_f32_to_f16(float value) {
    uint32_t x = f32_to_bits(value);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t mant = x & 0x7FFFFFu;
    if (exp == 0xFF) {
        if (mant) return (uint16_t)(sign | 0x7E00u | (mant >> 13));
        return (uint16_t)(sign | 0x7C00u);
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t h = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)h;
}

/* ------------------------------------------------------------------ I2_S */

/* bitlinear.rs:43-50 -- 00 -> -1, 01 -> 0, 10 -> +1, 11 -> 0. */
static inline int8_t code_to_ternary(uint8_t code) {
    static const int8_t map[4] = {-1, 0, 1, 0};
    return map[code & 3u];
}

int8_t or_ternary_from_code(uint8_t code) { return code_to_ternary(code); }

/* tensor.rs:278-309 -- the per-tensor scale must be finite. */
static int scale_ok(float s) { return isfinite(s) ? 0 : -1; }

/* bitlinear.rs:182-199 -- shape checks shared by the scalar and LUT paths
 * (which demand packed_len == in_dim/4 * out_dim exactly). */
static int i2s_shape_exact(size_t packed_len, uint32_t in_dim, uint32_t out_dim) {
    if (in_dim == 0 || in_dim % QK_I2_S != 0) return -1;
    if (packed_len != (size_t)(in_dim / 4) * out_dim) return -1;
    return 0;
}

/* bitlinear.rs:236-242 */
static inline void accumulate_code(float *pos, float *neg, uint8_t code, float x) {
    if (code == 0) *neg += x;
    else if (code == 2) *pos += x;
}

/* bitlinear.rs:146-242 */
int or_i2s_matvec_scalar(const uint8_t *packed, size_t packed_len, float scale,
                         uint32_t in_dim, uint32_t out_dim, const float *x,
                         float *y) {
    if (i2s_shape_exact(packed_len, in_dim, out_dim) || scale_ok(scale)) return -1;
    size_t bytes_per_row = in_dim / 4;
    uint32_t blocks = in_dim / QK_I2_S;
    for (uint32_t j = 0; j < out_dim; j++) {
        const uint8_t *row = packed + (size_t)j * bytes_per_row;
        float pos = 0.0f, neg = 0.0f;
        for (uint32_t bk = 0; bk < blocks; bk++) {
            const uint8_t *blk = row + (size_t)bk * I2S_BLOCK_BYTES;
            const float *xb = x + (size_t)bk * QK_I2_S;
            for (int gp = 0; gp < I2S_BLOCK_BYTES; gp++) {
                uint8_t b = blk[gp];
                accumulate_code(&pos, &neg, (b >> 6) & 3u, xb[gp]);
                accumulate_code(&pos, &neg, (b >> 4) & 3u, xb[gp + 32]);
                accumulate_code(&pos, &neg, (b >> 2) & 3u, xb[gp + 64]);
                accumulate_code(&pos, &neg, b & 3u, xb[gp + 96]);
            }
        }
        y[j] = scale * (pos - neg);
    }
    return 0;
}

/* bitlinear_sse2.rs:183-193 + :238-244 */
static void unpack_block(const uint8_t *blk, int8_t out[QK_I2_S]) {
    for (int gp = 0; gp < I2S_BLOCK_BYTES; gp++) {
        uint8_t b = blk[gp];
        out[gp] = code_to_ternary((b >> 6) & 3u);
        out[gp + 32] = code_to_ternary((b >> 4) & 3u);
        out[gp + 64] = code_to_ternary((b >> 2) & 3u);
        out[gp + 96] = code_to_ternary(b & 3u);
    }
}

/* bitlinear_sse2.rs:285-304.  Rust: max over |v| with strict '>', so NaN
 * never becomes the max; (v*inv).round() is round-half-away-from-zero
 * (roundf); clamp(-127,127) keeps NaN as NaN and `as i8` maps NaN to 0. */
float or_quantize_absmax_i8(const float *x, size_t n, int8_t *q) {
    float max_abs = 0.0f;
    for (size_t i = 0; i < n; i++) {
        float a = fabsf(x[i]);
        if (a > max_abs) max_abs = a;
    }
    if (max_abs == 0.0f) {
        memset(q, 0, n);
        return 1.0f;
    }
    float inv_scale = 127.0f / max_abs;
    for (size_t i = 0; i < n; i++) {
        float r = roundf(x[i] * inv_scale);
        if (isnan(r)) { q[i] = 0; continue; }
        if (r < -127.0f) r = -127.0f;
        if (r > 127.0f) r = 127.0f;
        q[i] = (int8_t)r;
    }
    return max_abs / 127.0f;
}

/* bitlinear_sse2.rs:353-386 -- compare-mask select, widen, madd with 1. */
static int32_t dot_i8_ternary(const int8_t w[QK_I2_S], const int8_t *act) {
    const __m128i ones = _mm_set1_epi8(1);
    const __m128i neg_ones = _mm_set1_epi8(-1);
    const __m128i zero = _mm_setzero_si128();
    const __m128i ones16 = _mm_set1_epi16(1);
    __m128i acc = _mm_setzero_si128();
    for (int i = 0; i + 16 <= QK_I2_S; i += 16) {
        __m128i wv = _mm_loadu_si128((const __m128i *)(w + i));
        __m128i xv = _mm_loadu_si128((const __m128i *)(act + i));
        __m128i pos = _mm_cmpeq_epi8(wv, ones);
        __m128i neg = _mm_cmpeq_epi8(wv, neg_ones);
        __m128i neg_x = _mm_sub_epi8(zero, xv);
        __m128i prod = _mm_or_si128(_mm_and_si128(xv, pos), _mm_and_si128(neg_x, neg));
        __m128i lo = _mm_srai_epi16(_mm_unpacklo_epi8(prod, prod), 8);
        __m128i hi = _mm_srai_epi16(_mm_unpackhi_epi8(prod, prod), 8);
        acc = _mm_add_epi32(acc, _mm_madd_epi16(lo, ones16));
        acc = _mm_add_epi32(acc, _mm_madd_epi16(hi, ones16));
    }
    int32_t lanes[4];
    _mm_storeu_si128((__m128i *)lanes, acc);
    return lanes[0] + lanes[1] + lanes[2] + lanes[3];
}

/* bitlinear_sse2.rs:129-177 -- the SSE2 validator accepts packed_len >=
 * in_dim/4 * out_dim. */
static int i2s_shape_sse2(size_t packed_len, uint32_t in_dim, uint32_t out_dim) {
    if (in_dim == 0 || in_dim % QK_I2_S != 0) return -1;
    if (packed_len < (size_t)(in_dim / 4) * out_dim) return -1;
    return 0;
}

/* bitlinear_sse2.rs:313-342 */
int or_i2s_matvec_sse2_i8(const uint8_t *packed, size_t packed_len,
                          float w_scale, uint32_t in_dim, uint32_t out_dim,
                          const float *x, float *y, int32_t *acc_out,
                          float *act_scale_out, int8_t *act_q_out) {
    if (i2s_shape_sse2(packed_len, in_dim, out_dim) || scale_ok(w_scale)) return -1;
    size_t bytes_per_row = in_dim / 4;
    uint32_t blocks = in_dim / QK_I2_S;
    int8_t *act = (int8_t *)malloc(in_dim);
    if (!act) return -2;
    float input_scale = or_quantize_absmax_i8(x, in_dim, act);
    float combined = w_scale * input_scale;
    int8_t unpacked[QK_I2_S];
    for (uint32_t j = 0; j < out_dim; j++) {
        const uint8_t *row = packed + (size_t)j * bytes_per_row;
        int32_t dot = 0;
        for (uint32_t bk = 0; bk < blocks; bk++) {
            unpack_block(row + (size_t)bk * I2S_BLOCK_BYTES, unpacked);
            dot += dot_i8_ternary(unpacked, act + (size_t)bk * QK_I2_S);
        }
        y[j] = combined * (float)dot;
        if (acc_out) acc_out[j] = dot;
    }
    if (act_scale_out) *act_scale_out = input_scale;
    if (act_q_out) memcpy(act_q_out, act, in_dim);
    free(act);
    return 0;
}

int or_i2s_gemm_rows(const uint8_t *packed, size_t packed_len, float w_scale,
                     uint32_t in_dim, uint32_t out_dim, uint32_t m,
                     const float *x, float *y, int32_t *acc_out,
                     float *act_scale_out, int n_threads) {
    if (i2s_shape_sse2(packed_len, in_dim, out_dim) || scale_ok(w_scale)) return -1;
    int rc = 0;
#ifdef _OPENMP
    int nt = n_threads > 0 ? n_threads : omp_get_max_threads();
#pragma omp parallel for num_threads(nt) schedule(static) reduction(| : rc)
#endif
    for (uint32_t t = 0; t < m; t++) {
        rc |= or_i2s_matvec_sse2_i8(packed, packed_len, w_scale, in_dim, out_dim,
                                    x + (size_t)t * in_dim, y + (size_t)t * out_dim,
                                    acc_out ? acc_out + (size_t)t * out_dim : NULL,
                                    act_scale_out ? act_scale_out + t : NULL, NULL);
    }
    (void)n_threads;
    return rc;
}

/* bitlinear_sse2.rs:249-255 -- (v0+v3) + (v2+v1). */
static float hsum_ps(__m128 v) {
    __m128 shuf = _mm_shuffle_ps(v, v, _MM_SHUFFLE(0, 1, 2, 3));
    __m128 sums = _mm_add_ps(v, shuf);
    __m128 shuf2 = _mm_movehl_ps(sums, sums);
    return _mm_cvtss_f32(_mm_add_ss(sums, shuf2));
}

/* bitlinear_sse2.rs:89-124, block_accumulate :206-235 */
int or_i2s_matvec_sse2_f32(const uint8_t *packed, size_t packed_len,
                           float scale, uint32_t in_dim, uint32_t out_dim,
                           const float *x, float *y) {
    if (i2s_shape_sse2(packed_len, in_dim, out_dim) || scale_ok(scale)) return -1;
    size_t bytes_per_row = in_dim / 4;
    uint32_t blocks = in_dim / QK_I2_S;
    const __m128i pos_target = _mm_set1_epi32(1);
    const __m128i neg_target = _mm_set1_epi32(-1);
    int8_t unpacked[QK_I2_S];
    for (uint32_t j = 0; j < out_dim; j++) {
        const uint8_t *row = packed + (size_t)j * bytes_per_row;
        __m128 pos_sum = _mm_setzero_ps(), neg_sum = _mm_setzero_ps();
        for (uint32_t bk = 0; bk < blocks; bk++) {
            unpack_block(row + (size_t)bk * I2S_BLOCK_BYTES, unpacked);
            const float *xb = x + (size_t)bk * QK_I2_S;
            for (int c = 0; c < QK_I2_S / 4; c++) {
                int off = c * 4;
                __m128 xv = _mm_loadu_ps(xb + off);
                int32_t four;
                memcpy(&four, unpacked + off, 4);
                __m128i v_i8 = _mm_cvtsi32_si128(four);
                __m128i v_i16 = _mm_srai_epi16(_mm_unpacklo_epi8(v_i8, v_i8), 8);
                __m128i v_i32 = _mm_srai_epi32(_mm_unpacklo_epi16(v_i16, v_i16), 16);
                __m128 pm = _mm_castsi128_ps(_mm_cmpeq_epi32(v_i32, pos_target));
                __m128 nm = _mm_castsi128_ps(_mm_cmpeq_epi32(v_i32, neg_target));
                pos_sum = _mm_add_ps(pos_sum, _mm_and_ps(xv, pm));
                neg_sum = _mm_add_ps(neg_sum, _mm_and_ps(xv, nm));
            }
        }
        y[j] = scale * (hsum_ps(pos_sum) - hsum_ps(neg_sum));
    }
    return 0;
}

/* bitlinear_lut.rs:59-131 */
int or_i2s_matvec_lut(const uint8_t *packed, size_t packed_len, float scale,
                      uint32_t in_dim, uint32_t out_dim, const float *x,
                      float *y) {
    if (i2s_shape_exact(packed_len, in_dim, out_dim) || scale_ok(scale)) return -1;
    size_t bytes_per_row = in_dim / 4;
    uint32_t blocks = in_dim / QK_I2_S;
    for (uint32_t j = 0; j < out_dim; j++) y[j] = 0.0f;
    float table[256], t0[4], t1[4], t2[4], t3[4];
    for (uint32_t bk = 0; bk < blocks; bk++) {
        size_t col = (size_t)bk * QK_I2_S;
        for (int gp = 0; gp < I2S_BLOCK_BYTES; gp++) {
            float x0 = x[col + gp], x1 = x[col + gp + 32];
            float x2 = x[col + gp + 64], x3 = x[col + gp + 96];
            t0[0] = -x0; t0[1] = 0.0f; t0[2] = x0; t0[3] = 0.0f;
            t1[0] = -x1; t1[1] = 0.0f; t1[2] = x1; t1[3] = 0.0f;
            t2[0] = -x2; t2[1] = 0.0f; t2[2] = x2; t2[3] = 0.0f;
            t3[0] = -x3; t3[1] = 0.0f; t3[2] = x3; t3[3] = 0.0f;
            for (int bv = 0; bv < 256; bv++) {
                table[bv] = t0[(bv >> 6) & 3] + t1[(bv >> 4) & 3] + t2[(bv >> 2) & 3] + t3[bv & 3];
            }
            size_t off = (size_t)bk * I2S_BLOCK_BYTES + gp;
            for (uint32_t j = 0; j < out_dim; j++) {
                y[j] += table[packed[(size_t)j * bytes_per_row + off]];
            }
        }
    }
    for (uint32_t j = 0; j < out_dim; j++) y[j] *= scale;
    return 0;
}

/* bitlinear.rs:247-299 */
int or_i2s_unpack_row(const uint8_t *packed, size_t packed_len,
                      uint32_t in_dim, uint32_t out_dim, uint32_t row,
                      int8_t *out) {
    if (row >= out_dim) return -1;
    if (in_dim == 0 || in_dim % QK_I2_S != 0) return -1;
    size_t bpr = in_dim / 4;
    size_t off = (size_t)row * bpr;
    if (off + bpr > packed_len) return -1;
    for (uint32_t bk = 0; bk < in_dim / QK_I2_S; bk++) {
        unpack_block(packed + off + (size_t)bk * I2S_BLOCK_BYTES, out + (size_t)bk * QK_I2_S);
    }
    return 0;
}

/* ------------------------------------------------------------------ Q6_K */

/* q6_k.rs:8-23 */
static int q6k_validate(size_t row_len, size_t n) {
    if (n % Q6K_VALUES != 0) return -1;
    if (row_len != n / Q6K_VALUES * Q6K_BYTES) return -1;
    return 0;
}

/* q6_k.rs:25-57 -- element index within the 256-value block and its
 * dequantised weight (d * scale) * q, visited in the reference's order. */
typedef void (*q6k_visit_fn)(void *ctx, size_t index, float weight);

static void q6k_for_each_weight(const uint8_t *block, q6k_visit_fn visit, void *ctx) {
    const uint8_t *ql0 = block, *qh0 = block + 128, *sc0 = block + 192;
    float d = or_f16_to_f32((uint16_t)(block[208] | (block[209] << 8)));
    for (int half = 0; half < 2; half++) {
        const uint8_t *ql = ql0 + half * 64, *qh = qh0 + half * 32, *sc = sc0 + half * 8;
        size_t out = (size_t)half * 128;
        for (int l = 0; l < 32; l++) {
            int s = l / 16;
            int q1 = (int8_t)((ql[l] & 0x0F) | ((qh[l] & 3) << 4)) - 32;
            int q2 = (int8_t)((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
            int q3 = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            int q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            visit(ctx, out + l, d * (float)(int8_t)sc[s] * (float)q1);
            visit(ctx, out + l + 32, d * (float)(int8_t)sc[s + 2] * (float)q2);
            visit(ctx, out + l + 64, d * (float)(int8_t)sc[s + 4] * (float)q3);
            visit(ctx, out + l + 96, d * (float)(int8_t)sc[s + 6] * (float)q4);
        }
    }
}

struct q6k_store_ctx { float *out; };
static void q6k_store(void *ctx, size_t i, float w) { ((struct q6k_store_ctx *)ctx)->out[i] = w; }

/* q6_k.rs:59-69 */
int or_q6k_dequantize_row(const uint8_t *row, size_t row_len, float *out, size_t n) {
    if (q6k_validate(row_len, n)) return -1;
    for (size_t b = 0; b < n / Q6K_VALUES; b++) {
        struct q6k_store_ctx c = {out + b * Q6K_VALUES};
        q6k_for_each_weight(row + b * Q6K_BYTES, q6k_store, &c);
    }
    return 0;
}

struct q6k_dot_ctx { float sum; const float *x; };
static void q6k_dot_visit(void *ctx, size_t i, float w) {
    struct q6k_dot_ctx *c = (struct q6k_dot_ctx *)ctx;
    c->sum += w * c->x[i];
}

/* q6_k.rs:84-96 */
int or_q6k_dot_row_scalar(const uint8_t *row, size_t row_len, const float *x,
                          size_t n, float *out) {
    if (q6k_validate(row_len, n)) return -1;
    struct q6k_dot_ctx c = {0.0f, NULL};
    for (size_t b = 0; b < n / Q6K_VALUES; b++) {
        c.x = x + b * Q6K_VALUES;
        q6k_for_each_weight(row + b * Q6K_BYTES, q6k_dot_visit, &c);
    }
    *out = c.sum;
    return 0;
}

/* q6_k_sse2.rs:21-28 -- acc += (q * scale) * x, no FMA. */
static inline __m128 q6k_accumulate(__m128 acc, const float *x, const int32_t q[4], __m128 scale) {
    __m128 quantized = _mm_cvtepi32_ps(_mm_setr_epi32(q[0], q[1], q[2], q[3]));
    __m128 values = _mm_loadu_ps(x);
    return _mm_add_ps(acc, _mm_mul_ps(_mm_mul_ps(quantized, scale), values));
}

/* q6_k_sse2.rs:32-37 -- (v0+v3) + (v1+v2). */
static float q6k_hsum(__m128 v) {
    __m128 reversed = _mm_shuffle_ps(v, v, _MM_SHUFFLE(0, 1, 2, 3));
    __m128 pairs = _mm_add_ps(v, reversed);
    __m128 high = _mm_movehl_ps(pairs, pairs);
    return _mm_cvtss_f32(_mm_add_ss(pairs, high));
}

/* q6_k_sse2.rs:46-116 */
int or_q6k_dot_row_sse2(const uint8_t *row, size_t row_len, const float *x,
                        size_t n, float *out) {
    if (q6k_validate(row_len, n)) return -1;
    __m128 acc[4] = {_mm_setzero_ps(), _mm_setzero_ps(), _mm_setzero_ps(), _mm_setzero_ps()};
    for (size_t b = 0; b < n / Q6K_VALUES; b++) {
        const uint8_t *block = row + b * Q6K_BYTES;
        float d = or_f16_to_f32((uint16_t)(block[208] | (block[209] << 8)));
        const float *xb = x + b * Q6K_VALUES;
        for (int half = 0; half < 2; half++) {
            int ql_base = half * 64, qh_base = 128 + half * 32, sc_base = 192 + half * 8;
            const float *xin = xb + half * 128;
            for (int band = 0; band < 2; band++) {
                __m128 sc[4];
                for (int a = 0; a < 4; a++) {
                    sc[a] = _mm_set1_ps(d * (float)(int8_t)block[sc_base + band + 2 * a]);
                }
                for (int chunk = 0; chunk < 4; chunk++) {
                    int l = band * 16 + chunk * 4;
                    int32_t q[4][4];
                    for (int lane = 0; lane < 4; lane++) {
                        int idx = l + lane;
                        uint8_t low13 = block[ql_base + idx];
                        uint8_t low24 = block[ql_base + idx + 32];
                        uint8_t high = block[qh_base + idx];
                        q[0][lane] = (int32_t)((low13 & 0x0F) | ((high & 3) << 4)) - 32;
                        q[1][lane] = (int32_t)((low24 & 0x0F) | (((high >> 2) & 3) << 4)) - 32;
                        q[2][lane] = (int32_t)((low13 >> 4) | (((high >> 4) & 3) << 4)) - 32;
                        q[3][lane] = (int32_t)((low24 >> 4) | (((high >> 6) & 3) << 4)) - 32;
                    }
                    acc[0] = q6k_accumulate(acc[0], xin + l, q[0], sc[0]);
                    acc[1] = q6k_accumulate(acc[1], xin + l + 32, q[1], sc[1]);
                    acc[2] = q6k_accumulate(acc[2], xin + l + 64, q[2], sc[2]);
                    acc[3] = q6k_accumulate(acc[3], xin + l + 96, q[3], sc[3]);
                }
            }
        }
    }
    *out = q6k_hsum(_mm_add_ps(_mm_add_ps(acc[0], acc[1]), _mm_add_ps(acc[2], acc[3])));
    return 0;
}

/* q6_k.rs:98-101 */
static int32_t nearest_int(float value) {
    return (int32_t)(f32_to_bits(value + 12582912.0f) & 0x007FFFFFu) - 0x00400000;
}
static int32_t clamp_i32(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* q6_k.rs:103-111 */
static float signed_abs_max(const float *in, int n) {
    float max = 0.0f;
    for (int i = 0; i < n; i++) if (fabsf(in[i]) > fabsf(max)) max = in[i];
    return max;
}

/* q6_k.rs:113-117 */
static void store_levels(const float *in, int8_t *levels, int n, float inv) {
    for (int i = 0; i < n; i++) levels[i] = (int8_t)(clamp_i32(nearest_int(inv * in[i]), -32, 31) + 32);
}

/* q6_k.rs:119-129 */
static void weighted_sums(const float *in, int n, float inv, float *lx, float *l2) {
    float sum_lx = 0.0f, sum_l2 = 0.0f;
    for (int i = 0; i < n; i++) {
        int32_t level = clamp_i32(nearest_int(inv * in[i]), -32, 31);
        float weight = in[i] * in[i];
        sum_lx += weight * in[i] * (float)level;
        sum_l2 += weight * (float)(level * level);
    }
    *lx = sum_lx;
    *l2 = sum_l2;
}

/* q6_k.rs:131-156 */
static float make_qx_quants(const float *in, int8_t *levels) {
    float max = signed_abs_max(in, 16);
    if (fabsf(max) < 1e-15f) {
        memset(levels, 0, 16);
        return 0.0f;
    }
    float inv = -32.0f / max;
    store_levels(in, levels, 16, inv);
    float sum_lx, sum_l2;
    weighted_sums(in, 16, inv, &sum_lx, &sum_l2);
    float scale = sum_l2 != 0.0f ? sum_lx / sum_l2 : 0.0f;
    float best = scale * sum_lx;
    for (int adj = -9; adj <= 9; adj++) {
        if (adj == 0) continue;
        inv = -(32.0f + 0.1f * (float)adj) / max;
        weighted_sums(in, 16, inv, &sum_lx, &sum_l2);
        if (sum_l2 > 0.0f && sum_lx * sum_lx > best * sum_l2) {
            store_levels(in, levels, 16, inv);
            scale = sum_lx / sum_l2;
            best = scale * sum_lx;
        }
    }
    return scale;
}

/* q6_k.rs:195-214 */
static void pack_block(const int8_t levels[256], const int8_t qs[16], uint16_t d_bits, uint8_t *out) {
    for (int half = 0; half < 2; half++) {
        int src = half * 128, ql = half * 64, qh = 128 + half * 32;
        for (int i = 0; i < 32; i++) {
            uint8_t q1 = (uint8_t)levels[src + i], q2 = (uint8_t)levels[src + i + 32];
            uint8_t q3 = (uint8_t)levels[src + i + 64], q4 = (uint8_t)levels[src + i + 96];
            out[ql + i] = (uint8_t)((q1 & 0x0F) | ((q3 & 0x0F) << 4));
            out[ql + i + 32] = (uint8_t)((q2 & 0x0F) | ((q4 & 0x0F) << 4));
            out[qh + i] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    }
    for (int i = 0; i < 16; i++) out[192 + i] = (uint8_t)qs[i];
    out[208] = (uint8_t)(d_bits & 0xFF);
    out[209] = (uint8_t)(d_bits >> 8);
}

/* q6_k.rs:158-229 */
static void quantize_block(const float *in, uint8_t *out) {
    int8_t levels[256];
    float scales[16], max_scale = 0.0f;
    for (int g = 0; g < 16; g++) {
        scales[g] = make_qx_quants(in + g * 16, levels + g * 16);
        if (fabsf(scales[g]) > fabsf(max_scale)) max_scale = scales[g];
    }
    if (fabsf(max_scale) < 1e-15f) {
        memset(out, 0, Q6K_BYTES);
        return;
    }
    float inv = -128.0f / max_scale;
    uint16_t d_bits = or_f32_to_f16(1.0f / inv);
    float d = or_f16_to_f32(d_bits);
    int8_t qs[16];
    for (int g = 0; g < 16; g++) {
        int32_t v = nearest_int(inv * scales[g]);
        if (v > 127) v = 127;
        qs[g] = (int8_t)v;
        float group_scale = d * (float)qs[g];
        if (group_scale != 0.0f) {
            for (int i = 0; i < 16; i++) {
                int32_t level = clamp_i32(nearest_int(in[g * 16 + i] / group_scale), -32, 31);
                levels[g * 16 + i] = (int8_t)(level + 32);
            }
        }
    }
    pack_block(levels, qs, d_bits, out);
}

/* q6_k.rs:232-238 */
int or_q6k_quantize_row(const float *in, size_t n, uint8_t *out, size_t out_len) {
    if (q6k_validate(out_len, n)) return -1;
    for (size_t b = 0; b < n / Q6K_VALUES; b++) quantize_block(in + b * Q6K_VALUES, out + b * Q6K_BYTES);
    return 0;
}

/* ------------------------------------------------------------------ Q8_0 */

/* q8_0.rs:7-23 */
static int q8_validate(size_t row_len, size_t n) {
    if (n % Q8_0_VALUES != 0) return -1;
    if (row_len != n / Q8_0_VALUES * Q8_0_BYTES) return -1;
    return 0;
}

/* q8_0.rs:25-33 -- non-finite block scale is an error. */
static int q8_scale(const uint8_t *block, float *scale) {
    *scale = or_f16_to_f32((uint16_t)(block[0] | (block[1] << 8)));
    return isfinite(*scale) ? 0 : -1;
}

/* q8_0.rs:35-48 */
int or_q8_0_dequantize_row(const uint8_t *row, size_t row_len, float *out, size_t n) {
    if (q8_validate(row_len, n)) return -1;
    for (size_t b = 0; b < n / Q8_0_VALUES; b++) {
        const uint8_t *blk = row + b * Q8_0_BYTES;
        float s;
        if (q8_scale(blk, &s)) return -1;
        for (int i = 0; i < Q8_0_VALUES; i++) out[b * Q8_0_VALUES + i] = s * (float)(int8_t)blk[2 + i];
    }
    return 0;
}

/* q8_0.rs:72-85 */
int or_q8_0_dot_row_scalar(const uint8_t *row, size_t row_len, const float *x,
                           size_t n, float *out) {
    if (q8_validate(row_len, n)) return -1;
    float sum = 0.0f;
    for (size_t b = 0; b < n / Q8_0_VALUES; b++) {
        const uint8_t *blk = row + b * Q8_0_BYTES;
        float s;
        if (q8_scale(blk, &s)) return -1;
        for (int i = 0; i < Q8_0_VALUES; i++) sum += s * (float)(int8_t)blk[2 + i] * x[b * Q8_0_VALUES + i];
    }
    *out = sum;
    return 0;
}

/* q8_0_simd.rs:145-157 -- (v0+v2) + (v1+v3). */
static float hsum_sse(__m128 v) {
    __m128 high = _mm_movehl_ps(v, v);
    __m128 pairs = _mm_add_ps(v, high);
    __m128 second = _mm_shuffle_ps(pairs, pairs, 0x55);
    return _mm_cvtss_f32(_mm_add_ss(pairs, second));
}

/* q8_0_simd.rs:72-104 */
__attribute__((target("avx2")))
int or_q8_0_dot_row_avx2(const uint8_t *row, size_t row_len, const float *x,
                         size_t n, float *out) {
    if (q8_validate(row_len, n)) return -1;
    float total = 0.0f;
    for (size_t b = 0; b < n / Q8_0_VALUES; b++) {
        const uint8_t *blk = row + b * Q8_0_BYTES;
        const int8_t *values = (const int8_t *)(blk + 2);
        const float *xin = x + b * Q8_0_VALUES;
        __m256 sum = _mm256_setzero_ps();
        for (int off = 0; off < 32; off += 8) {
            __m128i q = _mm_loadl_epi64((const __m128i *)(values + off));
            __m256 qf = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(q));
            sum = _mm256_add_ps(sum, _mm256_mul_ps(qf, _mm256_loadu_ps(xin + off)));
        }
        __m128 halves = _mm_add_ps(_mm256_castps256_ps128(sum), _mm256_extractf128_ps(sum, 1));
        float s;
        if (q8_scale(blk, &s)) return -1;
        total += s * hsum_sse(halves);
    }
    *out = total;
    return 0;
}

/* q8_0_simd.rs:108-141 */
int or_q8_0_dot_row_sse2(const uint8_t *row, size_t row_len, const float *x,
                         size_t n, float *out) {
    if (q8_validate(row_len, n)) return -1;
    float total = 0.0f;
    for (size_t b = 0; b < n / Q8_0_VALUES; b++) {
        const uint8_t *blk = row + b * Q8_0_BYTES;
        const uint8_t *values = blk + 2;
        const float *xin = x + b * Q8_0_VALUES;
        __m128 sum = _mm_setzero_ps();
        for (int off = 0; off < 32; off += 4) {
            int32_t packed;
            memcpy(&packed, values + off, 4);
            __m128i q8 = _mm_cvtsi32_si128(packed);
            __m128i q16 = _mm_srai_epi16(_mm_unpacklo_epi8(q8, q8), 8);
            __m128i q32 = _mm_srai_epi32(_mm_unpacklo_epi16(q16, q16), 16);
            sum = _mm_add_ps(sum, _mm_mul_ps(_mm_cvtepi32_ps(q32), _mm_loadu_ps(xin + off)));
        }
        float s;
        if (q8_scale(blk, &s)) return -1;
        total += s * hsum_sse(sum);
    }
    *out = total;
    return 0;
}

/* q8_0.rs:50-70 -- x86 dispatch: AVX2 when the CPU has it, else SSE2. */
static int q8_0_dot_row_dispatch(const uint8_t *row, size_t row_len, const float *x, size_t n, float *out) {
    if (__builtin_cpu_supports("avx2")) return or_q8_0_dot_row_avx2(row, row_len, x, n, out);
    return or_q8_0_dot_row_sse2(row, row_len, x, n, out);
}

/* linear.rs:171-224 */
int or_q8_0_matvec(const uint8_t *w, size_t w_len, uint32_t in_dim,
                   uint32_t out_dim, const float *x, float *y, int n_threads) {
    if (in_dim % Q8_0_VALUES != 0) return -1;
    size_t row_bytes = (size_t)in_dim / Q8_0_VALUES * Q8_0_BYTES;
    if (w_len != row_bytes * out_dim) return -1;
    int rc = 0;
#ifdef _OPENMP
    int nt = n_threads > 0 ? n_threads : omp_get_max_threads();
#pragma omp parallel for num_threads(nt) schedule(static) reduction(| : rc)
#endif
    for (uint32_t r = 0; r < out_dim; r++) {
        rc |= q8_0_dot_row_dispatch(w + (size_t)r * row_bytes, row_bytes, x, in_dim, y + r);
    }
    (void)n_threads;
    return rc;
}

/* ------------------------------------------------------------------ lm-head */

/* lm_head.rs:29-108 (F16 / Q8_0 / Q6_K arms). */
int or_compute_logits(const float *hidden, uint32_t n_embd,
                      const uint8_t *w, size_t w_len, uint32_t ggml_type,
                      uint32_t vocab, float *logits, int n_threads) {
    size_t row_bytes;
    switch (ggml_type) {
    case 1: row_bytes = (size_t)n_embd * 2; break;
    case 8:
        if (n_embd % Q8_0_VALUES) return -1;
        row_bytes = (size_t)n_embd / Q8_0_VALUES * Q8_0_BYTES;
        break;
    case 14:
        if (n_embd % Q6K_VALUES) return -1;
        row_bytes = (size_t)n_embd / Q6K_VALUES * Q6K_BYTES;
        break;
    default: return -1;
    }
    if (w_len != row_bytes * vocab) return -1;
    int rc = 0;
#ifdef _OPENMP
    int nt = n_threads > 0 ? n_threads : omp_get_max_threads();
#pragma omp parallel for num_threads(nt) schedule(static) reduction(| : rc)
#endif
    for (uint32_t v = 0; v < vocab; v++) {
        const uint8_t *row = w + (size_t)v * row_bytes;
        if (ggml_type == 1) {
            float sum = 0.0f;
            for (uint32_t i = 0; i < n_embd; i++) {
                sum += or_f16_to_f32((uint16_t)(row[2 * i] | (row[2 * i + 1] << 8))) * hidden[i];
            }
            logits[v] = sum;
        } else if (ggml_type == 8) {
            rc |= q8_0_dot_row_dispatch(row, row_bytes, hidden, n_embd, logits + v);
        } else {
            rc |= or_q6k_dot_row_sse2(row, row_bytes, hidden, n_embd, logits + v);
        }
    }
    (void)n_threads;
    return rc;
}

/* lm_head.rs:161-174 -- strict '>' scan: ties keep the first index and a
 * NaN never replaces the running best. */
int64_t or_argmax(const float *logits, size_t n) {
    if (n == 0) return -1;
    size_t best = 0;
    float best_v = logits[0];
    for (size_t i = 1; i < n; i++) {
        if (logits[i] > best_v) {
            best_v = logits[i];
            best = i;
        }
    }
    return (int64_t)best;
}
