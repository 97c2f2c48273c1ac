/*
 * bitnet_forward.c -- CPU oracle of the reference's single-token decode step
 * with its i8 KV cache, and of its greedy generation loop.
 *
 * TEST INFRASTRUCTURE ONLY (see willamette_oracle.h): the parity checker for
 * the library's device-resident decode step.  Follows, in order:
 *   forward_with_cache_progress_into   src/model/cached_forward.rs:206-259
 *   forward_one_layer                  src/model/cached_forward.rs:308-419
 *   scaled_dot_product_attention_into  src/model/cached_forward.rs:421-451
 *   apply_ffn_block                    src/model/cached_forward.rs:453-504
 *   greedy_generate_with_cache         src/model/generate.rs:111-190
 * and the primitives they call:
 *   rms_norm_f32          src/model/primitives.rs:227-254
 *   apply_rope_f32 (NEOX) src/model/primitives.rs:283-345
 *   attention_scale       src/model/primitives.rs:354-357
 *   softmax_inplace       src/model/attention.rs:45-73
 *   KVCache append / read src/model/kv_cache.rs:154-219, :245-259
 *   relu_square / silu / elementwise_mul  src/model/ffn.rs:37-65
 *   embedding_gather (Q6_K / Q8_0 row)    src/model/primitives.rs:120-190
 * Two forward variants (cached_forward.rs:373-504, ForwardVariant):
 * BitNetSubNorm (attn / ffn sub-norms, relu^2, NEOX RoPE) and VanillaLlama
 * (no sub-norms, SiLU, Norm RoPE pairs (2j, 2j+1)), the latter with Q8_0
 * linears (q8_0_matvec_f32, linear.rs:171-224) for the SmolLM shapes.
 * BitLinears go through or_i2s_matvec_sse2_i8 (the x86 default), split into
 * row chunks over OpenMP threads: each chunk quantises the same x the same
 * way and rows are independent, so the result equals one serial call.
 * Transcendentals (powf, sinf, cosf, expf, sqrtf) are the C library's, as
 * Rust's f32 methods call the platform libm.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "willamette_oracle.h"

#define I2S_MATS 7 /* q, k, v, o, gate, up, down */

void or_rms_norm(const float *x, const float *w, float eps, float *out, uint32_t n) {
    float sum_sq = 0.0f;
    for (uint32_t i = 0; i < n; ++i) sum_sq += x[i] * x[i];
    const float mean = sum_sq / (float)n;
    const float rsqrt = 1.0f / sqrtf(mean + eps);
    for (uint32_t i = 0; i < n; ++i) out[i] = x[i] * rsqrt * w[i];
}

void or_rope_neox(float *x, uint32_t n_rot, uint32_t position, float freq_base) {
    const uint32_t half = n_rot / 2;
    const float pos = (float)position;
    const float n_rot_f = (float)n_rot;
    for (uint32_t j = 0; j < half; ++j) {
        const float exponent = -2.0f * (float)j / n_rot_f;
        const float theta = pos * powf(freq_base, exponent);
        const float sin_t = sinf(theta), cos_t = cosf(theta);
        const float a = x[j], b = x[j + half];
        x[j] = a * cos_t - b * sin_t;
        x[j + half] = a * sin_t + b * cos_t;
    }
}

void or_rope_norm(float *x, uint32_t n_rot, uint32_t position, float freq_base) {
    const uint32_t half = n_rot / 2;
    const float pos = (float)position;
    const float n_rot_f = (float)n_rot;
    for (uint32_t j = 0; j < half; ++j) {
        const float exponent = -2.0f * (float)j / n_rot_f;
        const float theta = pos * powf(freq_base, exponent);
        const float sin_t = sinf(theta), cos_t = cosf(theta);
        const float a = x[2 * j], b = x[2 * j + 1];
        x[2 * j] = a * cos_t - b * sin_t;
        x[2 * j + 1] = a * sin_t + b * cos_t;
    }
}

void or_silu_inplace(float *x, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) x[i] /= 1.0f + expf(-x[i]);
}

void or_softmax_inplace(float *x, uint32_t n) {
    if (n == 0) return;
    float max = -INFINITY;
    for (uint32_t i = 0; i < n; ++i)
        if (x[i] > max) max = x[i];
    if (!isfinite(max)) {
        for (uint32_t i = 0; i < n; ++i) x[i] = 0.0f;
        return;
    }
    float sum = 0.0f;
    for (uint32_t i = 0; i < n; ++i) {
        x[i] = expf(x[i] - max);
        sum += x[i];
    }
    if (sum > 0.0f) {
        const float inv = 1.0f / sum;
        for (uint32_t i = 0; i < n; ++i) x[i] *= inv;
    }
}

/* kv_cache.rs:245-259: per-token absmax over the vector (f32::max skips NaN),
 * zeros and scale 0 for an all-zero or non-finite absmax. */
void or_kv_quantise(const float *x, uint32_t n, int8_t *q, float *scale) {
    float absmax = 0.0f;
    for (uint32_t i = 0; i < n; ++i) absmax = fmaxf(absmax, fabsf(x[i]));
    if (absmax == 0.0f || !isfinite(absmax)) {
        memset(q, 0, n);
        *scale = 0.0f;
        return;
    }
    *scale = absmax / 127.0f;
    const float inv = 127.0f / absmax;
    for (uint32_t i = 0; i < n; ++i) {
        float r = roundf(x[i] * inv);
        if (isnan(r)) r = 0.0f;
        r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
        q[i] = (int8_t)r;
    }
}

static int bitlinear(const uint8_t *packed, float w_scale, uint32_t in_dim, uint32_t out_dim,
                     const float *x, float *y, int n_threads) {
    const size_t row_bytes = in_dim / 4;
    const uint32_t chunk = 64;
    const uint32_t n_chunks = (out_dim + chunk - 1) / chunk;
    int rc = 0;
#pragma omp parallel for schedule(static) num_threads(n_threads) reduction(| : rc)
    for (uint32_t c = 0; c < n_chunks; ++c) {
        const uint32_t r0 = c * chunk;
        const uint32_t n = out_dim - r0 < chunk ? out_dim - r0 : chunk;
        rc |= or_i2s_matvec_sse2_i8(packed + r0 * row_bytes, n * row_bytes, w_scale, in_dim, n,
                                   x, y + r0, NULL, NULL, NULL) != 0;
    }
    return rc ? -1 : 0;
}

/* linear_matvec_f32 (linear.rs:11-25): I2_S -> the sse2_i8 kernel, Q8_0 ->
 * q8_0_matvec_f32 (linear.rs:171-224, rows independent). */
static int linear(const or_bitnet_config *c, const uint8_t *w, float w_scale, uint32_t in_dim,
                  uint32_t out_dim, const float *x, float *y, int n_threads) {
    if (c->linear_type == 8)
        return or_q8_0_matvec(w, (size_t)out_dim * (in_dim / 32) * 34, in_dim, out_dim, x, y,
                              n_threads) ? -1 : 0;
    return bitlinear(w, w_scale, in_dim, out_dim, x, y, n_threads);
}

static int check_finite(const float *x, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i)
        if (!isfinite(x[i])) return -1;
    return 0;
}

int or_bitnet_forward(const or_bitnet_config *c, const or_bitnet_weights *w, or_kv_cache *kv,
                      uint32_t token, uint32_t position, float *out, int n_threads) {
    const uint32_t E = c->n_embd, F = c->n_ff, HD = c->head_dim;
    const uint32_t KV = c->n_kv_heads * HD;
    if (n_threads <= 0) n_threads = 1;
    if (!c->n_heads || !c->n_kv_heads || c->n_heads % c->n_kv_heads || c->n_heads * HD != E ||
        c->n_rot == 0 || c->n_rot % 2 || c->n_rot > HD)
        return -1;
    if (kv->pos != position || position >= c->max_seq || token >= c->vocab) return -2;
    const uint32_t group = c->n_heads / c->n_kv_heads;
    const int llama = c->variant == 1;
    const size_t emb_row = c->embd_type == 8 ? (size_t)E / 32 * 34 : (size_t)E / 256 * 210;
    float *hidden = calloc(E, 4), *xn = calloc(E, 4), *q = calloc(E, 4), *k = calloc(KV, 4),
          *v = calloc(KV, 4), *att = calloc(E, 4), *sub = calloc(E, 4), *o = calloc(E, 4),
          *gate = calloc(F, 4), *up = calloc(F, 4), *fused = calloc(F, 4), *fn = calloc(F, 4),
          *down = calloc(E, 4), *scores = calloc((size_t)position + 1, 4);
    int rc = 0;
    if (!hidden || !xn || !q || !k || !v || !att || !sub || !o || !gate || !up || !fused ||
        !fn || !down || !scores) {
        rc = -3;
        goto done;
    }
    /* embedding_gather: the token's Q6_K / Q8_0 row, dequantised */
    if ((c->embd_type == 8
             ? or_q8_0_dequantize_row(w->token_embd + (size_t)token * emb_row, emb_row, hidden, E)
             : or_q6k_dequantize_row(w->token_embd + (size_t)token * emb_row, emb_row, hidden, E))) {
        rc = -4;
        goto done;
    }
    const float scale = 1.0f / sqrtf((float)HD);
    for (uint32_t l = 0; l < c->n_layers; ++l) {
        const uint8_t *const *m = w->w + (size_t)l * I2S_MATS;
        const float *s = w->w_scale + (size_t)l * I2S_MATS;
        const float *attn_norm = w->norms + (size_t)l * (3 * E + F);
        const float *attn_sub_norm = attn_norm + E, *ffn_norm = attn_norm + 2 * E;
        const float *ffn_sub_norm = attn_norm + 3 * E;

        or_rms_norm(hidden, attn_norm, c->eps, xn, E);
        rc |= linear(c, m[0], s[0], E, E, xn, q, n_threads);
        rc |= linear(c, m[1], s[1], E, KV, xn, k, n_threads);
        rc |= linear(c, m[2], s[2], E, KV, xn, v, n_threads);
        for (uint32_t h = 0; h < c->n_heads; ++h)
            (llama ? or_rope_norm : or_rope_neox)(q + h * HD, c->n_rot, position, c->freq_base);
        for (uint32_t h = 0; h < c->n_kv_heads; ++h)
            (llama ? or_rope_norm : or_rope_neox)(k + h * HD, c->n_rot, position, c->freq_base);
        /* KVCache::append then read_into (dequantised f32 of every position) */
        const size_t row = (size_t)l * c->max_seq + position;
        if (c->kv_f16) {
            uint16_t *kh = (uint16_t *)kv->k_q + row * KV, *vh = (uint16_t *)kv->v_q + row * KV;
            for (uint32_t i = 0; i < KV; ++i) {
                kh[i] = or_f32_to_f16(k[i]);
                vh[i] = or_f32_to_f16(v[i]);
            }
        } else {
            or_kv_quantise(k, KV, kv->k_q + row * KV, kv->k_s + row);
            or_kv_quantise(v, KV, kv->v_q + row * KV, kv->v_s + row);
        }
        const uint32_t n_past = position + 1;
        memset(att, 0, (size_t)E * 4);
        for (uint32_t h = 0; h < c->n_heads; ++h) {
            const uint32_t kvh = h / group;
            const float *qh = q + h * HD;
            for (uint32_t p = 0; p < n_past; ++p) {
                const size_t r = ((size_t)l * c->max_seq + p) * KV + kvh * HD;
                float d = 0.0f;
                if (c->kv_f16) {
                    const uint16_t *kp = (const uint16_t *)kv->k_q + r;
                    for (uint32_t i = 0; i < HD; ++i) d += qh[i] * or_f16_to_f32(kp[i]);
                } else {
                    const int8_t *kp = kv->k_q + r;
                    const float sk = kv->k_s[(size_t)l * c->max_seq + p];
                    for (uint32_t i = 0; i < HD; ++i) d += qh[i] * ((float)kp[i] * sk);
                }
                scores[p] = d * scale;
            }
            or_softmax_inplace(scores, n_past);
            float *oh = att + h * HD;
            for (uint32_t p = 0; p < n_past; ++p) {
                const size_t r = ((size_t)l * c->max_seq + p) * KV + kvh * HD;
                const float wgt = scores[p];
                if (c->kv_f16) {
                    const uint16_t *vp = (const uint16_t *)kv->v_q + r;
                    for (uint32_t i = 0; i < HD; ++i) oh[i] += wgt * or_f16_to_f32(vp[i]);
                } else {
                    const int8_t *vp = kv->v_q + r;
                    const float sv = kv->v_s[(size_t)l * c->max_seq + p];
                    for (uint32_t i = 0; i < HD; ++i) oh[i] += wgt * ((float)vp[i] * sv);
                }
            }
        }
        if (!llama) or_rms_norm(att, attn_sub_norm, c->eps, sub, E);
        rc |= linear(c, m[3], s[3], E, E, llama ? att : sub, o, n_threads);
        for (uint32_t i = 0; i < E; ++i) hidden[i] += o[i];
        or_rms_norm(hidden, ffn_norm, c->eps, xn, E);
        rc |= linear(c, m[4], s[4], E, F, xn, gate, n_threads);
        rc |= linear(c, m[5], s[5], E, F, xn, up, n_threads);
        if (llama) or_silu_inplace(gate, F);  /* silu (ffn.rs:45-49) */
        for (uint32_t i = 0; i < F; ++i) {
            float g = gate[i];
            if (!llama) {  /* relu_square (ffn.rs:37-42) */
                const float r = g > 0.0f ? g : 0.0f;
                g = r * r;
            }
            fused[i] = g * up[i];
        }
        if (!llama) or_rms_norm(fused, ffn_sub_norm, c->eps, fn, F);
        rc |= linear(c, m[6], s[6], F, E, llama ? fused : fn, down, n_threads);
        for (uint32_t i = 0; i < E; ++i) hidden[i] += down[i];
        if (rc) {
            rc = -5;
            goto done;
        }
        if (check_finite(hidden, E)) { /* cached_forward.rs:507-517 */
            rc = -6;
            goto done;
        }
    }
    or_rms_norm(hidden, w->output_norm, c->eps, out, E);
    kv->pos = position + 1;
done:
    free(hidden); free(xn); free(q); free(k); free(v); free(att); free(sub); free(o);
    free(gate); free(up); free(fused); free(fn); free(down); free(scores);
    return rc;
}

int or_bitnet_generate(const or_bitnet_config *c, const or_bitnet_weights *w, or_kv_cache *kv,
                       const uint32_t *prompt, uint32_t n_prompt, uint32_t n_new,
                       uint32_t *out_ids, float *hiddens, int n_threads) {
    if (n_prompt == 0) return -1;
    const uint32_t E = c->n_embd;
    const size_t emb_len = c->embd_type == 8 ? (size_t)c->vocab * (E / 32) * 34
                                             : (size_t)c->vocab * (E / 256) * 210;
    float *h = calloc(E, 4), *logits = calloc(c->vocab, 4);
    int rc = 0;
    if (!h || !logits) {
        rc = -3;
        goto done;
    }
    uint32_t pos = kv->pos;
    for (uint32_t i = 0; i < n_prompt; ++i)
        if ((rc = or_bitnet_forward(c, w, kv, prompt[i], pos++, h, n_threads))) goto done;
    for (uint32_t step = 0; step < n_new; ++step) {
        if (hiddens) memcpy(hiddens + (size_t)step * E, h, (size_t)E * 4);
        if ((rc = or_compute_logits(h, E, w->token_embd, emb_len, c->embd_type, c->vocab, logits,
                                    n_threads)))
            goto done;
        const int64_t next = or_argmax(logits, c->vocab);
        out_ids[step] = (uint32_t)next;
        if (step + 1 < n_new)
            if ((rc = or_bitnet_forward(c, w, kv, (uint32_t)next, pos++, h, n_threads))) goto done;
    }
done:
    free(h);
    free(logits);
    return rc;
}
