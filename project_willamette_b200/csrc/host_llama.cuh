// host_llama.cuh -- the batched Q8_0 Llama decode engine (row f2): sequences
// decoded in lock step, one CUDA graph per step, and its C ABI
// (wl_llama_batch_*).
//
// Part of the library's single translation unit: included, in order, by
// willamette_b200.cu after the headers and the parts before it (it is not a
// standalone header).
#pragma once

#include <algorithm>

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
             *d_counter = nullptr, *attn_counters = nullptr,
             *d_seq_order = nullptr;  // exact attention: sequences, longest context first
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
        ap.seq_order = m->d_seq_order;
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
    LB_ALLOC(m->d_seq_order, (size_t)S * 4);
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
    std::vector<uint32_t> ident(S);
    for (uint32_t b = 0; b < S; ++b) ident[b] = b;
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->d_ones, ones.data(), (size_t)S * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->d_seq_order, ident.data(), (size_t)S * 4, cudaMemcpyHostToDevice, s);
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
                    m->attn_counters, m->d_seq_order};
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
    {
        // every step adds one position to every sequence: the order by
        // context length holds for the whole call
        std::vector<uint32_t> order(S);
        for (uint32_t b = 0; b < S; ++b) order[b] = b;
        std::stable_sort(order.begin(), order.end(),
                         [&](uint32_t x, uint32_t y) { return m->pos[x] > m->pos[y]; });
        WL_CUDA(cudaMemcpyAsync(m->d_seq_order, order.data(), (size_t)S * 4, cudaMemcpyHostToDevice,
                                m->stream));  // pageable source: staged before the call returns
    }
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
