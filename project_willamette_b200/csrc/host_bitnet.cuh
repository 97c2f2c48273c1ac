// host_bitnet.cuh -- the BitNet decode engine (row f1): device buffers,
// the per-operation and persistent forwards, graph capture of a decode step,
// the tensor-parallel variant, and its C ABI (wl_bitnet_*).
//
// Part of the library's single translation unit: included, in order, by
// willamette_b200.cu after the headers and the parts before it (it is not a
// standalone header).
#pragma once

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
