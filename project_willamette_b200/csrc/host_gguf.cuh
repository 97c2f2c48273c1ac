// host_gguf.cuh -- GGUF models (row f4): the model configuration from the
// file's metadata, tensor checks as the reference's graph builder makes them,
// and engine creation straight from a parsed file (wl_gguf_*,
// *_create_from_gguf).
//
// Part of the library's single translation unit: included, in order, by
// willamette_b200.cu after the headers and the parts before it (it is not a
// standalone header).
#pragma once

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
