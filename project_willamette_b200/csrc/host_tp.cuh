// host_tp.cuh -- the tensor-parallel group (a CUDA IPC mapped symmetric block
// per rank, arrival counters, device-side waits) and its C ABI: group
// creation and connection, the gathered matvec, the row-sliced stream plan
// run, the vocab-sharded greedy lm-head.
//
// Part of the library's single translation unit: included, in order, by
// willamette_b200.cu after the headers and the parts before it (it is not a
// standalone header).
#pragma once

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

extern "C" {

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
    I2sStreamParams p = {};
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

}  // extern "C"
