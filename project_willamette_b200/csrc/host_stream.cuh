// host_stream.cuh -- stream plans (many independent I2_S matvecs per
// persistent launch: tensor maps, the op table, the byte-balanced split over
// CTAs, one quantisation job per distinct input) and the prefill GEMM host
// side (TMA tensor maps, tile choice, the expanded-weight path).
//
// Part of the library's single translation unit: included, in order, by
// willamette_b200.cu after the headers and the parts before it (it is not a
// standalone header).
#pragma once

// ------------------------------------------------------------- stream plans
struct wl_i2s_stream_plan {
    int device = 0;
    uint32_t n_ops = 0, n_quant = 0, grid = 0;
    bool c3 = true;
    void *d_block = nullptr;  // maps | ops | cta_blocks | quant jobs | scales | q buffers
    CUtensorMap *d_maps = nullptr;
    I2sStreamOp *d_ops = nullptr;
    uint32_t *d_cta_blocks = nullptr;
    QuantJob *d_qjobs = nullptr;
    uint32_t *status = nullptr;
    uintptr_t y_lo = 0, y_hi = 0;  // extent of the ops' outputs (tensor-parallel checks)
};

namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode_tiled(EncodeTiledFn *fn) {
    static EncodeTiledFn cached = nullptr;
    if (!cached) {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !f)
            return fail(WL_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
        cached = (EncodeTiledFn)f;
    }
    *fn = cached;
    return WL_OK;
}

// Tensor map of one packed I2_S weight: 2-D (row bytes, rows), 32-row x
// 128-byte boxes, 128-byte swizzle, zero fill out of bounds.
int encode_i2s_map(const uint8_t *packed, uint32_t K, uint32_t N, CUtensorMap *map) {
    EncodeTiledFn enc;
    int rc = get_encode_tiled(&enc);
    if (rc) return rc;
    const cuuint64_t dims[2] = {K / 4u, N};
    const cuuint64_t strides[1] = {K / 4u};
    const cuuint32_t box[2] = {STREAM_BOX_BYTES, STREAM_BOX_ROWS};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)packed, dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(WL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return WL_OK;
}

// ------------------------------------------------------------------ prefill GEMM
int encode_2d(EncodeTiledFn enc, CUtensorMap *map, const void *base, uint64_t inner_bytes,
              uint64_t rows, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    const cuuint64_t dims[2] = {inner_bytes, rows};
    const cuuint64_t strides[1] = {inner_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(WL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return WL_OK;
}

// Y[m][n] for m tokens from pre-quantised activations q [m][K] (with their
// scales and row sums) and code-3-free packed weights [N][K/4].
int launch_i2s_gemm(const uint8_t *packed, float w_scale, uint32_t K, uint32_t N, uint32_t M,
                    const int8_t *q, const float *act_scale, const int32_t *rowsum, float *y,
                    int32_t *acc, cudaStream_t s, bool pdl, uint32_t *status) {
    if (M == 0 || N == 0) return WL_OK;
    EncodeTiledFn enc;
    int rc = get_encode_tiled(&enc);
    if (rc) return rc;
    const uint32_t mt = (M + GEMM_BM - 1) / GEMM_BM;
    const uint32_t sms = (uint32_t)sm_count_for_launch();
    // widest tile that still gives every SM work
    int bn = 256;
    if ((uint64_t)mt * ((N + 255) / 256) < sms) bn = 128;
    if (bn == 128 && (uint64_t)mt * ((N + 127) / 128) < sms) bn = 64;
    I2sGemmParams p;
    memset(&p, 0, sizeof p);
    if ((rc = encode_2d(enc, &p.a_map, q, K, M, GEMM_BK, GEMM_BM, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = encode_2d(enc, &p.bp_map, packed, K / 4u, N, GEMM_BK / 4, (uint32_t)bn,
                        CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    p.act_scale = act_scale;
    p.rowsum = rowsum;
    p.w_scale = w_scale;
    p.M = M;
    p.N = N;
    p.K = K;
    p.y = y;
    p.acc = acc;
    p.status = status;
    const dim3 grid((N + bn - 1) / bn, mt);
    if (bn == 256)
        WL_CUDA(launch(i2s_gemm_kernel<256>, grid, dim3(GEMM_THREADS), GemmSmem<256>::DYN, s, pdl, p));
    else if (bn == 128)
        WL_CUDA(launch(i2s_gemm_kernel<128>, grid, dim3(GEMM_THREADS), GemmSmem<128>::DYN, s, pdl, p));
    else
        WL_CUDA(launch(i2s_gemm_kernel<64>, grid, dim3(GEMM_THREADS), GemmSmem<64>::DYN, s, pdl, p));
    return WL_OK;
}

// Y[m][n] from pre-quantised activations q [m][K] and int8 ternary weights
// t [N][K] (i2s_expand_kernel): the warp-specialised persistent GEMM.
int launch_i2s_gemm_s8(const int8_t *t, float w_scale, uint32_t K, uint32_t N, uint32_t M,
                       const int8_t *q, const float *act_scale, float *y, int32_t *acc,
                       cudaStream_t s, bool pdl, uint32_t *status) {
    if (M == 0 || N == 0) return WL_OK;
    EncodeTiledFn enc;
    int rc = get_encode_tiled(&enc);
    if (rc) return rc;
    const uint32_t mt = (M + GEMM_BM - 1) / GEMM_BM;
    const uint32_t sms = (uint32_t)sm_count_for_launch();
    // Tile width by estimated time: waves of persistent tiles x per-tile cost
    // (mainloop ~ BN columns, plus a fixed share for the epilogue and fill).
    int bn = 256;
    uint64_t best = ~0ull;
    for (int cand : {256, 128, 64}) {
        const uint64_t tiles = (uint64_t)mt * ((N + cand - 1) / cand);
        const uint64_t cost = ((tiles + sms - 1) / sms) * (uint64_t)(cand + 128);
        if (cost < best) {
            best = cost;
            bn = cand;
        }
    }
    I2sGemmWsParams p;
    memset(&p, 0, sizeof p);
    if ((rc = encode_2d(enc, &p.a_map, q, K, M, GEMM_BK, GEMM_BM, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = encode_2d(enc, &p.b_map, t, K, N, GEMM_BK, (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    // output boxes by TMA store when rows are 16-byte multiples
    if ((N % 4u) == 0 && aligned16(y)) {
        const cuuint64_t dims[2] = {N, M};
        const cuuint64_t strides[1] = {(cuuint64_t)N * 4u};
        const cuuint32_t box[2] = {32, 32};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&p.y_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)y, dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(WL_ERR_CUDA, "cuTensorMapEncodeTiled (y) failed (%d)", (int)r);
        p.use_tma_store = 1;
    }
    p.act_scale = act_scale;
    p.w_scale = w_scale;
    p.M = M;
    p.N = N;
    p.K = K;
    p.y = y;
    p.acc = acc;
    p.status = status;
    const uint32_t tiles = mt * ((N + bn - 1) / bn);
    const dim3 grid(std::min(tiles, sms));
    if (bn == 256)
        WL_CUDA(launch(i2s_gemm_ws_kernel<256>, grid, dim3(WS_THREADS), WsSmem<256>::DYN, s, pdl, p));
    else if (bn == 128)
        WL_CUDA(launch(i2s_gemm_ws_kernel<128>, grid, dim3(WS_THREADS), WsSmem<128>::DYN, s, pdl, p));
    else
        WL_CUDA(launch(i2s_gemm_ws_kernel<64>, grid, dim3(WS_THREADS), WsSmem<64>::DYN, s, pdl, p));
    return WL_OK;
}

int launch_i2s_expand(const uint8_t *packed, uint32_t K, uint32_t N, int8_t *out, cudaStream_t s) {
    const size_t blocks = (size_t)N * (K / 128u);
    if (!blocks) return WL_OK;
    const uint32_t grid = (uint32_t)std::min<size_t>((blocks + 255) / 256, 4u * 1184u);
    i2s_expand_kernel<<<grid, 256, 0, s>>>(packed, blocks, out);
    WL_CUDA(cudaGetLastError());
    return WL_OK;
}

int build_stream_plan(const wl_i2s_stream_op *ops, uint32_t n_ops, wl_i2s_stream_plan *plan) {
    // distinct inputs -> one quantisation each
    std::map<const float *, uint32_t> xid;
    std::vector<uint32_t> qK;
    std::vector<uint32_t> block_begin(n_ops);
    uint64_t total_blocks = 0;
    for (uint32_t j = 0; j < n_ops; ++j) {
        const wl_i2s_stream_op &o = ops[j];
        if (o.in_dim < STREAM_MIN_K || o.in_dim % 128 || o.in_dim > STREAM_MAX_K)
            return fail(WL_ERR_INVALID_ARGUMENT,
                        "op %u: in_dim %u must be a multiple of 128 in [%u, %u] for a stream plan",
                        j, o.in_dim, STREAM_MIN_K, STREAM_MAX_K);
        if (!o.packed || !aligned16(o.packed) || !o.x || !aligned16(o.x) || (!o.y && o.out_dim))
            return fail(WL_ERR_INVALID_ARGUMENT, "op %u: NULL or misaligned pointer", j);
        if (!std::isfinite(o.w_scale))
            return fail(WL_ERR_GGUF_PARSE, "op %u: i2s_scale: non-finite scale", j);
        auto it = xid.find(o.x);
        if (it == xid.end()) {
            xid.emplace(o.x, (uint32_t)qK.size());
            qK.push_back(o.in_dim);
        } else if (qK[it->second] != o.in_dim) {
            return fail(WL_ERR_INVALID_ARGUMENT, "op %u: input shared with a different in_dim", j);
        }
        block_begin[j] = (uint32_t)total_blocks;
        total_blocks += (o.out_dim + STREAM_BOX_ROWS - 1) / STREAM_BOX_ROWS;
    }
    if (total_blocks > 0x7FFFFFFFull) return fail(WL_ERR_INVALID_ARGUMENT, "too many rows");
    Ctx &c = ctx();
    std::lock_guard<std::mutex> g(c.mu);
    int rc = ensure_init(c);
    if (rc) return rc;
    const uint32_t G = (uint32_t)std::max(1, c.sm_count);
    const uint32_t nq = (uint32_t)qK.size();
    const size_t off_maps = 0;
    const size_t off_ops = align_up(off_maps + sizeof(CUtensorMap) * n_ops, 64);
    const size_t off_cta = align_up(off_ops + sizeof(I2sStreamOp) * n_ops, 16);
    const size_t off_q = align_up(off_cta + sizeof(uint32_t) * (G + 1), 16);
    const size_t off_sc = align_up(off_q + sizeof(QuantJob) * nq, 16);
    size_t bytes = align_up(off_sc + sizeof(float) * nq, 16);
    std::vector<size_t> qoff(nq);
    for (uint32_t i = 0; i < nq; ++i) {
        qoff[i] = bytes;
        bytes = align_up(bytes + qK[i], 16);
    }
    WL_CUDA(cudaMalloc(&plan->d_block, bytes));
    uint8_t *base = (uint8_t *)plan->d_block;
    std::vector<uint8_t> host(bytes, 0);
    std::vector<I2sStreamOp> hops(n_ops);
    bool any_c3 = false;
    uint32_t *found = c.d_status + 8;
    for (uint32_t j = 0; j < n_ops; ++j) {
        const wl_i2s_stream_op &o = ops[j];
        const uint32_t qi = xid[o.x];
        hops[j].q = (const int8_t *)(base + qoff[qi]);
        hops[j].act_scale = (const float *)(base + off_sc) + qi;
        hops[j].y = o.y;
        hops[j].acc = o.acc;
        hops[j].w_scale = o.w_scale;
        hops[j].K = o.in_dim;
        hops[j].N = o.out_dim;
        hops[j].block_begin = block_begin[j];
        hops[j].row_off = o.row_off;
        if (o.out_dim) {
            const uintptr_t lo = (uintptr_t)(o.y + o.row_off);
            const uintptr_t hi = lo + (uintptr_t)o.out_dim * sizeof(float);
            plan->y_lo = plan->y_lo ? std::min(plan->y_lo, lo) : lo;
            plan->y_hi = std::max(plan->y_hi, hi);
        }
        if (o.out_dim) {
            CUtensorMap m;
            if ((rc = encode_i2s_map(o.packed, o.in_dim, o.out_dim, &m))) return rc;
            memcpy(host.data() + off_maps + sizeof(CUtensorMap) * j, &m, sizeof m);
        }
        if (!(o.flags & WL_I2S_NO_CODE3) && !any_c3 && o.out_dim) {
            const size_t n16 = (size_t)o.out_dim * (o.in_dim / 4) / 16;
            WL_CUDA(cudaMemsetAsync(found, 0, 4, c.stream));
            const uint32_t grid = (uint32_t)std::min<size_t>((n16 + 255) / 256, 2048);
            i2s_scan_code3_kernel<<<grid, 256, 0, c.stream>>>((const uint4 *)o.packed, n16, found);
            WL_CUDA(cudaGetLastError());
            WL_CUDA(cudaMemcpyAsync(c.h_status + 8, found, 4, cudaMemcpyDeviceToHost, c.stream));
            WL_CUDA(cudaStreamSynchronize(c.stream));
            any_c3 = c.h_status[8] != 0;
        }
    }
    memcpy(host.data() + off_ops, hops.data(), sizeof(I2sStreamOp) * n_ops);
    // byte-balanced block boundaries per CTA
    std::vector<uint32_t> cb(G + 1, 0);
    {
        uint64_t total_bytes = 0;
        for (uint32_t j = 0; j < n_ops; ++j)
            total_bytes += (uint64_t)(ops[j].out_dim + STREAM_BOX_ROWS - 1) / STREAM_BOX_ROWS *
                           STREAM_BOX_ROWS * (ops[j].in_dim / 4);
        // each boundary at the block edge nearest its share (a boundary
        // always placed after the crossing block gave the first CTAs up to a
        // whole block more than the last ones)
        uint32_t j = 0, b = 1;
        uint64_t cum = 0;
        for (uint32_t blk = 0; blk < (uint32_t)total_blocks && b < G; ++blk) {
            while (j + 1 < n_ops && blk >= block_begin[j + 1]) ++j;
            const uint64_t before = cum;
            cum += (uint64_t)STREAM_BOX_ROWS * (ops[j].in_dim / 4);
            while (b < G && cum >= total_bytes * b / G) {
                const uint64_t target = total_bytes * b / G;
                cb[b] = (cum - target > target - before && blk > cb[b - 1]) ? blk : blk + 1;
                ++b;
            }
        }
        for (; b < G; ++b) cb[b] = (uint32_t)total_blocks;
        cb[G] = (uint32_t)total_blocks;
    }
    memcpy(host.data() + off_cta, cb.data(), sizeof(uint32_t) * (G + 1));
    std::vector<QuantJob> qj(nq);
    for (auto &kv : xid) {
        const uint32_t i = kv.second;
        qj[i].x = kv.first;
        qj[i].q = (int8_t *)(base + qoff[i]);
        qj[i].scale = (float *)(base + off_sc) + i;
        qj[i].n = qK[i];
    }
    memcpy(host.data() + off_q, qj.data(), sizeof(QuantJob) * nq);
    WL_CUDA(cudaMemcpyAsync(base, host.data(), bytes, cudaMemcpyHostToDevice, c.stream));
    WL_CUDA(cudaStreamSynchronize(c.stream));
    plan->device = c.device;
    plan->n_ops = n_ops;
    plan->n_quant = nq;
    plan->grid = G;
    plan->c3 = any_c3;
    plan->d_maps = (CUtensorMap *)(base + off_maps);
    plan->d_ops = (I2sStreamOp *)(base + off_ops);
    plan->d_cta_blocks = (uint32_t *)(base + off_cta);
    plan->d_qjobs = (QuantJob *)(base + off_q);
    plan->status = c.d_status;
    return WL_OK;
}

}  // namespace
