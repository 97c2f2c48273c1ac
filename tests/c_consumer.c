/*
 * c_consumer.c -- a plain C11 client of include/willamette_b200.h, linked
 * against the built shared library the way a foreign-language binding (a Rust
 * extern "C" block, cgo, a JNI or N-API stub) links it.  It calls only entry
 * points that need no GPU: the version string, the argument validation of
 * the host-buffer entry points with the reference's error classes
 * (src/model/bitlinear.rs:151-155, src/model/bitlinear_sse2.rs:167-175,
 * src/gguf/tensor.rs:286-307, src/model/linear.rs:23), the size limits of
 * the allocation-free matvec (wl_dev_i2s_matvec_f32_noalloc), the empty cases
 * (src/model/lm_head.rs:161 argmax of an empty slice), and the zero-copy GGUF
 * reader (src/gguf/reader.rs:120-415).  With "--no-gpu" it also checks that a
 * valid call on a machine without an sm_100 device is an error, never a CPU
 * result.  Exit status 0 when every check holds; each failure is printed.
 */
#include <math.h>
#include <stdio.h>
#include <string.h>

#include "willamette_b200.h"

static int failures;

#define CHECK(cond)                                                                   \
    do {                                                                              \
        if (!(cond)) {                                                                \
            fprintf(stderr, "FAIL line %d: %s (last error: %s)\n", __LINE__, #cond, \
                    wl_last_error());                                                 \
            ++failures;                                                               \
        }                                                                             \
    } while (0)

static size_t put_u32(uint8_t *b, size_t o, uint32_t v) {
    for (int i = 0; i < 4; ++i) b[o + i] = (uint8_t)(v >> (8 * i));
    return o + 4;
}

static size_t put_u64(uint8_t *b, size_t o, uint64_t v) {
    for (int i = 0; i < 8; ++i) b[o + i] = (uint8_t)(v >> (8 * i));
    return o + 8;
}

static size_t put_str(uint8_t *b, size_t o, const char *s) {
    const size_t n = strlen(s);
    o = put_u64(b, o, n);
    memcpy(b + o, s, n);
    return o + n;
}

static void i2s_view(wl_tensor_view *t, const uint64_t *shape, const uint8_t *data,
                     size_t data_len, const uint8_t *scale) {
    memset(t, 0, sizeof *t);
    t->name = "blk.0.attn_q.weight";
    t->shape = shape;
    t->n_dims = 2;
    t->ggml_type = WL_GGML_I2_S;
    t->data = data;
    t->data_len = data_len;
    t->scale_data = scale;
    t->scale_len = scale ? 32 : 0;
}

static void check_i2s_validation(int no_gpu) {
    static uint8_t packed[32];
    uint8_t scale[32] = {0}, bad_scale[32] = {0};
    const float one = 1.0f, nan_value = NAN;
    const uint64_t shape[2] = {128, 1}, flat[1] = {128}, empty[2] = {128, 0};
    float x[128], y = 123.0f;
    wl_tensor_view t;

    memset(packed, 0xAA, sizeof packed);
    memcpy(scale, &one, 4);
    memcpy(bad_scale, &nan_value, 4);
    for (int i = 0; i < 128; ++i) x[i] = 1.0f;

    /* wrong dtype -> UnsupportedTensorType carrying the raw type */
    i2s_view(&t, shape, packed, 32, scale);
    t.ggml_type = WL_GGML_F32;
    CHECK(wl_bitlinear_i2s_matvec_f32(&t, x, 128, &y, 1) == WL_ERR_UNSUPPORTED_TENSOR_TYPE);
    CHECK(wl_last_error_tensor_type() == WL_GGML_F32);
    /* not 2-D, wrong input / output lengths, packed area one byte short */
    i2s_view(&t, flat, packed, 32, scale);
    t.n_dims = 1;
    CHECK(wl_bitlinear_i2s_matvec_f32(&t, x, 128, &y, 1) == WL_ERR_GGUF_PARSE);
    i2s_view(&t, shape, packed, 32, scale);
    CHECK(wl_bitlinear_i2s_matvec_f32(&t, x, 64, &y, 1) == WL_ERR_GGUF_PARSE);
    CHECK(wl_bitlinear_i2s_matvec_f32(&t, x, 128, &y, 2) == WL_ERR_GGUF_PARSE);
    i2s_view(&t, shape, packed, 31, scale);
    CHECK(wl_bitlinear_i2s_matvec_f32(&t, x, 128, &y, 1) == WL_ERR_GGUF_PARSE);
    /* missing or non-finite scale */
    i2s_view(&t, shape, packed, 32, NULL);
    CHECK(wl_bitlinear_i2s_matvec_f32(&t, x, 128, &y, 1) == WL_ERR_GGUF_PARSE);
    i2s_view(&t, shape, packed, 32, bad_scale);
    CHECK(wl_bitlinear_i2s_matvec_f32(&t, x, 128, &y, 1) == WL_ERR_GGUF_PARSE);
    /* the output is never written on error */
    CHECK(y == 123.0f);

    /* out_dim 0: the reference loops over nothing and returns Ok */
    i2s_view(&t, empty, packed, 0, scale);
    CHECK(wl_bitlinear_i2s_matvec_f32(&t, x, 128, &y, 0) == WL_OK);

    /* a valid call without an sm_100 device fails loudly */
    if (no_gpu) {
        int st;
        i2s_view(&t, shape, packed, 32, scale);
        st = wl_bitlinear_i2s_matvec_f32(&t, x, 128, &y, 1);
        CHECK(st == WL_ERR_NO_DEVICE || st == WL_ERR_CUDA);
        CHECK(y == 123.0f);
    }
}

static void check_linear_dispatch(void) {
    static uint8_t data[64];
    const uint64_t shape[2] = {32, 2};
    float x[32] = {0}, y[2] = {0};
    wl_tensor_view t;

    memset(&t, 0, sizeof t);
    t.name = "w";
    t.shape = shape;
    t.n_dims = 2;
    t.data = data;
    t.data_len = sizeof data;
    t.ggml_type = 7u; /* Q5_1: no arm in linear_matvec_f32 */
    CHECK(wl_linear_matvec_f32(&t, x, 32, y, 2) == WL_ERR_UNSUPPORTED_TENSOR_TYPE);
    CHECK(wl_last_error_tensor_type() == 7u);
    t.ggml_type = WL_GGML_F16; /* served by the reference's CPU arm */
    CHECK(wl_linear_matvec_f32(&t, x, 32, y, 2) == WL_ERR_NOT_IMPLEMENTED);
}

/* The allocation-free matvec checks its sizes before any device work, so the
 * limit of its static scratch array is visible without a GPU.  The pointers
 * are never dereferenced on these paths. */
static void check_noalloc_limits(void) {
    static _Alignas(16) float xbuf[4];
    static _Alignas(16) uint8_t pbuf[16];
    float y = 5.0f;
    CHECK(wl_dev_i2s_matvec_f32_noalloc(pbuf, 0.05f, WL_NOALLOC_MAX_IN_DIM + 128u, 1, xbuf, &y,
                                        NULL) == WL_ERR_INVALID_ARGUMENT);
    CHECK(strstr(wl_last_error(), "WL_NOALLOC_MAX_IN_DIM") != NULL);
    CHECK(wl_dev_i2s_matvec_f32_noalloc(pbuf, 0.05f, 100u, 1, xbuf, &y, NULL) ==
          WL_ERR_GGUF_PARSE);
    CHECK(wl_dev_i2s_matvec_f32_noalloc(pbuf, NAN, 128u, 1, xbuf, &y, NULL) == WL_ERR_GGUF_PARSE);
    CHECK(y == 5.0f);
}

static void check_argmax_empty(void) {
    int64_t id = 7;
    CHECK(wl_argmax(NULL, 0, &id) == WL_OK);
    CHECK(id == -1);
}

/* A GGUF v3 file with one string key and one 4-element F32 tensor, data
 * section at the default 32-byte alignment.  Returns its length. */
static size_t build_gguf(uint8_t *b, size_t *data_off) {
    size_t o = 0;
    o = put_u32(b, o, 0x46554747u); /* "GGUF" */
    o = put_u32(b, o, 3u);
    o = put_u64(b, o, 1u); /* tensors */
    o = put_u64(b, o, 1u); /* metadata keys */
    o = put_str(b, o, "general.architecture");
    o = put_u32(b, o, 8u); /* string */
    o = put_str(b, o, "llama");
    o = put_str(b, o, "t");
    o = put_u32(b, o, 1u);
    o = put_u64(b, o, 4u);
    o = put_u32(b, o, WL_GGML_F32);
    o = put_u64(b, o, 0u);
    while (o % 32) b[o++] = 0;
    *data_off = o;
    for (int i = 0; i < 4; ++i) {
        const float v = (float)(i + 1);
        memcpy(b + o, &v, 4);
        o += 4;
    }
    return o;
}

static void check_gguf(void) {
    static uint8_t file[256];
    size_t data_off = 0;
    const size_t len = build_gguf(file, &data_off);
    wl_gguf *g = NULL, *bad = NULL;
    wl_tensor_view v;
    const char *arch = NULL;

    CHECK(wl_gguf_open(file, len, &g) == WL_OK);
    if (!g) return;
    CHECK(wl_gguf_version(g) == 3u);
    CHECK(wl_gguf_alignment(g) == 32u);
    CHECK(wl_gguf_tensor_count(g) == 1u);
    CHECK(wl_gguf_get_str(g, "general.architecture", &arch) == WL_OK);
    CHECK(arch != NULL && strcmp(arch, "llama") == 0);
    CHECK(wl_gguf_find_tensor(g, "t", &v) == WL_OK);
    CHECK(v.n_dims == 1 && v.shape[0] == 4u && v.ggml_type == WL_GGML_F32);
    CHECK(v.data == file + data_off && v.data_len == 16u && v.scale_data == NULL);
    CHECK(wl_gguf_find_tensor(g, "absent", &v) == WL_ERR_MISSING_METADATA);
    CHECK(wl_gguf_close(g) == WL_OK);

    /* error classes of GgufFile::parse */
    file[3] = 'X';
    CHECK(wl_gguf_open(file, len, &bad) == WL_ERR_INVALID_MAGIC);
    file[3] = 'F';
    put_u32(file, 4, 1u);
    CHECK(wl_gguf_open(file, len, &bad) == WL_ERR_UNSUPPORTED_VERSION);
    put_u32(file, 4, 3u);
    CHECK(wl_gguf_open(file, len - 4, &bad) == WL_ERR_TENSOR_OUT_OF_BOUNDS);
    CHECK(bad == NULL);
}

int main(int argc, char **argv) {
    const int no_gpu = argc > 1 && strcmp(argv[1], "--no-gpu") == 0;
    CHECK(strstr(wl_version(), "sm_100a") != NULL);
    check_i2s_validation(no_gpu);
    check_linear_dispatch();
    check_noalloc_limits();
    check_argmax_empty();
    check_gguf();
    if (failures) fprintf(stderr, "%d check(s) failed\n", failures);
    return failures ? 1 : 0;
}
