// gguf.h -- host-side GGUF v2 / v3 reader over the caller's bytes (an mmap of
// the model file), zero-copy: tensor data pointers point into those bytes.
//
// Reference: GgufFile::parse (src/gguf/reader.rs:120-415) with its limits
// (reader.rs:19-25), string / value / array readers (reader.rs:453-668),
// tensor byte lengths (compute_tensor_byte_len, reader.rs:688-770, and the
// row-based Q4_0 / Q8_0 / Q4_K / Q6_K rules of src/gguf/tensor.rs:112-230),
// and the I2_S 32-byte trailing scale block (reader.rs:360-395).  The checks
// and their order follow the reference so a file it rejects is rejected here
// with the matching error class.
#pragma once

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

namespace wl_gguf_detail {

enum : uint32_t {
    GV_U8 = 0, GV_I8 = 1, GV_U16 = 2, GV_I16 = 3, GV_U32 = 4, GV_I32 = 5, GV_F32 = 6,
    GV_BOOL = 7, GV_STR = 8, GV_ARR = 9, GV_U64 = 10, GV_I64 = 11, GV_F64 = 12
};

constexpr uint32_t GGUF_MAGIC = 0x46554747u;  // "GGUF"
constexpr uint64_t DEFAULT_ALIGNMENT = 32;
constexpr uint64_t MAX_TENSORS = 1000000, MAX_KV = 1000000, MAX_ARRAY = 1000000;
constexpr uint32_t MAX_DIMS = 4;
constexpr size_t MAX_ARRAY_DEPTH = 16;
constexpr uint64_t MAX_STRING = 1048576;
constexpr uint64_t I2S_SCALE_BLOCK = 32;

struct Value {
    uint32_t type = 0;
    uint64_t u = 0;   // unsigned types, bool
    int64_t i = 0;    // signed types
    double f = 0.0;   // f32 / f64
    std::string s;
    std::vector<Value> arr;

    bool as_u64(uint64_t *out) const {  // GgufValue::as_u64 (reader.rs:48-58)
        switch (type) {
        case GV_U8: case GV_U16: case GV_U32: case GV_U64: *out = u; return true;
        case GV_I32: case GV_I64: if (i >= 0) { *out = (uint64_t)i; return true; } return false;
        default: return false;
        }
    }
    bool as_f32(float *out) const {  // GgufValue::as_f32 (reader.rs:69-75)
        if (type == GV_F32 || type == GV_F64) { *out = (float)f; return true; }
        return false;
    }
};

struct Tensor {
    std::string name;
    std::vector<uint64_t> shape;
    uint32_t type = 0;
    uint64_t offset = 0, byte_len = 0;  // absolute file offset, packed bytes
    const uint8_t *data = nullptr;
    const uint8_t *scale = nullptr;     // I2_S trailing block, else null
};

// Error classes of WillametteError the reader produces.
enum Err { OK = 0, PARSE, MAGIC, VERSION, OOB };

struct Cursor {
    const uint8_t *p;
    uint64_t len, pos = 0;
    bool take(void *dst, uint64_t n) {
        if (n > len - pos) return false;
        memcpy(dst, p + pos, n);
        pos += n;
        return true;
    }
    template <typename T> bool get(T *v) { return take(v, sizeof(T)); }
    uint64_t remaining() const { return len - pos; }
};

struct Parser {
    Cursor c;
    std::string msg;
    Err fail(Err e, const std::string &m) {
        msg = m;
        return e;
    }

    bool read_string(std::string *s, std::string *why) {
        uint64_t n;
        if (!c.get(&n)) { *why = "string length: unexpected end of file"; return false; }
        if (n > MAX_STRING) { *why = "string length " + std::to_string(n) + " exceeds 1 MiB safety limit"; return false; }
        if (n > c.remaining()) { *why = "string body (" + std::to_string(n) + " bytes): unexpected end of file"; return false; }
        s->assign(reinterpret_cast<const char *>(c.p + c.pos), n);
        c.pos += n;
        return true;  // (UTF-8 validity is not checked here: keys and names are compared as bytes)
    }

    static int elem_bytes(uint32_t t) {  // validate_array's minimum sizes (reader.rs:645-657)
        switch (t) {
        case GV_U8: case GV_I8: case GV_BOOL: return 1;
        case GV_U16: case GV_I16: return 2;
        case GV_U32: case GV_I32: case GV_F32: return 4;
        case GV_U64: case GV_I64: case GV_F64: case GV_STR: return 8;
        case GV_ARR: return 12;
        default: return -1;
        }
    }

    bool read_typed(uint32_t t, Value *v, size_t depth, std::string *why) {
        v->type = t;
        switch (t) {
        case GV_U8: { uint8_t x; if (!c.get(&x)) break; v->u = x; return true; }
        case GV_I8: { int8_t x; if (!c.get(&x)) break; v->i = x; return true; }
        case GV_U16: { uint16_t x; if (!c.get(&x)) break; v->u = x; return true; }
        case GV_I16: { int16_t x; if (!c.get(&x)) break; v->i = x; return true; }
        case GV_U32: { uint32_t x; if (!c.get(&x)) break; v->u = x; return true; }
        case GV_I32: { int32_t x; if (!c.get(&x)) break; v->i = x; return true; }
        case GV_F32: { float x; if (!c.get(&x)) break; v->f = x; return true; }
        case GV_BOOL: { uint8_t x; if (!c.get(&x)) break; v->u = x != 0; return true; }
        case GV_STR: return read_string(&v->s, why);
        case GV_U64: { uint64_t x; if (!c.get(&x)) break; v->u = x; return true; }
        case GV_I64: { int64_t x; if (!c.get(&x)) break; v->i = x; return true; }
        case GV_F64: { double x; if (!c.get(&x)) break; v->f = x; return true; }
        case GV_ARR: {
            uint32_t et;
            uint64_t n;
            if (!c.get(&et) || !c.get(&n)) break;
            const size_t d = depth + 1;
            if (d > MAX_ARRAY_DEPTH) { *why = "metadata array nesting depth " + std::to_string(d) + " exceeds 16"; return false; }
            if (n > MAX_ARRAY) { *why = "array count " + std::to_string(n) + " exceeds safety limit 1000000"; return false; }
            const int eb = elem_bytes(et);
            if (eb < 0) { *why = "unknown type tag " + std::to_string(et) + " in array element"; return false; }
            if (n * (uint64_t)eb > c.remaining()) {
                *why = "array of " + std::to_string(n) + " elements cannot fit in " +
                       std::to_string(c.remaining()) + " remaining bytes";
                return false;
            }
            v->arr.resize(n);
            for (uint64_t k = 0; k < n; ++k)
                if (!read_typed(et, &v->arr[k], d, why)) {
                    *why = "array[" + std::to_string(k) + "]: " + *why;
                    return false;
                }
            return true;
        }
        default:
            *why = "unknown metadata value type: " + std::to_string(t);
            return false;
        }
        *why = "unexpected end of file";
        return false;
    }
};

inline bool align_up(uint64_t off, uint64_t a, uint64_t *out) {
    const uint64_t r = off % a;
    if (r == 0) { *out = off; return true; }
    if (off > UINT64_MAX - (a - r)) return false;
    *out = off + (a - r);
    return true;
}

// compute_tensor_byte_len (reader.rs:688-770): false + why on error,
// *known = false when the type's layout is unknown.
inline bool tensor_byte_len(const std::vector<uint64_t> &shape, uint32_t type, uint64_t *out,
                            bool *known, std::string *why) {
    *known = true;
    struct RowRule { uint32_t type; uint64_t per, bytes; const char *name; };
    static const RowRule rows[] = {{2, 32, 18, "Q4_0"}, {14, 256, 210, "Q6_K"}, {12, 256, 144, "Q4_K"},
                                   {8, 32, 34, "Q8_0"}};
    for (const RowRule &r : rows) {
        if (type != r.type) continue;
        if (shape.empty()) { *why = std::string(r.name) + " tensor has no dimensions"; return false; }
        const uint64_t row = shape[0];
        if (row == 0) { *out = 0; return true; }
        if (row % r.per) {
            *why = std::string(r.name) + " row length " + std::to_string(row) + " is not a multiple of " + std::to_string(r.per);
            return false;
        }
        uint64_t n = 1;
        for (size_t d = 1; d < shape.size(); ++d) {
            if (shape[d] && n > UINT64_MAX / shape[d]) { *why = std::string(r.name) + " row count overflow"; return false; }
            n *= shape[d];
        }
        const uint64_t rb = row / r.per * r.bytes;
        if (n && rb > UINT64_MAX / n) { *why = std::string(r.name) + " byte length overflow"; return false; }
        *out = rb * n;
        return true;
    }
    uint64_t n = 1;
    for (uint64_t d : shape) {
        if (d && n > UINT64_MAX / d) { *why = "shape product overflow"; return false; }
        n *= d;
    }
    if (n == 0) { *out = 0; return true; }
    uint64_t per = 0, bytes = 0;
    switch (type) {
    case 0: per = 1; bytes = 4; break;    // F32
    case 1: per = 1; bytes = 2; break;    // F16
    case 30: per = 1; bytes = 2; break;   // BF16
    case 28: per = 1; bytes = 8; break;   // F64
    case 24: per = 1; bytes = 1; break;   // I8
    case 25: per = 1; bytes = 2; break;   // I16
    case 26: per = 1; bytes = 4; break;   // I32
    case 27: per = 1; bytes = 8; break;   // I64
    case 3: per = 32; bytes = 20; break;  // Q4_1
    case 6: per = 32; bytes = 22; break;  // Q5_0
    case 7: per = 32; bytes = 24; break;  // Q5_1
    case 9: per = 32; bytes = 40; break;  // Q8_1
    case 10: per = 256; bytes = 84; break;   // Q2_K
    case 11: per = 256; bytes = 110; break;  // Q3_K
    case 13: per = 256; bytes = 176; break;  // Q5_K
    case 15: per = 256; bytes = 292; break;  // Q8_K
    case 36: per = 128; bytes = 32; break;   // I2_S: 2 bits per element
    case 37: per = 1; bytes = 1; break;      // I8_S
    default: *known = false; return true;
    }
    if (n % per) {
        *why = "element count " + std::to_string(n) + " is not divisible by block size " + std::to_string(per);
        return false;
    }
    if (n / per > UINT64_MAX / bytes) { *why = "byte length overflow"; return false; }
    *out = n / per * bytes;
    return true;
}

}  // namespace wl_gguf_detail

struct wl_gguf {
    uint32_t version = 0;
    uint64_t alignment = 0, data_start = 0, file_len = 0;
    std::map<std::string, wl_gguf_detail::Value> meta;
    std::vector<wl_gguf_detail::Tensor> tensors;
    std::unordered_map<std::string, size_t> by_name;
};

namespace wl_gguf_detail {

// GgufFile::parse.  Returns OK, or an error class with p.msg set.
inline Err parse(const uint8_t *data, uint64_t len, wl_gguf *g, Parser &p) {
    p.c = Cursor{data, len, 0};
    uint32_t magic, version;
    if (!p.c.get(&magic)) return p.fail(PARSE, "reading magic: unexpected end of file");
    if (magic != GGUF_MAGIC) {
        char b[64];
        snprintf(b, sizeof b, "Invalid GGUF magic (expected 0x46554747, got 0x%08X)", magic);
        return p.fail(MAGIC, b);
    }
    if (!p.c.get(&version)) return p.fail(PARSE, "reading version: unexpected end of file");
    if (version != 2 && version != 3)
        return p.fail(VERSION, "Unsupported GGUF version: " + std::to_string(version) + " (supported: 2, 3)");
    uint64_t n_tensors, n_kv;
    if (!p.c.get(&n_tensors)) return p.fail(PARSE, "reading tensor_count: unexpected end of file");
    if (!p.c.get(&n_kv)) return p.fail(PARSE, "reading metadata_kv_count: unexpected end of file");
    auto count_ok = [&](const char *what, uint64_t n, uint64_t limit, uint64_t min_entry) -> Err {
        if (n > limit)
            return p.fail(PARSE, std::string(what) + " " + std::to_string(n) + " exceeds safety limit " + std::to_string(limit));
        if (n > p.c.remaining() / min_entry + 1 || n * min_entry > p.c.remaining())
            return p.fail(PARSE, std::string(what) + " " + std::to_string(n) + " cannot fit in " +
                                     std::to_string(p.c.remaining()) + " remaining bytes");
        return OK;
    };
    Err e;
    if ((e = count_ok("tensor_count", n_tensors, MAX_TENSORS, 24))) return e;
    if ((e = count_ok("metadata_kv_count", n_kv, MAX_KV, 13))) return e;
    for (uint64_t k = 0; k < n_kv; ++k) {
        std::string key, why;
        if (!p.read_string(&key, &why))
            return p.fail(PARSE, "metadata[" + std::to_string(k) + "] key: " + why);
        uint32_t t;
        Value v;
        if (!p.c.get(&t)) why = "value type tag: unexpected end of file";
        if (why.empty() && p.read_typed(t, &v, 0, &why)) {
            g->meta[key] = std::move(v);
            continue;
        }
        return p.fail(PARSE, "metadata[" + std::to_string(k) + "] (key=\"" + key + "\") value: " + why);
    }
    uint64_t alignment = DEFAULT_ALIGNMENT;
    auto it = g->meta.find("general.alignment");
    if (it != g->meta.end()) {
        uint64_t a;
        if (it->second.as_u64(&a)) alignment = a;
    }
    if (alignment == 0 || (alignment & (alignment - 1)))
        return p.fail(PARSE, "invalid alignment value: " + std::to_string(alignment));
    if ((e = count_ok("tensor_count", n_tensors, MAX_TENSORS, 24))) return e;
    std::vector<uint64_t> rel(n_tensors);
    g->tensors.resize(n_tensors);
    for (uint64_t k = 0; k < n_tensors; ++k) {
        Tensor &t = g->tensors[k];
        std::string why;
        const std::string pre = "tensor[" + std::to_string(k) + "] ";
        if (!p.read_string(&t.name, &why)) return p.fail(PARSE, pre + "name: " + why);
        uint32_t nd;
        if (!p.c.get(&nd)) return p.fail(PARSE, pre + "n_dims: unexpected end of file");
        if (nd > MAX_DIMS) return p.fail(PARSE, pre + "n_dims " + std::to_string(nd) + " exceeds 4");
        t.shape.resize(nd);
        for (uint32_t d = 0; d < nd; ++d)
            if (!p.c.get(&t.shape[d])) return p.fail(PARSE, pre + "shape[" + std::to_string(d) + "]: unexpected end of file");
        if (!p.c.get(&t.type)) return p.fail(PARSE, pre + "ggml_type: unexpected end of file");
        if (!p.c.get(&rel[k])) return p.fail(PARSE, pre + "offset: unexpected end of file");
    }
    uint64_t data_start;
    if (!align_up(p.c.pos, alignment, &data_start)) return p.fail(PARSE, "tensor data section offset overflow");
    if (n_tensors && data_start > len)
        return p.fail(PARSE, "tensor data section starts beyond EOF: " + std::to_string(data_start) + " > " +
                                 std::to_string(len));
    // offsets sorted once: "next tensor" bounds and duplicate offsets
    std::vector<uint64_t> sorted(rel);
    std::sort(sorted.begin(), sorted.end());
    for (uint64_t k = 0; k < n_tensors; ++k) {
        Tensor &t = g->tensors[k];
        if (rel[k] > UINT64_MAX - data_start) return p.fail(PARSE, "tensor \"" + t.name + "\" offset overflow");
        const uint64_t abs = data_start + rel[k];
        auto lo = std::lower_bound(sorted.begin(), sorted.end(), rel[k]);
        if (lo + 1 != sorted.end() && *(lo + 1) == rel[k])
            return p.fail(PARSE, "tensor \"" + t.name + "\" shares data offset " + std::to_string(rel[k]) +
                                     " with another tensor");
        bool has_next = false;
        uint64_t next_abs = 0;
        auto up = std::upper_bound(sorted.begin(), sorted.end(), rel[k]);
        if (up != sorted.end()) {
            if (*up > UINT64_MAX - data_start) return p.fail(PARSE, "tensor \"" + t.name + "\" next offset overflow");
            has_next = true;
            next_abs = data_start + *up;
        }
        uint64_t bl = 0;
        bool known = true;
        std::string why;
        if (!tensor_byte_len(t.shape, t.type, &bl, &known, &why))
            return p.fail(PARSE, "tensor \"" + t.name + "\": " + why);
        if (!known)
            return p.fail(PARSE, "tensor \"" + t.name + "\" has unsupported type " + std::to_string(t.type) +
                                     "; byte length is unknown");
        if (bl > UINT64_MAX - abs) return p.fail(PARSE, "tensor \"" + t.name + "\" end offset overflow");
        const uint64_t end = abs + bl;
        if (end > len)
            return p.fail(OOB, "Tensor data out of bounds: tensor \"" + t.name + "\" requires bytes [" +
                                   std::to_string(abs) + ".." + std::to_string(end) + "), file size = " +
                                   std::to_string(len));
        if (has_next && end > next_abs)
            return p.fail(PARSE, "tensor \"" + t.name + "\" range " + std::to_string(abs) + ".." +
                                     std::to_string(end) + " overlaps next tensor at " + std::to_string(next_abs));
        t.offset = abs;
        t.byte_len = bl;
        t.data = data + abs;
        if (t.type == 36) {  // I2_S: 32-byte trailing block (f32 scale + padding)
            if (end > UINT64_MAX - I2S_SCALE_BLOCK)
                return p.fail(PARSE, "tensor \"" + t.name + "\" scale-block offset overflow");
            const uint64_t se = end + I2S_SCALE_BLOCK;
            if (se > len)
                return p.fail(OOB, "Tensor data out of bounds: tensor \"" + t.name + " (scale block)\" requires bytes [" +
                                       std::to_string(end) + ".." + std::to_string(se) + "), file size = " +
                                       std::to_string(len));
            if (has_next && se > next_abs)
                return p.fail(PARSE, "I2_S tensor \"" + t.name + "\" scale block ends at " + std::to_string(se) +
                                         ", overlapping next tensor at " + std::to_string(next_abs));
            t.scale = data + end;
        }
    }
    g->version = version;
    g->alignment = alignment;
    g->data_start = data_start;
    g->file_len = len;
    for (size_t k = 0; k < g->tensors.size(); ++k) g->by_name.emplace(g->tensors[k].name, k);
    return OK;
}

}  // namespace wl_gguf_detail
