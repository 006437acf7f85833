// GGUF container reader and the device uploads built on it (include/bebelm_attn.h,
// "GGUF weights").
//
// Restates the reference's parser (src/gguf.rs:301-341, read_value :343-370, the
// little-endian bounds-checked cursor :381-432) and its ggml block table
// (src/tensor.rs:68-106) in C++: header (magic "GGUF", version 2 or 3, tensor and
// key/value counts), the metadata key/value pairs (13 value types, nested arrays),
// general.alignment (default 32), the tensor table (name, dims fastest-first, ggml
// type, offset relative to the data section), the data section at the next alignment
// boundary, and the per-tensor byte range check. Errors carry the reference's
// GgufError wording. The file is memory-mapped read-only, as GgufFile::open maps it,
// so a tensor's bytes go from the page cache straight into the device upload.
//
// On top: the model's metadata check (config::validate, src/config.rs:50-96), and the
// uploads of an attention layer's six tensors (src/model.rs:228-233, 434-439, 454)
// and of the logits head (src/model.rs:379-388) by their GGUF names.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <type_traits>
#include <unordered_map>
#include <vector>

#include "bebelm_attn.h"
#include "internal.h"

using bebelm::set_last_error;

namespace {

int ferr(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int ferr(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return set_last_error(code, buf);
}

// GGUF metadata value types (the on-disk discriminants, src/gguf.rs:64-78).
enum VT : uint32_t {
    VT_U8 = 0, VT_I8, VT_U16, VT_I16, VT_U32, VT_I32, VT_F32, VT_BOOL, VT_STRING, VT_ARRAY, VT_U64, VT_I64, VT_F64
};

struct Value {
    uint32_t type = 0;
    uint64_t u = 0;  // integers widened (signed ones sign-extended), bools, raw bits of floats
    double f = 0.0;  // F32 / F64
    std::string s;
    uint32_t elem_type = 0;
    std::vector<Value> items;
};

// (elements per block, bytes per block) of a ggml type, or (0, 0) when the reference
// does not model it (src/tensor.rs:41-100).
void ggml_block(uint32_t t, uint64_t* be, uint64_t* bb) {
    static const struct { uint32_t t; uint64_t e, b; } k[] = {
        {0, 1, 4},      {1, 1, 2},      {30, 1, 2},     {28, 1, 8},     {24, 1, 1},     {25, 1, 2},     {26, 1, 4},
        {27, 1, 8},     {2, 32, 18},    {3, 32, 20},    {6, 32, 22},    {7, 32, 24},    {8, 32, 34},    {9, 32, 36},
        {10, 256, 84},  {11, 256, 110}, {12, 256, 144}, {13, 256, 176}, {14, 256, 210}, {15, 256, 292},
    };
    for (const auto& x : k)
        if (x.t == t) {
            *be = x.e;
            *bb = x.b;
            return;
        }
    *be = *bb = 0;
}

// Strict UTF-8 check (what String::from_utf8 accepts): no overlong forms, no surrogates,
// nothing above U+10FFFF.
bool valid_utf8(const unsigned char* p, size_t n) {
    size_t i = 0;
    while (i < n) {
        const unsigned c = p[i];
        if (c < 0x80) {
            ++i;
            continue;
        }
        int len;
        unsigned cp;
        if (c >= 0xC2 && c <= 0xDF) { len = 2; cp = c & 0x1F; }
        else if (c >= 0xE0 && c <= 0xEF) { len = 3; cp = c & 0x0F; }
        else if (c >= 0xF0 && c <= 0xF4) { len = 4; cp = c & 0x07; }
        else return false;
        if (i + len > n) return false;
        for (int k = 1; k < len; ++k) {
            if ((p[i + k] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (p[i + k] & 0x3F);
        }
        if ((len == 3 && cp < 0x800) || (len == 4 && (cp < 0x10000 || cp > 0x10FFFF)) ||
            (cp >= 0xD800 && cp <= 0xDFFF))
            return false;
        i += len;
    }
    return true;
}

// Little-endian cursor over the file bytes; every read is bounds-checked.
struct Cursor {
    const unsigned char* buf;
    size_t len, pos = 0;
    int eof(uint64_t n) {
        return ferr(BEBELM_ERR_FORMAT, "unexpected end of file: need %llu bytes at offset %zu, file is %zu bytes",
                    (unsigned long long)n, pos, len);
    }
    int take(uint64_t n, const unsigned char** out) {
        if (n > len - pos) return eof(n);
        *out = buf + pos;
        pos += (size_t)n;
        return 0;
    }
    template <class T> int le(T* v) {
        const unsigned char* p;
        if (int rc = take(sizeof(T), &p)) return rc;
        uint64_t x = 0;
        for (size_t k = 0; k < sizeof(T); ++k) x |= (uint64_t)p[k] << (8 * k);
        *v = (T)x;
        return 0;
    }
    int str(std::string* s) {
        uint64_t n;
        if (int rc = le(&n)) return rc;
        const unsigned char* p;
        if (int rc = take(n, &p)) return rc;
        if (!valid_utf8(p, (size_t)n)) return ferr(BEBELM_ERR_FORMAT, "invalid UTF-8 in a GGUF string");
        s->assign(reinterpret_cast<const char*>(p), (size_t)n);
        return 0;
    }
};

template <class T> int read_int(Cursor& r, Value* v) {
    T x;
    if (int rc = r.le(&x)) return rc;
    v->u = (uint64_t)(int64_t)x;  // unsigned types zero-extend, signed ones sign-extend
    if (!std::is_signed<T>::value) v->u = (uint64_t)x;
    return 0;
}

int read_value(Cursor& r, uint32_t vt, Value* v, int depth) {
    v->type = vt;
    switch (vt) {
        case VT_U8: return read_int<uint8_t>(r, v);
        case VT_I8: return read_int<int8_t>(r, v);
        case VT_U16: return read_int<uint16_t>(r, v);
        case VT_I16: return read_int<int16_t>(r, v);
        case VT_U32: return read_int<uint32_t>(r, v);
        case VT_I32: return read_int<int32_t>(r, v);
        case VT_U64: return read_int<uint64_t>(r, v);
        case VT_I64: return read_int<int64_t>(r, v);
        case VT_BOOL: {
            uint8_t x;
            if (int rc = r.le(&x)) return rc;
            v->u = x != 0;
            return 0;
        }
        case VT_F32: {
            uint32_t x;
            if (int rc = r.le(&x)) return rc;
            float f;
            std::memcpy(&f, &x, 4);
            v->f = f;
            v->u = x;
            return 0;
        }
        case VT_F64: {
            uint64_t x;
            if (int rc = r.le(&x)) return rc;
            std::memcpy(&v->f, &x, 8);
            v->u = x;
            return 0;
        }
        case VT_STRING: return r.str(&v->s);
        case VT_ARRAY: {
            uint32_t et;
            uint64_t n;
            if (int rc = r.le(&et)) return rc;
            if (et > VT_F64) return ferr(BEBELM_ERR_FORMAT, "unknown metadata value type %u", et);
            if (int rc = r.le(&n)) return rc;
            if (depth > 64) return ferr(BEBELM_ERR_FORMAT, "metadata arrays nested too deeply");
            v->elem_type = et;
            // a malformed huge length cannot reserve much: the loop runs into the end of the file
            v->items.reserve((size_t)std::min<uint64_t>(n, 4096));
            for (uint64_t k = 0; k < n; ++k) {
                v->items.emplace_back();
                if (int rc = read_value(r, et, &v->items.back(), depth + 1)) return rc;
            }
            return 0;
        }
        default: return ferr(BEBELM_ERR_FORMAT, "unknown metadata value type %u", vt);
    }
}

struct Tensor {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type;
    uint64_t offset, data_start, data_len, n_elements;
};

}  // namespace

struct bebelm_gguf {
    // the bytes: a read-only mapping of the file, or an owned copy
    void* map = nullptr;
    size_t map_len = 0;
    std::vector<unsigned char> owned;
    const unsigned char* bytes = nullptr;
    size_t len = 0;
    uint32_t version = 0;
    uint64_t alignment = 32, data_offset = 0;
    std::unordered_map<std::string, Value> meta;
    std::vector<std::string> meta_order;  // keys in file order (first appearance)
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, size_t> by_name;
    ~bebelm_gguf() {
        if (map) munmap(map, map_len);
    }
};

namespace {

int parse(bebelm_gguf* g) {
    Cursor r{g->bytes, g->len};
    const unsigned char* magic;
    if (int rc = r.take(4, &magic)) return rc;
    if (std::memcmp(magic, "GGUF", 4) != 0)
        return ferr(BEBELM_ERR_FORMAT, "not a GGUF file (magic = [%u, %u, %u, %u])", magic[0], magic[1], magic[2],
                    magic[3]);
    if (int rc = r.le(&g->version)) return rc;
    if (g->version != 2 && g->version != 3)
        return ferr(BEBELM_ERR_FORMAT, "unsupported GGUF version %u", g->version);
    uint64_t n_tensors, n_kv;
    if (int rc = r.le(&n_tensors)) return rc;
    if (int rc = r.le(&n_kv)) return rc;
    for (uint64_t k = 0; k < n_kv; ++k) {
        std::string key;
        uint32_t vt;
        if (int rc = r.str(&key)) return rc;
        if (int rc = r.le(&vt)) return rc;
        if (vt > VT_F64) return ferr(BEBELM_ERR_FORMAT, "unknown metadata value type %u", vt);
        Value v;
        if (int rc = read_value(r, vt, &v, 0)) return rc;
        if (!g->meta.count(key)) g->meta_order.push_back(key);
        g->meta[key] = std::move(v);  // a repeated key keeps its last value, as a map insert does
    }
    auto al = g->meta.find("general.alignment");
    if (al != g->meta.end() && (al->second.type == VT_U32 || al->second.type == VT_U64)) g->alignment = al->second.u;
    struct Raw {
        std::string name;
        std::vector<uint64_t> dims;
        uint32_t type;
        uint64_t offset;
    };
    std::vector<Raw> raw;
    raw.reserve((size_t)std::min<uint64_t>(n_tensors, 1 << 16));
    for (uint64_t k = 0; k < n_tensors; ++k) {
        Raw t;
        uint32_t nd;
        if (int rc = r.str(&t.name)) return rc;
        if (int rc = r.le(&nd)) return rc;
        for (uint32_t d = 0; d < nd; ++d) {
            uint64_t x;
            if (int rc = r.le(&x)) return rc;
            t.dims.push_back(x);
        }
        if (int rc = r.le(&t.type)) return rc;
        if (int rc = r.le(&t.offset)) return rc;
        raw.push_back(std::move(t));
    }
    const uint64_t a = g->alignment, pos = r.pos;
    g->data_offset = a == 0 ? pos : (pos + a - 1) / a * a;
    for (auto& t : raw) {
        uint64_t be, bb;
        ggml_block(t.type, &be, &bb);
        // the element count as a mathematical product: its residue mod the block size, and
        // whether it exceeds 64 bits (then no file holds it), are known without overflow
        uint64_t n = 1, n_mod = be ? 1 % be : 0;
        bool huge = false, zero = false;
        for (uint64_t d : t.dims) {
            if (be) n_mod = (uint64_t)((unsigned __int128)n_mod * (d % be) % be);
            if (d == 0) zero = true;
            else if (!huge && n > UINT64_MAX / d) huge = true;
            else if (!huge) n *= d;
        }
        if (zero) n = 0, huge = false;
        if (!be || n_mod != 0)
            return ferr(BEBELM_ERR_FORMAT, "tensor '%s' has unmodeled ggml type %u", t.name.c_str(), t.type);
        const unsigned __int128 nbytes = (unsigned __int128)(n / be) * bb;
        const unsigned __int128 start = (unsigned __int128)g->data_offset + t.offset;
        if (huge || start + nbytes > (unsigned __int128)g->len)
            return ferr(BEBELM_ERR_FORMAT, "tensor '%s' data range falls outside the file", t.name.c_str());
        g->by_name.emplace(t.name, g->tensors.size());
        g->tensors.push_back(Tensor{std::move(t.name), std::move(t.dims), t.type, t.offset, (uint64_t)start,
                                    (uint64_t)nbytes, n});
    }
    return 0;
}

int finish(bebelm_gguf* g, bebelm_gguf** out) {
    if (int rc = parse(g)) {
        delete g;
        return rc;
    }
    *out = g;
    return 0;
}

const Value* find_value(const bebelm_gguf* g, const char* key) {
    if (!g || !key) return nullptr;
    auto it = g->meta.find(key);
    return it == g->meta.end() ? nullptr : &it->second;
}

bool is_int(uint32_t t) {
    return t == VT_U8 || t == VT_I8 || t == VT_U16 || t == VT_I16 || t == VT_U32 || t == VT_I32 || t == VT_U64 ||
           t == VT_I64;
}

void fill_info(const bebelm_gguf* g, const Tensor& t, bebelm_gguf_tensor* o) {
    std::memset(o, 0, sizeof *o);
    o->name = t.name.c_str();
    o->name_len = t.name.size();
    o->n_dims = (uint32_t)t.dims.size();
    for (size_t d = 0; d < t.dims.size() && d < BEBELM_GGUF_MAX_DIMS; ++d) o->dims[d] = t.dims[d];
    o->n_elements = t.n_elements;
    o->ggml_type = (int)t.type;
    o->offset = t.offset;
    o->data_start = t.data_start;
    o->data_len = t.data_len;
    o->data = g->bytes + t.data_start;
}

const Tensor* need_tensor(const bebelm_gguf* g, const std::string& name, int* rc) {
    auto it = g->by_name.find(name);
    if (it == g->by_name.end()) {
        *rc = ferr(BEBELM_ERR_NOT_FOUND, "tensor '%s' is not in the file", name.c_str());
        return nullptr;
    }
    *rc = 0;
    return &g->tensors[it->second];
}

// A 2-D weight [n_out][n_in] as stored (dims {n_in, n_out}), in a dtype the projections take.
int weight2d(const bebelm_gguf* g, const std::string& name, const Tensor** t, uint64_t* n_in, uint64_t* n_out) {
    int rc;
    *t = need_tensor(g, name, &rc);
    if (!*t) return rc;
    if ((*t)->dims.size() != 2) return ferr(BEBELM_ERR_FORMAT, "tensor '%s' is not 2-D", name.c_str());
    const uint32_t ty = (*t)->type;
    if (ty != BEBELM_GGML_F32 && ty != BEBELM_GGML_F16 && ty != BEBELM_GGML_Q4_K && ty != BEBELM_GGML_Q6_K)
        return ferr(BEBELM_ERR_UNSUPPORTED, "tensor '%s' has ggml type %u; the projections take F32, F16, Q4_K, Q6_K",
                    name.c_str(), ty);
    *n_in = (*t)->dims[0];
    *n_out = (*t)->dims[1];
    return 0;
}

// An F32 vector of n elements (the norm gains: the reference's precomputed F32 tensors,
// src/model.rs:52-76).
int gain_f32(const bebelm_gguf* g, const std::string& name, uint64_t n, const float** out) {
    int rc;
    const Tensor* t = need_tensor(g, name, &rc);
    if (!t) return rc;
    if (t->type != BEBELM_GGML_F32 || t->n_elements != n)
        return ferr(BEBELM_ERR_FORMAT, "tensor '%s' must be F32 with %llu elements", name.c_str(),
                    (unsigned long long)n);
    *out = reinterpret_cast<const float*>(g->bytes + t->data_start);
    return 0;
}

}  // namespace

extern "C" {

int bebelm_gguf_open(const char* path, bebelm_gguf** out) {
    if (!path || !out) return ferr(BEBELM_ERR_INVALID, "null argument");
    *out = nullptr;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return ferr(BEBELM_ERR_IO, "io error: cannot open '%s': %s", path, strerror(errno));
    struct stat st;
    if (fstat(fd, &st) != 0) {
        const int e = errno;
        close(fd);
        return ferr(BEBELM_ERR_IO, "io error: cannot stat '%s': %s", path, strerror(e));
    }
    auto* g = new bebelm_gguf();
    g->len = (size_t)st.st_size;
    if (g->len) {
        void* m = mmap(nullptr, g->len, PROT_READ, MAP_PRIVATE, fd, 0);
        if (m == MAP_FAILED) {
            const int e = errno;
            close(fd);
            delete g;
            return ferr(BEBELM_ERR_IO, "io error: cannot map '%s': %s", path, strerror(e));
        }
        g->map = m;
        g->map_len = g->len;
        g->bytes = static_cast<const unsigned char*>(m);
    } else {
        g->owned.assign(1, 0);
        g->bytes = g->owned.data();
    }
    close(fd);
    return finish(g, out);
}

int bebelm_gguf_from_bytes(const void* data, size_t n, bebelm_gguf** out) {
    if (!out || (!data && n)) return ferr(BEBELM_ERR_INVALID, "null argument");
    *out = nullptr;
    auto* g = new bebelm_gguf();
    const auto* p = static_cast<const unsigned char*>(data);
    g->owned.assign(p, p + n);
    g->owned.push_back(0);  // keeps bytes non-null for an empty input
    g->bytes = g->owned.data();
    g->len = n;
    return finish(g, out);
}

int bebelm_gguf_close(bebelm_gguf* g) {
    delete g;
    return 0;
}

int bebelm_gguf_header(const bebelm_gguf* g, uint32_t* version, uint64_t* alignment, uint64_t* data_offset,
                       size_t* n_tensors, size_t* n_kv) {
    if (!g) return ferr(BEBELM_ERR_INVALID, "null handle");
    if (version) *version = g->version;
    if (alignment) *alignment = g->alignment;
    if (data_offset) *data_offset = g->data_offset;
    if (n_tensors) *n_tensors = g->tensors.size();
    if (n_kv) *n_kv = g->meta.size();
    return 0;
}

int bebelm_gguf_tensor_at(const bebelm_gguf* g, size_t i, bebelm_gguf_tensor* out) {
    if (!g || !out) return ferr(BEBELM_ERR_INVALID, "null argument");
    if (i >= g->tensors.size()) return ferr(BEBELM_ERR_INVALID, "tensor index %zu out of range", i);
    fill_info(g, g->tensors[i], out);
    return 0;
}

int bebelm_gguf_find_tensor(const bebelm_gguf* g, const char* name, bebelm_gguf_tensor* out) {
    if (!g || !name || !out) return ferr(BEBELM_ERR_INVALID, "null argument");
    int rc;
    const Tensor* t = need_tensor(g, name, &rc);
    if (!t) return rc;
    fill_info(g, *t, out);
    return 0;
}

int bebelm_gguf_key_at(const bebelm_gguf* g, size_t i, const char** key, size_t* key_len, int* value_type) {
    if (!g || !key) return ferr(BEBELM_ERR_INVALID, "null argument");
    if (i >= g->meta_order.size()) return ferr(BEBELM_ERR_INVALID, "key index %zu out of range", i);
    *key = g->meta_order[i].c_str();
    if (key_len) *key_len = g->meta_order[i].size();
    if (value_type) *value_type = (int)g->meta.at(g->meta_order[i]).type;
    return 0;
}

int bebelm_gguf_get_u32(const bebelm_gguf* g, const char* key, uint32_t* out) {
    if (!out) return ferr(BEBELM_ERR_INVALID, "null argument");
    const Value* v = find_value(g, key);
    if (!v || !is_int(v->type)) return ferr(BEBELM_ERR_NOT_FOUND, "no integer metadata '%s'", key ? key : "");
    *out = (uint32_t)v->u;  // widened, then truncated as `as u32` does
    return 0;
}

int bebelm_gguf_get_f32(const bebelm_gguf* g, const char* key, float* out) {
    if (!out) return ferr(BEBELM_ERR_INVALID, "null argument");
    const Value* v = find_value(g, key);
    if (!v || (v->type != VT_F32 && v->type != VT_F64))
        return ferr(BEBELM_ERR_NOT_FOUND, "no float metadata '%s'", key ? key : "");
    *out = (float)v->f;
    return 0;
}

int bebelm_gguf_get_str(const bebelm_gguf* g, const char* key, char* buf, size_t cap, size_t* len) {
    const Value* v = find_value(g, key);
    if (!v || v->type != VT_STRING) return ferr(BEBELM_ERR_NOT_FOUND, "no string metadata '%s'", key ? key : "");
    if (len) *len = v->s.size();
    if (buf && cap) {
        const size_t n = std::min(cap - 1, v->s.size());
        std::memcpy(buf, v->s.data(), n);
        buf[n] = 0;
    }
    return 0;
}

int bebelm_gguf_get_u32_array(const bebelm_gguf* g, const char* key, uint32_t* out, size_t cap, size_t* len) {
    const Value* v = find_value(g, key);
    if (!v || v->type != VT_ARRAY) return ferr(BEBELM_ERR_NOT_FOUND, "no array metadata '%s'", key ? key : "");
    for (const Value& it : v->items)
        if (!is_int(it.type)) return ferr(BEBELM_ERR_NOT_FOUND, "metadata '%s' is not an integer array", key);
    if (len) *len = v->items.size();
    for (size_t k = 0; out && k < cap && k < v->items.size(); ++k) out[k] = (uint32_t)v->items[k].u;
    return 0;
}

int bebelm_gguf_array_len(const bebelm_gguf* g, const char* key, int* elem_type, size_t* len) {
    const Value* v = find_value(g, key);
    if (!v || v->type != VT_ARRAY) return ferr(BEBELM_ERR_NOT_FOUND, "no array metadata '%s'", key ? key : "");
    if (elem_type) *elem_type = (int)v->elem_type;
    if (len) *len = v->items.size();
    return 0;
}

int bebelm_gguf_get_str_at(const bebelm_gguf* g, const char* key, size_t i, const char** s, size_t* len) {
    const Value* v = find_value(g, key);
    if (!v || v->type != VT_ARRAY) return ferr(BEBELM_ERR_NOT_FOUND, "no array metadata '%s'", key ? key : "");
    if (i >= v->items.size() || v->items[i].type != VT_STRING)
        return ferr(BEBELM_ERR_NOT_FOUND, "metadata '%s' has no string at %zu", key, i);
    if (s) *s = v->items[i].s.c_str();
    if (len) *len = v->items[i].s.size();
    return 0;
}

// config::validate (src/config.rs:50-96): the metadata must match LFM2.5-8B-A1B.
int bebelm_gguf_validate(const bebelm_gguf* g) {
    if (!g) return ferr(BEBELM_ERR_INVALID, "null handle");
    const Value* arch = find_value(g, "general.architecture");
    if (!arch || arch->type != VT_STRING) return ferr(BEBELM_ERR_FORMAT, "missing general.architecture");
    if (arch->s != "lfm2moe")
        return ferr(BEBELM_ERR_FORMAT, "architecture: expected \"lfm2moe\", got \"%s\"", arch->s.c_str());
    static const struct { const char* key; uint32_t want; } ints[] = {
        {"lfm2moe.block_count", 24}, {"lfm2moe.embedding_length", 2048}, {"lfm2moe.vocab_size", 128000},
        {"lfm2moe.attention.head_count", 32}, {"lfm2moe.expert_count", 32}, {"lfm2moe.expert_used_count", 4},
        {"lfm2moe.feed_forward_length", 7168}, {"lfm2moe.expert_feed_forward_length", 1792},
        {"lfm2moe.leading_dense_block_count", 2}, {"lfm2moe.shortconv.l_cache", 3},
    };
    for (const auto& e : ints) {
        uint32_t got;
        if (bebelm_gguf_get_u32(g, e.key, &got)) return ferr(BEBELM_ERR_FORMAT, "missing metadata %s", e.key);
        if (got != e.want) return ferr(BEBELM_ERR_FORMAT, "%s: expected %u, got %u", e.key, e.want, got);
    }
    static const struct { const char* key; float want, tol; } fls[] = {
        {"lfm2moe.rope.freq_base", 5000000.0f, 1.0f}, {"lfm2moe.attention.layer_norm_rms_epsilon", 1e-5f, 1e-9f}};
    for (const auto& e : fls) {
        float got;
        if (bebelm_gguf_get_f32(g, e.key, &got)) return ferr(BEBELM_ERR_FORMAT, "missing metadata %s", e.key);
        if (std::fabs(got - e.want) > e.tol)
            return ferr(BEBELM_ERR_FORMAT, "%s: expected %g, got %g", e.key, e.want, got);
    }
    size_t n = 0;
    uint32_t kv[64];
    if (bebelm_gguf_get_u32_array(g, "lfm2moe.attention.head_count_kv", kv, 64, &n))
        return ferr(BEBELM_ERR_FORMAT, "attention.head_count_kv missing or not an array");
    if (n != 24) return ferr(BEBELM_ERR_FORMAT, "head_count_kv has %zu entries, expected 24", n);
    static const int attn[] = {2, 6, 10, 14, 18, 21};
    for (size_t i = 0; i < n; ++i) {
        bool is_attn = false;
        for (int a : attn) is_attn |= (int)i == a;
        const uint32_t want = is_attn ? 8 : 0;
        if (kv[i] != want)
            return ferr(BEBELM_ERR_FORMAT, "layer %zu: head_count_kv=%u, expected %u (schedule mismatch)", i, kv[i],
                        want);
    }
    return 0;
}

int bebelm_attn_weights_from_gguf(const bebelm_gguf* g, int block, int device, bebelm_attn_weights** out) {
    if (!g || !out) return ferr(BEBELM_ERR_INVALID, "null argument");
    *out = nullptr;
    const std::string p = "blk." + std::to_string(block) + ".";
    const Tensor *tq, *tk, *tv, *to;
    uint64_t qi, qo, ki, ko, vi, vo, oi, oo;
    if (int rc = weight2d(g, p + "attn_q.weight", &tq, &qi, &qo)) return rc;
    if (int rc = weight2d(g, p + "attn_k.weight", &tk, &ki, &ko)) return rc;
    if (int rc = weight2d(g, p + "attn_v.weight", &tv, &vi, &vo)) return rc;
    if (int rc = weight2d(g, p + "attn_output.weight", &to, &oi, &oo)) return rc;
    const uint64_t hidden = qi;
    if (ki != hidden || vi != hidden || ko != vo || oi != qo || oo != hidden || qo % 64 || ko % 64)
        return ferr(BEBELM_ERR_FORMAT, "%sattn_* tensors have inconsistent shapes", p.c_str());
    const float *qg, *kg;
    if (int rc = gain_f32(g, p + "attn_q_norm.weight", 64, &qg)) return rc;
    if (int rc = gain_f32(g, p + "attn_k_norm.weight", 64, &kg)) return rc;
    return bebelm_attn_weights_create(device, (int)(qo / 64), (int)(ko / 64), (size_t)hidden, (int)tq->type,
                                      g->bytes + tq->data_start, (int)tk->type, g->bytes + tk->data_start,
                                      (int)tv->type, g->bytes + tv->data_start, (int)to->type,
                                      g->bytes + to->data_start, qg, kg, out);
}

int bebelm_head_from_gguf(const bebelm_gguf* g, int device, bebelm_head** out) {
    if (!g || !out) return ferr(BEBELM_ERR_INVALID, "null argument");
    *out = nullptr;
    const Tensor* te;
    uint64_t hidden, vocab;
    if (int rc = weight2d(g, "token_embd.weight", &te, &hidden, &vocab)) return rc;
    const float* gain;
    if (int rc = gain_f32(g, "token_embd_norm.weight", hidden, &gain)) return rc;
    return bebelm_head_create(device, (int)te->type, g->bytes + te->data_start, (size_t)hidden, (size_t)vocab, gain,
                              out);
}

}  // extern "C"
