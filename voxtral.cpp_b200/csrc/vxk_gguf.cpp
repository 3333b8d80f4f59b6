// GGUF model files (include/vxk.h, vxk_gguf_*): the metadata and tensor
// table of a voxtral.cpp model, read the way the reference's loader reads them
// through ggml (gguf_init_from_file with no_alloc, gguf_find_key /
// gguf_get_val_*, gguf_get_data_offset + gguf_get_tensor_offset:
// src/voxtral.cpp:1040-1190), restated from the published GGUF v3 layout
// (ggml, absent here):
//   "GGUF" u32 version u64 n_tensors u64 n_kv
//   n_kv x { string key, u32 type, value }        string = u64 length + bytes
//   n_tensors x { string name, u32 n_dims, u64 ne[n_dims], u32 ggml_type,
//                 u64 offset from the data section }
//   data section at the next multiple of general.alignment (default 32).
// The file is memory-mapped read-only; every read is bounds-checked and a
// malformed file is refused with VXK_STATUS_INVALID_ARGUMENT.
#include "vxk.h"
#include "vxk_internal.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

thread_local std::string g_gguf_open_error;

struct GgufError {
    std::string message;
};

[[noreturn]] void gfail(const std::string & m) { throw GgufError{m}; }

enum : uint32_t {
    T_U8 = 0, T_I8 = 1, T_U16 = 2, T_I16 = 3, T_U32 = 4, T_I32 = 5, T_F32 = 6, T_BOOL = 7,
    T_STR = 8, T_ARR = 9, T_U64 = 10, T_I64 = 11, T_F64 = 12
};

int scalar_size(uint32_t t) {
    switch (t) {
        case T_U8: case T_I8: case T_BOOL: return 1;
        case T_U16: case T_I16: return 2;
        case T_U32: case T_I32: case T_F32: return 4;
        case T_U64: case T_I64: case T_F64: return 8;
        default: return 0;
    }
}

// Block (values, bytes) of the ggml types a voxtral.cpp model may hold
// (tools/quantize_all.py and src/voxtral-quantize.cpp:80-115 list them).
bool type_block(int32_t t, int64_t * values, int64_t * bytes) {
    switch (t) {
        case 0: *values = 1; *bytes = 4; return true;      // F32
        case 1: *values = 1; *bytes = 2; return true;      // F16
        case 30: *values = 1; *bytes = 2; return true;     // BF16
        case 2: *values = 32; *bytes = 18; return true;    // Q4_0
        case 3: *values = 32; *bytes = 20; return true;    // Q4_1
        case 6: *values = 32; *bytes = 22; return true;    // Q5_0
        case 7: *values = 32; *bytes = 24; return true;    // Q5_1
        case 8: *values = 32; *bytes = 34; return true;    // Q8_0
        case 10: *values = 256; *bytes = 84; return true;  // Q2_K
        case 11: *values = 256; *bytes = 110; return true; // Q3_K
        case 12: *values = 256; *bytes = 144; return true; // Q4_K
        case 13: *values = 256; *bytes = 176; return true; // Q5_K
        case 14: *values = 256; *bytes = 210; return true; // Q6_K
        case 24: *values = 1; *bytes = 1; return true;     // I8
        case 25: *values = 1; *bytes = 2; return true;     // I16
        case 26: *values = 1; *bytes = 4; return true;     // I32
        default: return false;
    }
}

struct Value {
    uint32_t type = 0;
    uint32_t elem = 0;                 // arrays
    uint64_t count = 0;                // arrays
    const uint8_t * data = nullptr;    // scalars and numeric arrays: raw little-endian bytes in the map
    std::string str;                   // strings
    std::vector<std::string> strs;     // string arrays
};

class Cursor {
public:
    Cursor(const uint8_t * p, uint64_t n) : base_(p), n_(n) {}
    const uint8_t * take(uint64_t k) {
        if (k > n_ - pos_) gfail("truncated GGUF file");
        const uint8_t * r = base_ + pos_;
        pos_ += k;
        return r;
    }
    template <typename T> T get() {
        T v;
        std::memcpy(&v, take(sizeof(T)), sizeof(T));
        return v;
    }
    std::string str() {
        const uint64_t len = get<uint64_t>();
        if (len > (1ull << 30)) gfail("GGUF string too long");
        const uint8_t * p = take(len);
        return std::string(reinterpret_cast<const char *>(p), len);
    }
    uint64_t pos() const { return pos_; }

private:
    const uint8_t * base_;
    uint64_t n_;
    uint64_t pos_ = 0;
};

}  // namespace

struct vxk_gguf {
    void * map = nullptr;
    uint64_t size = 0;
    uint32_t version = 0;
    uint64_t data_start = 0;
    uint32_t alignment = 32;
    std::vector<std::string> keys;
    std::vector<Value> values;
    std::unordered_map<std::string, int64_t> key_index;
    std::vector<std::string> names;
    std::vector<vxk_gguf_tensor> tensors;
    std::unordered_map<std::string, int64_t> tensor_index;
    std::string last_error;
};

namespace {

void parse(vxk_gguf * g) {
    Cursor c(static_cast<const uint8_t *>(g->map), g->size);
    if (std::memcmp(c.take(4), "GGUF", 4) != 0) gfail("not a GGUF file (magic)");
    g->version = c.get<uint32_t>();
    if (g->version < 2 || g->version > 3) gfail("unsupported GGUF version " + std::to_string(g->version));
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    // a key takes at least 13 bytes (length, one byte, type, value) and a
    // tensor entry at least 32 (length, one byte, n_dims, one dim, type, offset)
    if (n_kv > g->size / 13 || n_tensors > g->size / 32) gfail("implausible GGUF counts");
    for (uint64_t i = 0; i < n_kv; ++i) {
        std::string key = c.str();
        Value v;
        v.type = c.get<uint32_t>();
        if (v.type == T_STR) {
            v.str = c.str();
        } else if (v.type == T_ARR) {
            v.elem = c.get<uint32_t>();
            v.count = c.get<uint64_t>();
            if (v.elem == T_STR) {
                if (v.count > (1ull << 26)) gfail("implausible GGUF string array");
                for (uint64_t j = 0; j < v.count; ++j) v.strs.push_back(c.str());
            } else {
                const int es = scalar_size(v.elem);
                if (es == 0) gfail("unsupported GGUF array element type for key " + key);
                if (v.count > g->size / (uint64_t) es) gfail("truncated GGUF array");
                v.data = c.take(v.count * (uint64_t) es);
            }
        } else {
            const int es = scalar_size(v.type);
            if (es == 0) gfail("unsupported GGUF value type for key " + key);
            v.data = c.take((uint64_t) es);
        }
        if (key == "general.alignment" && v.type == T_U32) {
            uint32_t a;
            std::memcpy(&a, v.data, 4);
            if (a == 0 || (a & (a - 1)) != 0) gfail("general.alignment is not a power of two");
            g->alignment = a;
        }
        g->key_index[key] = (int64_t) g->keys.size();
        g->keys.push_back(std::move(key));
        g->values.push_back(std::move(v));
    }
    g->names.reserve(n_tensors);
    std::vector<uint64_t> rel(n_tensors);
    for (uint64_t i = 0; i < n_tensors; ++i) {
        g->names.push_back(c.str());
        vxk_gguf_tensor t{};
        t.n_dims = (int32_t) c.get<uint32_t>();
        if (t.n_dims < 1 || t.n_dims > 4) gfail("tensor " + g->names.back() + " has " + std::to_string(t.n_dims) + " dims");
        int64_t n = 1;
        for (int d = 0; d < 4; ++d) t.ne[d] = 1;
        for (int d = 0; d < t.n_dims; ++d) {
            const uint64_t e = c.get<uint64_t>();
            if (e == 0 || e > ((uint64_t) 1 << 46) / (uint64_t) n)
                gfail("tensor " + g->names.back() + " has an implausible shape");
            t.ne[d] = (int64_t) e;
            n *= (int64_t) e;
        }
        t.type = (int32_t) c.get<uint32_t>();
        rel[i] = c.get<uint64_t>();
        int64_t bv = 0, bb = 0;
        if (type_block(t.type, &bv, &bb)) {
            if (t.ne[0] % bv != 0) gfail("tensor " + g->names.back() + ": row length not a multiple of its block");
            t.n_bytes = (uint64_t) (n / bv * bb);
        } else {
            t.n_bytes = 0;  // a type this library does not read; its bytes are not located
        }
        g->tensors.push_back(t);
    }
    const uint64_t a = g->alignment;
    g->data_start = (c.pos() + a - 1) / a * a;
    for (uint64_t i = 0; i < n_tensors; ++i) {
        vxk_gguf_tensor & t = g->tensors[i];
        t.name = g->names[i].c_str();
        if (rel[i] % a != 0) gfail("tensor " + g->names[i] + " is not aligned");
        // checked before the sum: a relative offset near 2^64 would wrap it
        if (g->data_start > g->size || rel[i] > g->size - g->data_start)
            gfail("tensor " + g->names[i] + " runs past the file");
        t.offset = g->data_start + rel[i];
        if (t.n_bytes > g->size - t.offset) gfail("tensor " + g->names[i] + " runs past the file");
        g->tensor_index[g->names[i]] = (int64_t) i;
    }
}

const Value * find_value(const vxk_gguf * g, const char * key) {
    if (!g || !key) return nullptr;
    const auto it = g->key_index.find(key);
    return it == g->key_index.end() ? nullptr : &g->values[(size_t) it->second];
}

bool read_int(const Value & v, int64_t * out) {
    switch (v.type) {
        case T_U8: *out = *v.data; return true;
        case T_I8: *out = (int8_t) *v.data; return true;
        case T_BOOL: *out = *v.data != 0; return true;
        case T_U16: { uint16_t x; std::memcpy(&x, v.data, 2); *out = x; return true; }
        case T_I16: { int16_t x; std::memcpy(&x, v.data, 2); *out = x; return true; }
        case T_U32: { uint32_t x; std::memcpy(&x, v.data, 4); *out = x; return true; }
        case T_I32: { int32_t x; std::memcpy(&x, v.data, 4); *out = x; return true; }
        case T_U64: { uint64_t x; std::memcpy(&x, v.data, 8); *out = (int64_t) x; return true; }
        case T_I64: { int64_t x; std::memcpy(&x, v.data, 8); *out = x; return true; }
        default: return false;
    }
}

}  // namespace

extern "C" {

vxk_status vxk_gguf_open(const char * path, vxk_gguf ** out) {
    if (out) *out = nullptr;
    if (!path || !out) {
        g_gguf_open_error = "null argument";
        return VXK_STATUS_INVALID_ARGUMENT;
    }
    vxk_gguf * g = new (std::nothrow) vxk_gguf();
    if (!g) return VXK_STATUS_OUT_OF_MEMORY;
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) {
        g_gguf_open_error = std::string("cannot open ") + path;
        delete g;
        return VXK_STATUS_INVALID_ARGUMENT;
    }
    struct stat st {};
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        ::close(fd);
        g_gguf_open_error = std::string("not a GGUF file (size): ") + path;
        delete g;
        return VXK_STATUS_INVALID_ARGUMENT;
    }
    g->size = (uint64_t) st.st_size;
    g->map = mmap(nullptr, (size_t) g->size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (g->map == MAP_FAILED) {
        g->map = nullptr;
        g_gguf_open_error = std::string("cannot map ") + path;
        delete g;
        return VXK_STATUS_BACKEND_ERROR;
    }
    try {
        parse(g);
    } catch (const GgufError & e) {
        g_gguf_open_error = e.message;
        vxk_gguf_close(g);
        return VXK_STATUS_INVALID_ARGUMENT;
    } catch (...) {
        g_gguf_open_error = "internal error";
        vxk_gguf_close(g);
        return VXK_STATUS_INTERNAL_ERROR;
    }
    *out = g;
    return VXK_STATUS_OK;
}

void vxk_gguf_close(vxk_gguf * g) {
    if (!g) return;
    if (g->map) munmap(g->map, (size_t) g->size);
    delete g;
}

vxk_status vxk_gguf_last_error(const vxk_gguf * g, char * buf, size_t capacity) {
    if (!buf || capacity == 0) return VXK_STATUS_INVALID_ARGUMENT;
    const std::string & m = g ? g->last_error : g_gguf_open_error;
    const size_t n = std::min(capacity - 1, m.size());
    std::memcpy(buf, m.data(), n);
    buf[n] = '\0';
    return m.size() < capacity ? VXK_STATUS_OK : VXK_STATUS_BUFFER_TOO_SMALL;
}

uint32_t vxk_gguf_version(const vxk_gguf * g) { return g ? g->version : 0u; }

int64_t vxk_gguf_n_tensors(const vxk_gguf * g) { return g ? (int64_t) g->tensors.size() : -1; }

vxk_status vxk_gguf_get_tensor(const vxk_gguf * g, int64_t i, vxk_gguf_tensor * out) {
    if (!g || !out || i < 0 || i >= (int64_t) g->tensors.size()) return VXK_STATUS_INVALID_ARGUMENT;
    *out = g->tensors[(size_t) i];
    return VXK_STATUS_OK;
}

int64_t vxk_gguf_find_tensor(const vxk_gguf * g, const char * name) {
    if (!g || !name) return -1;
    const auto it = g->tensor_index.find(name);
    return it == g->tensor_index.end() ? -1 : it->second;
}

const void * vxk_gguf_tensor_data(const vxk_gguf * g, int64_t i) {
    if (!g || i < 0 || i >= (int64_t) g->tensors.size() || g->tensors[(size_t) i].n_bytes == 0) return nullptr;
    return static_cast<const uint8_t *>(g->map) + g->tensors[(size_t) i].offset;
}

int64_t vxk_gguf_n_keys(const vxk_gguf * g) { return g ? (int64_t) g->keys.size() : -1; }

const char * vxk_gguf_key(const vxk_gguf * g, int64_t i) {
    if (!g || i < 0 || i >= (int64_t) g->keys.size()) return nullptr;
    return g->keys[(size_t) i].c_str();
}

int32_t vxk_gguf_key_type(const vxk_gguf * g, const char * key) {
    const Value * v = find_value(g, key);
    return v ? (int32_t) v->type : -1;
}

vxk_status vxk_gguf_get_int(const vxk_gguf * g, const char * key, int64_t * out) {
    const Value * v = find_value(g, key);
    if (!v || !out) return VXK_STATUS_INVALID_ARGUMENT;
    return read_int(*v, out) ? VXK_STATUS_OK : VXK_STATUS_INVALID_ARGUMENT;
}

vxk_status vxk_gguf_get_float(const vxk_gguf * g, const char * key, double * out) {
    const Value * v = find_value(g, key);
    if (!v || !out) return VXK_STATUS_INVALID_ARGUMENT;
    if (v->type == T_F32) {
        float x;
        std::memcpy(&x, v->data, 4);
        *out = x;
        return VXK_STATUS_OK;
    }
    if (v->type == T_F64) {
        std::memcpy(out, v->data, 8);
        return VXK_STATUS_OK;
    }
    return VXK_STATUS_INVALID_ARGUMENT;
}

vxk_status vxk_gguf_get_str(const vxk_gguf * g, const char * key, const char ** out) {
    const Value * v = find_value(g, key);
    if (!v || !out || v->type != T_STR) return VXK_STATUS_INVALID_ARGUMENT;
    *out = v->str.c_str();
    return VXK_STATUS_OK;
}

vxk_status vxk_gguf_get_array(const vxk_gguf * g, const char * key, int32_t * elem_type, int64_t * count,
                              const void ** data) {
    const Value * v = find_value(g, key);
    if (!v || v->type != T_ARR || !elem_type || !count || !data) return VXK_STATUS_INVALID_ARGUMENT;
    *elem_type = (int32_t) v->elem;
    *count = (int64_t) v->count;
    *data = v->elem == T_STR ? nullptr : v->data;  // string arrays: vxk_gguf_get_array_str
    return VXK_STATUS_OK;
}

vxk_status vxk_gguf_get_array_str(const vxk_gguf * g, const char * key, int64_t i, const char ** out) {
    const Value * v = find_value(g, key);
    if (!v || !out || v->type != T_ARR || v->elem != T_STR || i < 0 || i >= (int64_t) v->strs.size())
        return VXK_STATUS_INVALID_ARGUMENT;
    *out = v->strs[(size_t) i].c_str();
    return VXK_STATUS_OK;
}

vxk_status vxk_qweight_create_from_gguf(const vxk_gguf * g, const char * tensor, int32_t device, int32_t max_batch,
                                        vxk_qweight ** out) {
    if (out) *out = nullptr;
    const int64_t i = vxk_gguf_find_tensor(g, tensor);
    if (i < 0 || !out) return VXK_STATUS_INVALID_ARGUMENT;
    const vxk_gguf_tensor & t = g->tensors[(size_t) i];
    if (t.n_dims != 2 || (t.type != VXK_QTYPE_Q8_0 && t.type != VXK_QTYPE_Q4_K && t.type != VXK_QTYPE_Q6_K))
        return VXK_STATUS_INVALID_ARGUMENT;
    vxk_qweight_config c = vxk_qweight_default_config();
    c.device = device;
    c.type = (vxk_qtype) t.type;
    c.n_rows = (int32_t) t.ne[1];
    c.n_cols = (int32_t) t.ne[0];
    c.max_batch = max_batch;
    return vxk_qweight_create(&c, vxk_gguf_tensor_data(g, i), (size_t) t.n_bytes, out);
}

}  // extern "C"
