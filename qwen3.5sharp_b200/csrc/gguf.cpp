// gguf.cpp -- GGUF v2/v3 reader (memory-mapped, host only) and weight upload
// straight from the mapped file (include/q35k.h, "GGUF ingestion").
//
// Behaviour follows the reference reader (Qwen35Sharp.Gguf/GgufFile.cs):
// little-endian fields, metadata parsed at open (:110-139), alignment from
// general.alignment (default 32, a power of two, :141-143), tensor infos of
// 1..4 non-negative dims with type and data-section offset (:145-163), data
// section at the aligned end of the infos (:166-171).  Every read is bounds
// checked: a truncated or corrupt file is an error status, never a crash.
#include "../../include/q35k.h"
#include "api_internal.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <climits>
#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace q35k {
void set_thread_error(const std::string& msg);
}

namespace {

enum ValueType {
    V_U8 = 0, V_I8 = 1, V_U16 = 2, V_I16 = 3, V_U32 = 4, V_I32 = 5, V_F32 = 6, V_BOOL = 7,
    V_STRING = 8, V_ARRAY = 9, V_U64 = 10, V_I64 = 11, V_F64 = 12,
};

struct Value {
    int type = -1;   // ValueType; V_ARRAY for arrays
    int elem = -1;   // element type of an array
    uint64_t count = 0;
    bool is_int = false, is_float = false;
    int64_t i = 0;
    double f = 0.0;
    std::string s;
    bool i_overflow = false;  // a u64 above INT64_MAX (not an int64)
};

struct Tensor {
    std::string name;
    int type = 0;
    int n_dims = 0;
    int64_t dims[4] = {0, 0, 0, 0};
    uint64_t offset = 0;
};

struct ParseError {
    int code;
    std::string msg;
};

class Cursor {
public:
    Cursor(const uint8_t* base, uint64_t len) : base_(base), len_(len) {}
    uint64_t pos() const { return pos_; }
    template <typename T>
    T read() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, base_ + pos_, sizeof(T));
        pos_ += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = read<uint64_t>();
        if (n > (uint64_t)INT_MAX) throw ParseError{Q35K_EDATA, "GGUF string length " + std::to_string(n) + " exceeds 2 GB"};
        need(n);
        std::string s(reinterpret_cast<const char*>(base_ + pos_), (size_t)n);
        pos_ += n;
        return s;
    }

private:
    void need(uint64_t n) const {
        if (n > len_ || pos_ > len_ - n) throw ParseError{Q35K_EDATA, "unexpected end of GGUF file"};
    }
    const uint8_t* base_;
    uint64_t len_, pos_ = 0;
};

Value read_scalar(Cursor& c, int type) {
    Value v;
    v.type = type;
    switch (type) {
    case V_U8: v.i = c.read<uint8_t>(); v.is_int = true; break;
    case V_I8: v.i = c.read<int8_t>(); v.is_int = true; break;
    case V_U16: v.i = c.read<uint16_t>(); v.is_int = true; break;
    case V_I16: v.i = c.read<int16_t>(); v.is_int = true; break;
    case V_U32: v.i = c.read<uint32_t>(); v.is_int = true; break;
    case V_I32: v.i = c.read<int32_t>(); v.is_int = true; break;
    case V_U64: {
        const uint64_t u = c.read<uint64_t>();
        v.i_overflow = u > (uint64_t)INT64_MAX;
        v.i = (int64_t)u;
        v.is_int = !v.i_overflow;
        break;
    }
    case V_I64: v.i = c.read<int64_t>(); v.is_int = true; break;
    case V_F32: v.f = c.read<float>(); v.is_float = true; break;
    case V_F64: v.f = c.read<double>(); v.is_float = true; break;
    case V_BOOL: v.i = c.read<uint8_t>() != 0; break;  // not coerced to an integer
    case V_STRING: v.s = c.str(); break;
    case V_ARRAY: throw ParseError{Q35K_EDATA, "nested GGUF arrays are not supported"};
    default: throw ParseError{Q35K_EDATA, "unknown GGUF value type " + std::to_string(type)};
    }
    return v;
}

Value read_value(Cursor& c) {
    const int type = c.read<int32_t>();
    if (type != V_ARRAY) return read_scalar(c, type);
    Value v;
    v.type = V_ARRAY;
    v.elem = c.read<int32_t>();
    v.count = c.read<uint64_t>();
    if (v.count > (uint64_t)INT_MAX)
        throw ParseError{Q35K_EDATA, "GGUF array length " + std::to_string(v.count) + " exceeds int.MaxValue"};
    for (uint64_t k = 0; k < v.count; k++) (void)read_scalar(c, v.elem);  // elements are skipped
    return v;
}

}  // namespace

struct q35k_gguf {
    int fd = -1;
    const uint8_t* base = nullptr;
    uint64_t len = 0;
    uint64_t data = 0;  // file offset of the data section
    int version = 0;
    uint32_t alignment = 32;
    std::unordered_map<std::string, Value> kv;
    std::vector<Tensor> tensors;                  // file order
    std::unordered_map<std::string, int> by_name;  // a later duplicate replaces an earlier one

    ~q35k_gguf() {
        if (base) munmap(const_cast<uint8_t*>(base), (size_t)len);
        if (fd >= 0) close(fd);
    }

    void parse() {
        Cursor c(base, len);
        const uint32_t magic = c.read<uint32_t>();
        if (magic != 0x46554747u) {
            char buf[64];
            snprintf(buf, sizeof buf, "not a GGUF file (magic 0x%08X)", magic);
            throw ParseError{Q35K_EDATA, buf};
        }
        const uint32_t ver = c.read<uint32_t>();
        if (ver < 2 || ver > 3)
            throw ParseError{Q35K_ENOTSUP, "GGUF version " + std::to_string(ver) + " is not supported (need 2 or 3)"};
        version = (int)ver;
        const uint64_t n_tensors = c.read<uint64_t>();
        const uint64_t n_kv = c.read<uint64_t>();
        if (n_tensors > (uint64_t)INT_MAX || n_kv > (uint64_t)INT_MAX)
            throw ParseError{Q35K_EDATA, "GGUF header counts are implausibly large"};
        for (uint64_t k = 0; k < n_kv; k++) {
            std::string key = c.str();
            if (key.empty()) throw ParseError{Q35K_EDATA, "GGUF key " + std::to_string(k) + " is empty"};
            kv[key] = read_value(c);
        }
        auto al = kv.find("general.alignment");
        if (al != kv.end() && al->second.i_overflow) throw ParseError{Q35K_EDATA, "GGUF alignment is out of range"};
        if (al != kv.end() && al->second.is_int) {
            if (al->second.i < 0 || al->second.i > (int64_t)UINT32_MAX)
                throw ParseError{Q35K_EDATA, "GGUF alignment is out of range"};
            alignment = (uint32_t)al->second.i;
        }
        if (alignment == 0 || (alignment & (alignment - 1)) != 0)
            throw ParseError{Q35K_EDATA, "GGUF alignment " + std::to_string(alignment) + " is not a power of two"};
        for (uint64_t k = 0; k < n_tensors; k++) {
            Tensor t;
            t.name = c.str();
            const uint32_t nd = c.read<uint32_t>();
            if (nd == 0 || nd > 4)
                throw ParseError{Q35K_EDATA, "tensor '" + t.name + "' has invalid dim count " + std::to_string(nd)};
            t.n_dims = (int)nd;
            for (uint32_t d = 0; d < nd; d++) {
                t.dims[d] = c.read<int64_t>();
                if (t.dims[d] < 0)
                    throw ParseError{Q35K_EDATA, "tensor '" + t.name + "' dim " + std::to_string(d) + " is negative"};
            }
            t.type = c.read<int32_t>();
            t.offset = c.read<uint64_t>();
            by_name[t.name] = (int)tensors.size();
            tensors.push_back(std::move(t));
        }
        uint64_t pos = c.pos();
        if (n_tensors > 0) pos = (pos + alignment - 1) & ~(uint64_t)(alignment - 1);
        if (pos > len) throw ParseError{Q35K_EDATA, "GGUF data section starts past end of file"};
        data = pos;
    }
};

// Block bytes of the K-quant types; 0 for the rest.
static int kquant_block_bytes(int type) {
    switch (type) {
    case Q35K_TYPE_Q4_K: return Q35K_Q4K_BYTES;
    case Q35K_TYPE_Q5_K: return Q35K_Q5K_BYTES;
    case Q35K_TYPE_Q6_K: return Q35K_Q6K_BYTES;
    default: return 0;
    }
}

static const Value* find_kv(const q35k_gguf* g, const char* key) {
    if (!g || !key) return nullptr;
    auto it = g->kv.find(key);
    return it == g->kv.end() ? nullptr : &it->second;
}

extern "C" {

int q35k_gguf_open(const char* path, q35k_gguf** out) {
    if (!out) return Q35K_EINVAL;
    *out = nullptr;
    if (!path || !*path) {
        q35k::set_thread_error("GGUF path is empty");
        return Q35K_EINVAL;
    }
    q35k_gguf* g = new (std::nothrow) q35k_gguf();
    if (!g) return Q35K_ENOMEM;
    g->fd = open(path, O_RDONLY | O_CLOEXEC);
    struct stat st;
    if (g->fd < 0 || fstat(g->fd, &st) != 0) {
        q35k::set_thread_error(std::string("cannot open GGUF file '") + path + "': " + strerror(errno));
        delete g;
        return Q35K_EIO;
    }
    g->len = (uint64_t)st.st_size;
    if (g->len < 24) {
        q35k::set_thread_error("GGUF file is too small: " + std::to_string(g->len) + " bytes");
        delete g;
        return Q35K_EDATA;
    }
    void* m = mmap(nullptr, (size_t)g->len, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (m == MAP_FAILED) {
        q35k::set_thread_error(std::string("cannot map GGUF file: ") + strerror(errno));
        delete g;
        return Q35K_EIO;
    }
    g->base = static_cast<const uint8_t*>(m);
    try {
        g->parse();
    } catch (const ParseError& e) {
        q35k::set_thread_error(e.msg);
        delete g;
        return e.code;
    } catch (const std::bad_alloc&) {
        q35k::set_thread_error("out of host memory while parsing GGUF metadata");
        delete g;
        return Q35K_ENOMEM;
    }
    *out = g;
    return Q35K_OK;
}

int q35k_gguf_close(q35k_gguf* g) {
    delete g;
    return Q35K_OK;
}

int q35k_gguf_info(const q35k_gguf* g, int* version, int* n_tensors, uint32_t* alignment, uint64_t* data_offset) {
    if (!g) return Q35K_EINVAL;
    if (version) *version = g->version;
    if (n_tensors) *n_tensors = (int)g->tensors.size();
    if (alignment) *alignment = g->alignment;
    if (data_offset) *data_offset = g->data;
    return Q35K_OK;
}

int q35k_gguf_find(const q35k_gguf* g, const char* name) {
    if (!g || !name) return -1;
    auto it = g->by_name.find(name);
    return it == g->by_name.end() ? -1 : it->second;
}

int q35k_gguf_tensor(const q35k_gguf* g, int index, const char** name, int* type, int* n_dims, int64_t* dims4,
                     uint64_t* offset) {
    if (!g || index < 0 || index >= (int)g->tensors.size()) return Q35K_EINVAL;
    const Tensor& t = g->tensors[index];
    if (name) *name = t.name.c_str();
    if (type) *type = t.type;
    if (n_dims) *n_dims = t.n_dims;
    if (dims4)
        for (int d = 0; d < 4; d++) dims4[d] = d < t.n_dims ? t.dims[d] : 1;
    if (offset) *offset = t.offset;
    return Q35K_OK;
}

int q35k_gguf_tensor_data(const q35k_gguf* g, int index, size_t bytes, const void** data) {
    if (!g || !data || index < 0 || index >= (int)g->tensors.size()) return Q35K_EINVAL;
    *data = nullptr;
    const Tensor& t = g->tensors[index];
    const uint64_t room = g->len - g->data;
    if (t.offset > room || bytes > room - t.offset) {
        q35k::set_thread_error("tensor '" + t.name + "' lies past the end of the GGUF file");
        return Q35K_EDATA;
    }
    *data = g->base + g->data + t.offset;
    return Q35K_OK;
}

int q35k_gguf_get_int(const q35k_gguf* g, const char* key, int64_t* value) {
    const Value* v = find_kv(g, key);
    if (!v || !v->is_int || !value) return Q35K_EINVAL;
    *value = v->i;
    return Q35K_OK;
}

int q35k_gguf_get_float(const q35k_gguf* g, const char* key, double* value) {
    const Value* v = find_kv(g, key);
    if (!v || !value || !(v->is_float || v->is_int)) return Q35K_EINVAL;
    *value = v->is_float ? v->f : (double)v->i;
    return Q35K_OK;
}

int q35k_gguf_get_string(const q35k_gguf* g, const char* key, const char** value) {
    const Value* v = find_kv(g, key);
    if (!v || v->type != V_STRING || !value) return Q35K_EINVAL;
    *value = v->s.c_str();
    return Q35K_OK;
}

int q35k_gguf_get_array(const q35k_gguf* g, const char* key, int* elem_type, uint64_t* count) {
    const Value* v = find_kv(g, key);
    if (!v || v->type != V_ARRAY) return Q35K_EINVAL;
    if (elem_type) *elem_type = v->elem;
    if (count) *count = v->count;
    return Q35K_OK;
}

int q35k_weight_upload_gguf(q35k_ctx* ctx, const q35k_gguf* g, const char* name, q35k_weight** out) {
    if (!ctx) return Q35K_EINVAL;
    if (!g || !name || !out) return ctx->fail(Q35K_EINVAL, "NULL argument");
    *out = nullptr;
    const int i = q35k_gguf_find(g, name);
    if (i < 0) return ctx->fail(Q35K_EINVAL, "GGUF has no tensor '%s'", name);
    const Tensor& t = g->tensors[i];
    const int bb = kquant_block_bytes(t.type);
    if (bb == 0)
        return ctx->fail(Q35K_ENOTSUP, "tensor '%s' has type %d, not Q4_K, Q5_K or Q6_K", t.name.c_str(), t.type);
    // GGUF dim 0 is the row length (LoadWeights, Qwen35Model.cs:477-481).
    const int64_t n_in = t.dims[0];
    const int64_t n_out = t.n_dims > 1 ? t.dims[1] : 1;
    for (int d = 2; d < t.n_dims; d++)
        if (t.dims[d] != 1)
            return ctx->fail(Q35K_ENOTSUP, "tensor '%s' is a stack of matrices (experts are not on this path)",
                             t.name.c_str());
    if (n_in <= 0 || n_in % Q35K_QK)
        return ctx->fail(Q35K_ENOTSUP, "%s: nIn=%lld is not a multiple of 256", t.name.c_str(), (long long)n_in);
    if (n_in > INT_MAX || n_out <= 0 || n_out > INT_MAX)
        return ctx->fail(Q35K_ENOTSUP, "tensor '%s' is empty or too large", t.name.c_str());
    const uint64_t bytes = (uint64_t)n_out * (uint64_t)(n_in / Q35K_QK) * (uint64_t)bb;
    const uint64_t room = g->len - g->data;
    if (t.offset > room || bytes > room - t.offset)
        return ctx->fail(Q35K_EDATA, "tensor '%s' lies past the end of the GGUF file", t.name.c_str());
    return q35k_weight_upload(ctx, t.type, g->base + g->data + t.offset, (int)n_in, (int)n_out, out);
}

}  // extern "C"
