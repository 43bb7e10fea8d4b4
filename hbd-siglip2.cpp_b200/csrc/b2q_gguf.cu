// b2q_gguf.cu — GGUF reader and tower loaders (host code).
//
// Counterpart of GGUFLoader + load_tensor_data_from_file
// (src/gguf_loader.cpp:205-337): the file is mapped read-only, the header,
// key/value section and tensor table are parsed (GGUF v2/v3 layout:
// magic "GGUF", version, tensor count, kv count, kvs, tensor infos, data
// aligned to general.alignment, default 32), and each tower tensor is handed
// to b2q_vision_set_tensor / b2q_text_set_tensor by its GGUF name.
//
// Type policy (the converter's, scripts/convert_siglip2_to_gguf.py:210-265):
// biases, LayerNorm parameters, position tables, the probe and the logit
// scalars are F32; every other ".weight" is a projection (or the text token
// table).  Projections stored Q8_0 are used as they are (ffn_down already
// K-padded 4304 -> 4320 by tools/siglip2-quantize/main.cpp:174-186);
// projections stored F16, BF16 or F32 are quantized to Q8_0 here with the
// ggml/gguf-py rule, K zero-padded to a multiple of 32 (the reference does
// the F16 -> Q8_0 step at load time too, gguf_loader.cpp:297-318).  Small
// tensors stored F16/BF16 are widened to F32.
#include "b2q_internal.h"

#include <cuda_fp16.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

using namespace b2q;

namespace {

enum : uint32_t {
    GGUF_U8 = 0, GGUF_I8 = 1, GGUF_U16 = 2, GGUF_I16 = 3, GGUF_U32 = 4, GGUF_I32 = 5, GGUF_F32 = 6,
    GGUF_BOOL = 7, GGUF_STRING = 8, GGUF_ARRAY = 9, GGUF_U64 = 10, GGUF_I64 = 11, GGUF_F64 = 12
};
enum : int32_t { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_BF16 = 30 };

struct TensorInfo {
    std::string name;
    int32_t type = 0;
    int32_t n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0;
    const uint8_t* data = nullptr;
    size_t nbytes = 0;
};

// bounds-checked little-endian cursor over the mapped file
struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;
    template <class T>
    T get() {
        T v{};
        if (static_cast<size_t>(end - p) < sizeof(T)) {
            ok = false;
            return v;
        }
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || static_cast<uint64_t>(end - p) < n) {
            ok = false;
            return {};
        }
        std::string s(reinterpret_cast<const char*>(p), n);
        p += n;
        return s;
    }
    void skip(uint64_t n) {
        if (static_cast<uint64_t>(end - p) < n) ok = false;
        else p += n;
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case GGUF_U8: case GGUF_I8: case GGUF_BOOL: return 1;
        case GGUF_U16: case GGUF_I16: return 2;
        case GGUF_U32: case GGUF_I32: case GGUF_F32: return 4;
        case GGUF_U64: case GGUF_I64: case GGUF_F64: return 8;
        default: return 0;
    }
}

bool skip_value(Cursor& c, uint32_t type, int depth = 0) {
    if (type == GGUF_STRING) {
        c.str();
        return c.ok;
    }
    if (type == GGUF_ARRAY) {
        if (depth > 2) return false;
        const uint32_t et = c.get<uint32_t>();
        const uint64_t n = c.get<uint64_t>();
        if (!c.ok) return false;
        const size_t es = scalar_size(et);
        if (es) {
            if (n > UINT64_MAX / es) return false;
            c.skip(n * es);
            return c.ok;
        }
        for (uint64_t i = 0; i < n && c.ok; ++i)
            if (!skip_value(c, et, depth + 1)) return false;
        return c.ok;
    }
    const size_t s = scalar_size(type);
    if (!s) return false;
    c.skip(s);
    return c.ok;
}

float f16_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }
float bf16_to_f32(uint16_t h) {
    const uint32_t u = static_cast<uint32_t>(h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// Q8_0 rule of ggml / gguf-py (gguf/quants.py:381-394): d = max|x|/127,
// q = round-half-away(x * (1/d)), d stored as fp16.  rows x K fp32 -> rows x Kp/32 blocks.
void quantize_q8_0_rows(const float* x, int64_t rows, int64_t K, int64_t Kp, uint8_t* out) {
    const int64_t Kb = Kp / 32;
    for (int64_t n = 0; n < rows; ++n) {
        for (int64_t kb = 0; kb < Kb; ++kb) {
            float v[32];
            for (int j = 0; j < 32; ++j) {
                const int64_t k = kb * 32 + j;
                v[j] = k < K ? x[n * K + k] : 0.0f;
            }
            float amax = 0.0f;
            for (int j = 0; j < 32; ++j) amax = std::fmax(amax, std::fabs(v[j]));
            const float d = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            uint8_t* blk = out + (n * Kb + kb) * 34;
            const uint16_t dh = __half_as_ushort(__float2half_rn(d));
            memcpy(blk, &dh, 2);
            for (int j = 0; j < 32; ++j) blk[2 + j] = static_cast<uint8_t>(static_cast<int8_t>(std::roundf(v[j] * id)));
        }
    }
}

bool ends_with(const std::string& s, const char* suffix) {
    const size_t n = strlen(suffix);
    return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}

// Tensors the towers use as Q8_0 (projections and the text token table).
bool is_q8_tensor(const std::string& n) {
    if (!ends_with(n, ".weight")) return false;
    if (n.find(".ln") != std::string::npos || n.find(".post_ln") != std::string::npos ||
        n.find(".final_ln") != std::string::npos)
        return false;
    return !ends_with(n, "position_embd.weight");
}

}  // namespace

struct b2q_gguf {
    void* map = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32;
    std::vector<TensorInfo> tensors;
    ~b2q_gguf() {
        if (map) munmap(map, size);
    }
    const TensorInfo* find(const char* name) const {
        for (const auto& t : tensors)
            if (t.name == name) return &t;
        return nullptr;
    }
};

namespace {

b2q_status bytes_of(const TensorInfo& t, size_t* out) {
    int64_t n = 1;
    for (int d = 0; d < t.n_dims; ++d) {
        if (t.ne[d] <= 0 || n > INT64_MAX / t.ne[d]) return set_error(B2Q_ERR_SHAPE, "GGUF: bad shape of " + t.name);
        n *= t.ne[d];
    }
    // element counts whose byte size would not fit a size_t are malformed
    const uint64_t un = static_cast<uint64_t>(n);
    switch (t.type) {
        case T_F32:
            if (un > SIZE_MAX / 4) return set_error(B2Q_ERR_SHAPE, "GGUF: tensor " + t.name + " too large");
            *out = static_cast<size_t>(un) * 4;
            return B2Q_OK;
        case T_F16: case T_BF16:
            if (un > SIZE_MAX / 2) return set_error(B2Q_ERR_SHAPE, "GGUF: tensor " + t.name + " too large");
            *out = static_cast<size_t>(un) * 2;
            return B2Q_OK;
        case T_Q8_0:
            if (t.ne[0] % 32) return set_error(B2Q_ERR_SHAPE, "GGUF: Q8_0 tensor " + t.name + " with ne0 % 32 != 0");
            if (un / 32 > SIZE_MAX / 34) return set_error(B2Q_ERR_SHAPE, "GGUF: tensor " + t.name + " too large");
            *out = static_cast<size_t>(un / 32) * 34;
            return B2Q_OK;
        default:
            *out = 0;   // other types are listed but cannot be loaded into a tower
            return B2Q_OK;
    }
}

// Hands one tower tensor to `set` (b2q_vision_set_tensor / b2q_text_set_tensor).
template <class Tower, class Set>
b2q_status load_one(Tower* tower, const TensorInfo& t, Set set, void* stream) {
    const int64_t ne0 = t.ne[0];
    int64_t rows = 1;
    for (int d = 1; d < t.n_dims; ++d) rows *= t.ne[d];
    const bool q8 = is_q8_tensor(t.name);
    if (t.type == T_Q8_0) {
        if (!q8) return set_error(B2Q_ERR_INVALID, "GGUF: " + t.name + " is Q8_0 but the tower reads it as F32");
        return set(tower, t.name.c_str(), 8, t.data, ne0, rows, stream);
    }
    if (t.type != T_F32 && t.type != T_F16 && t.type != T_BF16)
        return set_error(B2Q_ERR_INVALID, "GGUF: unsupported type " + std::to_string(t.type) + " for " + t.name);
    std::vector<float> f(static_cast<size_t>(ne0 * rows));
    for (size_t i = 0; i < f.size(); ++i) {
        if (t.type == T_F32) {
            memcpy(&f[i], t.data + 4 * i, 4);
        } else {
            uint16_t h;
            memcpy(&h, t.data + 2 * i, 2);
            f[i] = t.type == T_F16 ? f16_to_f32(h) : bf16_to_f32(h);
        }
    }
    if (!q8) return set(tower, t.name.c_str(), 0, f.data(), ne0, rows, stream);
    const int64_t Kp = (ne0 + 31) / 32 * 32;
    std::vector<uint8_t> q(static_cast<size_t>(rows * (Kp / 32) * 34));
    quantize_q8_0_rows(f.data(), rows, ne0, Kp, q.data());
    return set(tower, t.name.c_str(), 8, q.data(), Kp, rows, stream);
}

template <class Tower, class Set>
b2q_status load_prefix(Tower* tower, const b2q_gguf* g, const char* prefix, Set set, void* stream, int* count) {
    *count = 0;
    for (const auto& t : g->tensors) {
        if (t.name.rfind(prefix, 0) != 0) continue;
        const b2q_status st = load_one(tower, t, set, stream);
        if (st != B2Q_OK) return st;
        ++*count;
    }
    if (*count == 0) return set_error(B2Q_ERR_INVALID, std::string("GGUF: no tensors named ") + prefix + "*");
    return B2Q_OK;
}

}  // namespace

extern "C" {

b2q_status b2q_gguf_open(const char* path, b2q_gguf** out) {
    if (!path || !out) return set_error(B2Q_ERR_INVALID, "null pointer");
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return set_error(B2Q_ERR_INVALID, std::string("GGUF: cannot open ") + path);
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size < 24) {
        close(fd);
        return set_error(B2Q_ERR_INVALID, std::string("GGUF: not a GGUF file: ") + path);
    }
    void* m = mmap(nullptr, static_cast<size_t>(sb.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return set_error(B2Q_ERR_INVALID, std::string("GGUF: cannot map ") + path);
    b2q_gguf* g = new b2q_gguf();
    g->map = m;
    g->size = static_cast<size_t>(sb.st_size);
    Cursor c{static_cast<const uint8_t*>(m), static_cast<const uint8_t*>(m) + g->size};
    auto fail = [&](const std::string& why) {
        delete g;
        return set_error(B2Q_ERR_INVALID, "GGUF: " + why);
    };
    if (c.get<uint32_t>() != 0x46554747u) return fail("bad magic");
    g->version = c.get<uint32_t>();
    if (g->version < 2 || g->version > 3) return fail("unsupported version " + std::to_string(g->version));
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    if (!c.ok || n_tensors > (1u << 20) || n_kv > (1u << 20)) return fail("bad header");
    for (uint64_t i = 0; i < n_kv; ++i) {
        const std::string key = c.str();
        const uint32_t type = c.get<uint32_t>();
        if (!c.ok) return fail("truncated key/value section");
        if (key == "general.alignment" && type == GGUF_U32) {
            g->alignment = c.get<uint32_t>();
            if (g->alignment == 0 || (g->alignment & (g->alignment - 1))) return fail("bad general.alignment");
        } else if (!skip_value(c, type)) {
            return fail("bad value of " + key);
        }
    }
    g->tensors.resize(n_tensors);
    for (auto& t : g->tensors) {
        t.name = c.str();
        t.n_dims = static_cast<int32_t>(c.get<uint32_t>());
        if (!c.ok || t.n_dims < 1 || t.n_dims > 4) return fail("bad tensor info");
        for (int d = 0; d < t.n_dims; ++d) t.ne[d] = static_cast<int64_t>(c.get<uint64_t>());
        t.type = static_cast<int32_t>(c.get<uint32_t>());
        t.offset = c.get<uint64_t>();
        if (!c.ok) return fail("truncated tensor table");
    }
    const uint64_t hdr = static_cast<uint64_t>(c.p - static_cast<const uint8_t*>(m));
    const uint64_t data_start = (hdr + g->alignment - 1) / g->alignment * g->alignment;
    for (auto& t : g->tensors) {
        if (bytes_of(t, &t.nbytes) != B2Q_OK) {
            delete g;
            return B2Q_ERR_SHAPE;
        }
        // written so that no sum can wrap: data_start <= size, then the offset,
        // then the byte count, each against what is left
        if (data_start > g->size || t.offset > g->size - data_start || t.nbytes > g->size - data_start - t.offset)
            return fail("tensor " + t.name + " runs past the end of the file");
        t.data = static_cast<const uint8_t*>(m) + data_start + t.offset;
    }
    *out = g;
    return B2Q_OK;
}

b2q_status b2q_gguf_close(b2q_gguf* g) {
    delete g;
    return B2Q_OK;
}

int64_t b2q_gguf_n_tensors(const b2q_gguf* g) { return g ? static_cast<int64_t>(g->tensors.size()) : 0; }

b2q_status b2q_gguf_tensor(const b2q_gguf* g, int64_t i, const char** name, int32_t* ggml_type, int32_t* n_dims,
                           int64_t* ne, const void** data) {
    if (!g || i < 0 || i >= static_cast<int64_t>(g->tensors.size())) return set_error(B2Q_ERR_INVALID, "bad tensor index");
    const TensorInfo& t = g->tensors[i];
    if (name) *name = t.name.c_str();
    if (ggml_type) *ggml_type = t.type;
    if (n_dims) *n_dims = t.n_dims;
    if (ne)
        for (int d = 0; d < 4; ++d) ne[d] = t.ne[d];
    if (data) *data = t.data;
    return B2Q_OK;
}

b2q_status b2q_gguf_scalar_f32(const b2q_gguf* g, const char* name, float* out) {
    if (!g || !name || !out) return set_error(B2Q_ERR_INVALID, "null pointer");
    const TensorInfo* t = g->find(name);
    if (!t) return set_error(B2Q_ERR_INVALID, std::string("GGUF: no tensor ") + name);
    uint16_t h;
    switch (t->type) {
        case T_F32: memcpy(out, t->data, 4); return B2Q_OK;
        case T_F16: memcpy(&h, t->data, 2); *out = f16_to_f32(h); return B2Q_OK;
        case T_BF16: memcpy(&h, t->data, 2); *out = bf16_to_f32(h); return B2Q_OK;
        default: return set_error(B2Q_ERR_INVALID, std::string("GGUF: ") + name + " is not a float scalar");
    }
}

b2q_status b2q_vision_load_gguf(b2q_vision* v, const b2q_gguf* g, void* stream) {
    if (!v || !g) return set_error(B2Q_ERR_INVALID, "null pointer");
    int n = 0;
    return load_prefix(v, g, "v.", b2q_vision_set_tensor, stream, &n);
}

b2q_status b2q_text_load_gguf(b2q_text* t, const b2q_gguf* g, void* stream) {
    if (!t || !g) return set_error(B2Q_ERR_INVALID, "null pointer");
    int n = 0;
    return load_prefix(t, g, "t.", b2q_text_set_tensor, stream, &n);
}

}  // extern "C"
