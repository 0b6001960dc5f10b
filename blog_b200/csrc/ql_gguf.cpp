// ql_gguf.cpp -- GGUF container reader and weight upload (host side of the loader path).
//
// The reference engine loads its quantized weights through GgufFile (AI/codes/local-llm/src/
// format/gguf/GgufFile.cpp:152-250): mmap the file, parse the header, the metadata key/value
// table and the tensor table, locate each tensor's bytes, then validate the container
// (MF::validate, src/format/MF.cpp:43-84) and upload the raw blocks unchanged
// (CudaWeightPool.cpp:148-175).  This file is the same loader behind the C ABI:
//   * GGUF v2 and v3, little-endian; the magic, version and every length are checked against
//     the file size before use;
//   * tensor dims are stored innermost-first and reported outermost-first (a [rows, cols]
//     matrix is stored as {cols, rows}), as the reference does;
//   * the data section starts at the end of the tensor table rounded up to general.alignment
//     (32 when absent or zero); tensor offsets are relative to it; byte sizes follow the ggml
//     block traits (elements / block elements * block bytes, the element count a block multiple);
//   * validation rejects an empty tensor table, empty or duplicate names, empty shapes,
//     non-positive dims, unsupported types and empty data, and admits Q4_0 (the reference's
//     validator rejects it although its parser reads it: this library computes with Q4_0);
//   * ql_weight_upload copies a matrix, or the tensor-parallel shard of it (a row range, or a
//     range of whole blocks of every row), from host bytes to device memory in one pitched copy:
//     the kernels consume the raw GGUF layout, so no repack is needed.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <climits>
#include <cstdint>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/qlinear_b200.h"

namespace ql {
int set_last_error(int code, const char *msg);
}

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF"

enum ValueType : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
    kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12
};

struct Value {
    uint32_t type = kU32;
    int64_t i = 0;
    double f = 0.0;
    std::string s;
    uint32_t elem = kU32;            // arrays: element type
    std::vector<int64_t> ai;          // integer and bool arrays
    std::vector<double> af;           // float arrays
    std::vector<std::string> as;      // string arrays
};

struct Tensor {
    std::string name;
    std::vector<int64_t> shape;  // outermost first
    int32_t type = -1;
    uint64_t offset = 0;
    const uint8_t *data = nullptr;
    size_t nbytes = 0;
};

struct File {
    int fd = -1;
    size_t size = 0;
    const uint8_t *base = nullptr;
    uint32_t version = 0;
    uint32_t alignment = 32;
    std::map<std::string, Value> meta;
    std::vector<Tensor> tensors;
    std::map<std::string, int64_t> index;
    ~File() {
        if (base) munmap(const_cast<uint8_t *>(base), size);
        if (fd >= 0) ::close(fd);
    }
};

struct ParseError {
    std::string msg;
};

// ggml block traits: elements and bytes per block (0 elements: unknown type).
void block_trait(int32_t t, int64_t *elems, size_t *bytes) {
    switch (t) {
    case 0: *elems = 1; *bytes = 4; return;      // F32
    case 1: *elems = 1; *bytes = 2; return;      // F16
    case 30: *elems = 1; *bytes = 2; return;     // BF16
    case 2: *elems = 32; *bytes = 18; return;    // Q4_0
    case 3: *elems = 32; *bytes = 20; return;    // Q4_1
    case 6: *elems = 32; *bytes = 22; return;    // Q5_0
    case 7: *elems = 32; *bytes = 24; return;    // Q5_1
    case 8: *elems = 32; *bytes = 34; return;    // Q8_0
    case 9: *elems = 32; *bytes = 36; return;    // Q8_1
    case 10: *elems = 256; *bytes = 84; return;  // Q2_K
    case 11: *elems = 256; *bytes = 110; return; // Q3_K
    case 12: *elems = 256; *bytes = 144; return; // Q4_K
    case 13: *elems = 256; *bytes = 176; return; // Q5_K
    case 14: *elems = 256; *bytes = 210; return; // Q6_K
    case 15: *elems = 256; *bytes = 292; return; // Q8_K
    default: *elems = 0; *bytes = 0; return;
    }
}

// Types this library computes with (F32/F16/BF16 pass through unquantized).
bool supported(int32_t t) { return t == 0 || t == 1 || t == 30 || t == 2 || t == 6 || t == 8 || t == 12 || t == 14; }

struct Cursor {
    const uint8_t *p;
    size_t size, pos = 0;
    void need(size_t n) {
        if (n > size || pos > size - n) throw ParseError{"truncated file at byte " + std::to_string(pos)};
    }
    template <class T>
    T get() {
        need(sizeof(T));
        T v;
        memcpy(&v, p + pos, sizeof(T));
        pos += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        need(n);
        std::string s(reinterpret_cast<const char *>(p + pos), (size_t)n);
        pos += n;
        return s;
    }
    int64_t scalar_int(uint32_t t) {
        switch (t) {
        case kU8: return get<uint8_t>();
        case kI8: return get<int8_t>();
        case kU16: return get<uint16_t>();
        case kI16: return get<int16_t>();
        case kU32: return get<uint32_t>();
        case kI32: return get<int32_t>();
        case kU64: return (int64_t)get<uint64_t>();
        case kI64: return get<int64_t>();
        case kBool: return get<uint8_t>() != 0;
        default: throw ParseError{"not an integer type"};
        }
    }
    Value value(uint32_t t, int depth) {
        Value v;
        v.type = t;
        switch (t) {
        case kF32: v.f = get<float>(); v.i = (int64_t)v.f; break;
        case kF64: v.f = get<double>(); v.i = (int64_t)v.f; break;
        case kString: v.s = str(); break;
        case kArray: {
            if (depth > 0) throw ParseError{"nested metadata arrays are not supported"};
            v.elem = get<uint32_t>();
            const uint64_t n = get<uint64_t>();
            if (n > size) throw ParseError{"metadata array length exceeds the file"};
            for (uint64_t k = 0; k < n; ++k) {
                if (v.elem == kString) v.as.push_back(str());
                else if (v.elem == kF32) v.af.push_back(get<float>());
                else if (v.elem == kF64) v.af.push_back(get<double>());
                else if (v.elem <= kI64 && v.elem != kArray) v.ai.push_back(scalar_int(v.elem));
                else throw ParseError{"bad metadata array element type " + std::to_string(v.elem)};
            }
            break;
        }
        default:
            if (t > kF64) throw ParseError{"bad metadata value type " + std::to_string(t)};
            v.i = scalar_int(t);
            v.f = (double)v.i;
        }
        return v;
    }
};

File *parse(const char *path) {
    File *f = new File();
    try {
        f->fd = ::open(path, O_RDONLY);
        if (f->fd < 0) throw ParseError{std::string("cannot open ") + path + ": " + strerror(errno)};
        struct stat st {};
        if (fstat(f->fd, &st) != 0) throw ParseError{std::string("cannot stat ") + path};
        f->size = (size_t)st.st_size;
        if (f->size < 24) throw ParseError{"file too small for a GGUF header"};
        void *m = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
        if (m == MAP_FAILED) throw ParseError{std::string("mmap failed: ") + strerror(errno)};
        f->base = static_cast<const uint8_t *>(m);
        Cursor c{f->base, f->size};
        if (c.get<uint32_t>() != kMagic) throw ParseError{"not a GGUF file (bad magic)"};
        f->version = c.get<uint32_t>();
        if (f->version != 2 && f->version != 3)
            throw ParseError{"unsupported GGUF version " + std::to_string(f->version)};
        const uint64_t ntensors = c.get<uint64_t>(), nkv = c.get<uint64_t>();
        if (ntensors > f->size || nkv > f->size) throw ParseError{"table counts exceed the file"};
        for (uint64_t k = 0; k < nkv; ++k) {
            std::string key = c.str();
            const uint32_t t = c.get<uint32_t>();
            f->meta[key] = c.value(t, 0);
        }
        auto al = f->meta.find("general.alignment");
        if (al != f->meta.end() && al->second.type != kString && al->second.type != kArray && al->second.i > 0)
            f->alignment = (uint32_t)al->second.i;
        for (uint64_t k = 0; k < ntensors; ++k) {
            Tensor t;
            t.name = c.str();
            const uint32_t nd = c.get<uint32_t>();
            if (nd > 8) throw ParseError{"tensor " + t.name + ": too many dims"};
            std::vector<int64_t> dims(nd);
            for (uint32_t d = 0; d < nd; ++d) dims[d] = (int64_t)c.get<uint64_t>();
            t.type = (int32_t)c.get<uint32_t>();
            t.offset = c.get<uint64_t>();
            t.shape.assign(dims.rbegin(), dims.rend());
            int64_t be;
            size_t bb;
            block_trait(t.type, &be, &bb);
            if (be == 0) throw ParseError{"tensor " + t.name + ": unknown ggml type " + std::to_string(t.type)};
            int64_t n = 1;
            for (int64_t d : dims) {
                if (d < 0 || (d > 0 && n > INT64_MAX / d)) throw ParseError{"tensor " + t.name + ": bad dims"};
                n *= d;
            }
            if (n % be) throw ParseError{"tensor " + t.name + ": element count not a multiple of the block size"};
            t.nbytes = (size_t)(n / be) * bb;
            f->tensors.push_back(std::move(t));
        }
        size_t data0 = c.pos;
        if (data0 % f->alignment) data0 += f->alignment - data0 % f->alignment;
        if (data0 > f->size) throw ParseError{"data section starts past the end of the file"};
        for (size_t k = 0; k < f->tensors.size(); ++k) {
            Tensor &t = f->tensors[k];
            if (t.offset > f->size - data0 || t.nbytes > f->size - data0 - t.offset)
                throw ParseError{"tensor " + t.name + ": data past the end of the file"};
            t.data = f->base + data0 + t.offset;
            f->index.emplace(t.name, (int64_t)k);  // the first of duplicate names wins the lookup
        }
    } catch (const ParseError &e) {
        delete f;
        ql::set_last_error(QL_EINVAL, ("ql_gguf_open: " + e.msg).c_str());
        return nullptr;
    }
    return f;
}

const Value *meta(void *file, const char *key) {
    if (!file || !key) return nullptr;
    File *f = static_cast<File *>(file);
    auto it = f->meta.find(key);
    return it == f->meta.end() ? nullptr : &it->second;
}

}  // namespace

extern "C" {

int ql_gguf_open(const char *path, void **file) {
    if (!path || !file) return ql::set_last_error(QL_EINVAL, "ql_gguf_open: null argument");
    File *f = parse(path);
    if (!f) return QL_EINVAL;
    *file = f;
    return QL_OK;
}

int ql_gguf_close(void *file) {
    delete static_cast<File *>(file);
    return QL_OK;
}

int ql_gguf_version(void *file) { return file ? (int)static_cast<File *>(file)->version : 0; }

int64_t ql_gguf_tensor_count(void *file) { return file ? (int64_t) static_cast<File *>(file)->tensors.size() : -1; }

int64_t ql_gguf_find_tensor(void *file, const char *name) {
    if (!file || !name) return -1;
    File *f = static_cast<File *>(file);
    auto it = f->index.find(name);
    return it == f->index.end() ? -1 : it->second;
}

int ql_gguf_tensor_info(void *file, int64_t i, const char **name, int32_t *quant_type, int32_t *n_dims,
                        int64_t *shape, const uint8_t **data, size_t *nbytes) {
    File *f = static_cast<File *>(file);
    if (!f || i < 0 || i >= (int64_t)f->tensors.size())
        return ql::set_last_error(QL_EINVAL, "ql_gguf_tensor_info: no such tensor");
    const Tensor &t = f->tensors[(size_t)i];
    if (name) *name = t.name.c_str();
    if (quant_type) *quant_type = t.type;
    if (n_dims) *n_dims = (int32_t)t.shape.size();
    if (shape)
        for (size_t d = 0; d < t.shape.size() && d < 8; ++d) shape[d] = t.shape[d];
    if (data) *data = t.data;
    if (nbytes) *nbytes = t.nbytes;
    return QL_OK;
}

int ql_gguf_metadata_type(void *file, const char *key) {
    const Value *v = meta(file, key);
    return v ? (int)v->type : -1;
}

int ql_gguf_metadata_int(void *file, const char *key, int64_t *out) {
    const Value *v = meta(file, key);
    if (!v || v->type == kString || v->type == kArray || !out)
        return ql::set_last_error(QL_EINVAL, "ql_gguf_metadata_int: no numeric value for this key");
    *out = v->i;
    return QL_OK;
}

int ql_gguf_metadata_float(void *file, const char *key, double *out) {
    const Value *v = meta(file, key);
    if (!v || v->type == kString || v->type == kArray || !out)
        return ql::set_last_error(QL_EINVAL, "ql_gguf_metadata_float: no numeric value for this key");
    *out = v->f;
    return QL_OK;
}

int ql_gguf_metadata_string(void *file, const char *key, const char **out) {
    const Value *v = meta(file, key);
    if (!v || v->type != kString || !out)
        return ql::set_last_error(QL_EINVAL, "ql_gguf_metadata_string: no string value for this key");
    *out = v->s.c_str();
    return QL_OK;
}

int64_t ql_gguf_metadata_array_len(void *file, const char *key) {
    const Value *v = meta(file, key);
    if (!v || v->type != kArray) return -1;
    return (int64_t)(v->elem == kString ? v->as.size() : (v->elem == kF32 || v->elem == kF64) ? v->af.size()
                                                                                             : v->ai.size());
}

int ql_gguf_metadata_array_int(void *file, const char *key, int64_t i, int64_t *out) {
    const Value *v = meta(file, key);
    if (!v || v->type != kArray || v->elem == kString || v->elem == kF32 || v->elem == kF64 || !out || i < 0 ||
        i >= (int64_t)v->ai.size())
        return ql::set_last_error(QL_EINVAL, "ql_gguf_metadata_array_int: no such integer element");
    *out = v->ai[(size_t)i];
    return QL_OK;
}

int ql_gguf_metadata_array_float(void *file, const char *key, int64_t i, double *out) {
    const Value *v = meta(file, key);
    if (!v || v->type != kArray || (v->elem != kF32 && v->elem != kF64) || !out || i < 0 ||
        i >= (int64_t)v->af.size())
        return ql::set_last_error(QL_EINVAL, "ql_gguf_metadata_array_float: no such float element");
    *out = v->af[(size_t)i];
    return QL_OK;
}

int ql_gguf_metadata_array_string(void *file, const char *key, int64_t i, const char **out) {
    const Value *v = meta(file, key);
    if (!v || v->type != kArray || v->elem != kString || !out || i < 0 || i >= (int64_t)v->as.size())
        return ql::set_last_error(QL_EINVAL, "ql_gguf_metadata_array_string: no such string element");
    *out = v->as[(size_t)i].c_str();
    return QL_OK;
}

int ql_gguf_validate(void *file) {
    File *f = static_cast<File *>(file);
    if (!f) return ql::set_last_error(QL_EINVAL, "ql_gguf_validate: null file");
    if (f->tensors.empty()) return ql::set_last_error(QL_EINVAL, "ql_gguf_validate: the file holds no tensors");
    std::set<std::string> seen;
    for (const Tensor &t : f->tensors) {
        if (t.name.empty()) return ql::set_last_error(QL_EINVAL, "ql_gguf_validate: a tensor has an empty name");
        if (!seen.insert(t.name).second)
            return ql::set_last_error(QL_EINVAL, ("ql_gguf_validate: duplicate tensor " + t.name).c_str());
        if (t.shape.empty())
            return ql::set_last_error(QL_EINVAL, ("ql_gguf_validate: empty shape: " + t.name).c_str());
        for (int64_t d : t.shape)
            if (d <= 0) return ql::set_last_error(QL_EINVAL, ("ql_gguf_validate: non-positive dim: " + t.name).c_str());
        if (!supported(t.type))
            return ql::set_last_error(QL_EINVAL, ("ql_gguf_validate: unsupported type " + std::to_string(t.type) +
                                                  " of " + t.name + " (F32/F16/BF16/Q4_0/Q4_K/Q5_0/Q6_K/Q8_0)")
                                                     .c_str());
        if (t.data == nullptr || t.nbytes == 0)
            return ql::set_last_error(QL_EINVAL, ("ql_gguf_validate: empty data: " + t.name).c_str());
    }
    return QL_OK;
}

int ql_weight_upload(const uint8_t *host, size_t row_bytes, int64_t row0, int64_t nrows, size_t byte0,
                     size_t nbytes_per_row, uint8_t *dst) {
    if (!host || !dst || row0 < 0 || nrows < 0 || byte0 > row_bytes || nbytes_per_row > row_bytes - byte0)
        return ql::set_last_error(QL_EINVAL, "ql_weight_upload: bad range");
    if (nrows == 0 || nbytes_per_row == 0) return QL_OK;
    cudaError_t e = cudaMemcpy2DAsync(dst, nbytes_per_row, host + (size_t)row0 * row_bytes + byte0, row_bytes,
                                      nbytes_per_row, (size_t)nrows, cudaMemcpyHostToDevice,
                                      static_cast<cudaStream_t>(ql_get_stream()));
    if (e != cudaSuccess) return ql::set_last_error(QL_ECUDA, cudaGetErrorString(e));
    return QL_OK;
}

}  // extern "C"
