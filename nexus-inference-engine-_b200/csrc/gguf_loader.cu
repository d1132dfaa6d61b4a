// Residency loader: GGUF v2/v3 files straight into HBM (host code only).
//
// Replaces the reference's import path, GGUFImporter::parse_gguf
// (nexus/src/import/gguf_importer.cpp:359-455) followed by mmap + wrap_pointer
// streaming at every call (compute_dispatch.cpp:142-154).  The file layout is
// the published GGUF one, read the way the reference reads it:
//   header      u32 magic "GGUF", u32 version (2 or 3), u64 tensor count,
//               u64 metadata count
//   metadata    key (u64 length + bytes), u32 value type, value; arrays are
//               u32 element type + u64 count + elements (skipped, as the
//               reference does, keeping their type and length)
//   tensor index name, u32 n_dims, u64 dims[n_dims] (dims[0] fastest),
//               u32 ggml type, u64 offset from the data section
//   data        starts at the next multiple of general.alignment (default 32;
//               0 also means 32) after the index
// Differences, all on the side of refusing bad input: every read is checked
// against the file size, n_dims is at most 4, and each tensor's bytes must lie
// inside the file; a violation is NXQ_ERR_FORMAT with the position.  The file
// is mapped read-only once; registration hands the mapped blocks to
// nxq_weight_register, which builds the tiled HBM copy.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "nxq_internal.h"

namespace nxq {
namespace {

constexpr uint32_t kGgufMagic = 0x46554747u;  // "GGUF" read as a little-endian u32
constexpr uint32_t kGgufHandleMagic = 0x4E584746u;
constexpr int kMaxDims = 4;
constexpr int kMaxArrayDepth = 8;

// Elements per block and bytes per block of the ggml tensor types whose size a
// loader must know to bound-check the data section (published ggml layouts).
bool type_geometry(uint32_t t, uint64_t* qk, uint64_t* bb) {
    static const struct { uint32_t t, qk, bb; } kTab[] = {
        {0, 1, 4},      {1, 1, 2},      {2, 32, 18},    {3, 32, 20},    {6, 32, 22},
        {7, 32, 24},    {8, 32, 34},    {9, 32, 36},    {10, 256, 84},  {11, 256, 110},
        {12, 256, 144}, {13, 256, 176}, {14, 256, 210}, {15, 256, 292}, {24, 1, 1},
        {25, 1, 2},     {26, 1, 4},     {27, 1, 8},     {28, 1, 8},     {30, 1, 2},
    };
    for (const auto& e : kTab)
        if (e.t == t) {
            *qk = e.qk;
            *bb = e.bb;
            return true;
        }
    return false;
}

struct MetaKV {
    std::string key;
    uint32_t type = 0;
    uint64_t u = 0;        // unsigned integers and bool
    int64_t i = 0;         // signed integers
    double f = 0.0;        // floats
    std::string s;         // strings
    uint32_t arr_type = 0; // arrays: element type and length
    uint64_t arr_count = 0;
};

struct TensorInfo {
    std::string name;
    int n_dims = 0;
    int64_t dims[kMaxDims] = {1, 1, 1, 1};
    uint32_t type = 0;
    uint64_t offset = 0;
    uint64_t bytes = 0;  // 0: type unknown to the loader
};

// Bounds-checked cursor over the mapped file.
struct Cursor {
    const uint8_t* base;
    uint64_t size;
    uint64_t pos = 0;
    bool take(void* dst, uint64_t n) {
        if (n > size - pos) return false;
        std::memcpy(dst, base + pos, n);
        pos += n;
        return true;
    }
    bool skip(uint64_t n) {
        if (n > size - pos) return false;
        pos += n;
        return true;
    }
    bool str(std::string* s) {
        uint64_t n = 0;
        if (!take(&n, 8) || n > size - pos) return false;
        if (s) s->assign(reinterpret_cast<const char*>(base + pos), n);
        pos += n;
        return true;
    }
};

uint64_t scalar_bytes(uint32_t t) {
    switch (t) {
        case NXQ_GGUF_U8: case NXQ_GGUF_I8: case NXQ_GGUF_BOOL: return 1;
        case NXQ_GGUF_U16: case NXQ_GGUF_I16: return 2;
        case NXQ_GGUF_U32: case NXQ_GGUF_I32: case NXQ_GGUF_F32: return 4;
        case NXQ_GGUF_U64: case NXQ_GGUF_I64: case NXQ_GGUF_F64: return 8;
        default: return 0;
    }
}

// Skips one value of type t (arrays recursively, bounded depth).
bool skip_value(Cursor& c, uint32_t t, int depth) {
    if (const uint64_t n = scalar_bytes(t)) return c.skip(n);
    if (t == NXQ_GGUF_STRING) return c.str(nullptr);
    if (t != NXQ_GGUF_ARRAY || depth >= kMaxArrayDepth) return false;
    uint32_t et = 0;
    uint64_t count = 0;
    if (!c.take(&et, 4) || !c.take(&count, 8)) return false;
    if (const uint64_t n = scalar_bytes(et)) return count <= (c.size - c.pos) / n && c.skip(count * n);
    for (uint64_t k = 0; k < count; ++k)
        if (!skip_value(c, et, depth + 1)) return false;
    return true;
}

bool read_value(Cursor& c, MetaKV& kv) {
    if (!c.take(&kv.type, 4)) return false;
    uint8_t b1;
    uint16_t b2;
    uint32_t b4;
    uint64_t b8;
    switch (kv.type) {
        case NXQ_GGUF_U8: if (!c.take(&b1, 1)) return false; kv.u = b1; kv.i = b1; return true;
        case NXQ_GGUF_I8: if (!c.take(&b1, 1)) return false; kv.i = (int8_t)b1; kv.u = (uint64_t)kv.i; return true;
        case NXQ_GGUF_U16: if (!c.take(&b2, 2)) return false; kv.u = b2; kv.i = b2; return true;
        case NXQ_GGUF_I16: if (!c.take(&b2, 2)) return false; kv.i = (int16_t)b2; kv.u = (uint64_t)kv.i; return true;
        case NXQ_GGUF_U32: if (!c.take(&b4, 4)) return false; kv.u = b4; kv.i = b4; return true;
        case NXQ_GGUF_I32: if (!c.take(&b4, 4)) return false; kv.i = (int32_t)b4; kv.u = (uint64_t)kv.i; return true;
        case NXQ_GGUF_U64: if (!c.take(&b8, 8)) return false; kv.u = b8; kv.i = (int64_t)b8; return true;
        case NXQ_GGUF_I64: if (!c.take(&b8, 8)) return false; kv.i = (int64_t)b8; kv.u = b8; return true;
        case NXQ_GGUF_BOOL: if (!c.take(&b1, 1)) return false; kv.u = b1 != 0; kv.i = b1 != 0; return true;
        case NXQ_GGUF_F32: {
            float f;
            if (!c.take(&f, 4)) return false;
            kv.f = f;
            return true;
        }
        case NXQ_GGUF_F64: return c.take(&kv.f, 8);
        case NXQ_GGUF_STRING: return c.str(&kv.s);
        case NXQ_GGUF_ARRAY: {
            const uint64_t at = c.pos;
            if (!c.take(&kv.arr_type, 4) || !c.take(&kv.arr_count, 8)) return false;
            c.pos = at;
            return skip_value(c, NXQ_GGUF_ARRAY, 0);
        }
        default: return false;
    }
}

}  // namespace

struct GgufFile {
    uint32_t magic = kGgufHandleMagic;
    int fd = -1;
    void* map = nullptr;
    uint64_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32;
    uint64_t data_start = 0;
    std::vector<MetaKV> meta;
    std::vector<TensorInfo> tensors;
    std::unordered_map<std::string, int64_t> tensor_by_name, meta_by_key;

    ~GgufFile() {
        magic = 0;
        if (map && map != MAP_FAILED) munmap(map, size);
        if (fd >= 0) close(fd);
    }
    const uint8_t* bytes() const { return static_cast<const uint8_t*>(map); }
};

namespace {

int parse(GgufFile& g) {
    Cursor c{g.bytes(), g.size};
    uint32_t magic = 0, version = 0;
    uint64_t n_tensors = 0, n_meta = 0;
    if (!c.take(&magic, 4) || !c.take(&version, 4) || !c.take(&n_tensors, 8) || !c.take(&n_meta, 8))
        return fail(NXQ_ERR_FORMAT, "gguf: file of %llu bytes is shorter than the header", (unsigned long long)g.size);
    if (magic != kGgufMagic) return fail(NXQ_ERR_FORMAT, "gguf: bad magic 0x%08X", magic);
    if (version < 2 || version > 3) return fail(NXQ_ERR_FORMAT, "gguf: unsupported version %u (2 or 3)", version);
    g.version = version;
    // Every key/value and every index entry takes at least 12 bytes, which
    // bounds the counts before anything is reserved.
    if (n_meta > g.size / 12 || n_tensors > g.size / 12)
        return fail(NXQ_ERR_FORMAT, "gguf: counts (%llu tensors, %llu keys) exceed the file size",
                    (unsigned long long)n_tensors, (unsigned long long)n_meta);
    g.meta.reserve(n_meta);
    for (uint64_t k = 0; k < n_meta; ++k) {
        MetaKV kv;
        const uint64_t at = c.pos;
        if (!c.str(&kv.key) || !read_value(c, kv))
            return fail(NXQ_ERR_FORMAT, "gguf: metadata entry %llu at byte %llu is malformed or truncated",
                        (unsigned long long)k, (unsigned long long)at);
        if (kv.key == "general.alignment") {
            if (kv.type == NXQ_GGUF_ARRAY || kv.type == NXQ_GGUF_STRING || kv.type == NXQ_GGUF_F32 ||
                kv.type == NXQ_GGUF_F64)
                return fail(NXQ_ERR_FORMAT, "gguf: general.alignment is not an integer");
            g.alignment = kv.u == 0 ? 32 : kv.u;
            if (g.alignment > (1u << 30)) return fail(NXQ_ERR_FORMAT, "gguf: alignment %llu", (unsigned long long)kv.u);
        }
        g.meta_by_key.emplace(kv.key, (int64_t)g.meta.size());
        g.meta.push_back(std::move(kv));
    }
    g.tensors.reserve(n_tensors);
    for (uint64_t k = 0; k < n_tensors; ++k) {
        TensorInfo t;
        uint32_t nd = 0;
        const uint64_t at = c.pos;
        if (!c.str(&t.name) || !c.take(&nd, 4))
            return fail(NXQ_ERR_FORMAT, "gguf: tensor entry %llu at byte %llu is truncated", (unsigned long long)k,
                        (unsigned long long)at);
        if (nd < 1 || nd > kMaxDims)
            return fail(NXQ_ERR_FORMAT, "gguf: tensor '%s' has %u dimensions (1..%d)", t.name.c_str(), nd, kMaxDims);
        t.n_dims = (int)nd;
        uint64_t elems = 1;
        for (uint32_t d = 0; d < nd; ++d) {
            uint64_t v = 0;
            if (!c.take(&v, 8)) return fail(NXQ_ERR_FORMAT, "gguf: tensor '%s' is truncated", t.name.c_str());
            if (v == 0 || v > (1ull << 40) || elems > (1ull << 50) / v)
                return fail(NXQ_ERR_FORMAT, "gguf: tensor '%s' dimension %u = %llu", t.name.c_str(), d,
                            (unsigned long long)v);
            t.dims[d] = (int64_t)v;
            elems *= v;
        }
        if (!c.take(&t.type, 4) || !c.take(&t.offset, 8))
            return fail(NXQ_ERR_FORMAT, "gguf: tensor '%s' is truncated", t.name.c_str());
        uint64_t qk = 0, bb = 0;
        if (type_geometry(t.type, &qk, &bb)) t.bytes = (elems + qk - 1) / qk * bb;
        if (!g.tensor_by_name.emplace(t.name, (int64_t)g.tensors.size()).second)
            return fail(NXQ_ERR_FORMAT, "gguf: tensor name '%s' appears twice", t.name.c_str());
        g.tensors.push_back(std::move(t));
    }
    g.data_start = (c.pos + g.alignment - 1) / g.alignment * g.alignment;
    for (const TensorInfo& t : g.tensors) {
        if (g.data_start > g.size || t.offset > g.size - g.data_start || t.bytes > g.size - g.data_start - t.offset)
            return fail(NXQ_ERR_FORMAT, "gguf: tensor '%s' (%llu bytes at data offset %llu) runs past the end of the file",
                        t.name.c_str(), (unsigned long long)t.bytes, (unsigned long long)t.offset);
    }
    return NXQ_OK;
}

GgufFile* handle(nxq_gguf_t h) {
    GgufFile* g = reinterpret_cast<GgufFile*>(h);
    return (g && g->magic == kGgufHandleMagic) ? g : nullptr;
}

const MetaKV* meta_of(GgufFile* g, const char* key) {
    if (!key) return nullptr;
    auto it = g->meta_by_key.find(key);
    return it == g->meta_by_key.end() ? nullptr : &g->meta[it->second];
}

// Host blocks, N and K of tensor i as a weight (expert `slice` of a 3-D tensor).
int weight_view(GgufFile* g, int64_t i, int64_t slice, const uint8_t** data, size_t* bytes, int64_t* N,
                int64_t* K) {
    if (i < 0 || i >= (int64_t)g->tensors.size()) return fail(NXQ_ERR_ARG, "gguf: tensor index %lld", (long long)i);
    const TensorInfo& t = g->tensors[i];
    Geometry geo;
    if (!geometry_of((int)t.type, &geo))
        return fail(NXQ_ERR_CODEC, "gguf: tensor '%s' has type %u, not a block type nxq registers", t.name.c_str(), t.type);
    const int64_t E = t.dims[2] * t.dims[3];
    if (t.dims[3] != 1 || slice < 0 || slice >= E)
        return fail(NXQ_ERR_SHAPE, "gguf: tensor '%s' (%d dims) has no slice %lld", t.name.c_str(), t.n_dims,
                    (long long)slice);
    *K = t.dims[0];
    *N = t.dims[1];
    if (*K % geo.qk) return fail(NXQ_ERR_SHAPE, "gguf: tensor '%s' rows of %lld are not whole blocks", t.name.c_str(), (long long)*K);
    const uint64_t per = (uint64_t)*N * (uint64_t)(*K / geo.qk) * (uint64_t)geo.bb;
    *bytes = per;
    *data = g->bytes() + g->data_start + t.offset + per * (uint64_t)slice;
    return NXQ_OK;
}

void copy_str(const std::string& s, char* buf, size_t n) {
    if (!buf || n == 0) return;
    const size_t k = s.size() < n - 1 ? s.size() : n - 1;
    std::memcpy(buf, s.data(), k);
    buf[k] = '\0';
}

}  // namespace
}  // namespace nxq

using nxq::GgufFile;
using nxq::fail;

extern "C" {

NXQ_API int nxq_gguf_open(const char* path, nxq_gguf_t* out) {
    if (!path || !out) return fail(NXQ_ERR_ARG, "gguf_open: null argument");
    *out = nullptr;
    auto* g = new (std::nothrow) GgufFile();
    if (!g) return fail(NXQ_ERR_NOMEM, "gguf_open: out of host memory");
    g->fd = open(path, O_RDONLY | O_CLOEXEC);
    if (g->fd < 0) {
        delete g;
        return fail(NXQ_ERR_ARG, "gguf_open: cannot open '%s' (%s)", path, strerror(errno));
    }
    struct stat st;
    if (fstat(g->fd, &st) != 0 || st.st_size <= 0) {
        delete g;
        return fail(NXQ_ERR_FORMAT, "gguf_open: '%s' is empty or unreadable", path);
    }
    g->size = (uint64_t)st.st_size;
    g->map = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (g->map == MAP_FAILED) {
        g->map = nullptr;
        delete g;
        return fail(NXQ_ERR_NOMEM, "gguf_open: mmap of '%s' failed (%s)", path, strerror(errno));
    }
    int rc;
    try {
        rc = nxq::parse(*g);
    } catch (const std::bad_alloc&) {
        rc = fail(NXQ_ERR_NOMEM, "gguf_open: out of host memory while indexing '%s'", path);
    }
    if (rc != NXQ_OK) {
        delete g;
        return rc;
    }
    *out = reinterpret_cast<nxq_gguf_t>(g);
    return NXQ_OK;
}

NXQ_API int nxq_gguf_close(nxq_gguf_t h) {
    GgufFile* g = nxq::handle(h);
    if (!g) return fail(NXQ_ERR_ARG, "gguf_close: not an open file handle");
    delete g;
    return NXQ_OK;
}

NXQ_API int nxq_gguf_header(nxq_gguf_t h, uint32_t* version, uint64_t* alignment, uint64_t* data_start) {
    GgufFile* g = nxq::handle(h);
    if (!g) return fail(NXQ_ERR_ARG, "gguf_header: not an open file handle");
    if (version) *version = g->version;
    if (alignment) *alignment = g->alignment;
    if (data_start) *data_start = g->data_start;
    return NXQ_OK;
}

NXQ_API int nxq_gguf_tensor_count(nxq_gguf_t h, int64_t* n) {
    GgufFile* g = nxq::handle(h);
    if (!g || !n) return fail(NXQ_ERR_ARG, "gguf_tensor_count: bad argument");
    *n = (int64_t)g->tensors.size();
    return NXQ_OK;
}

NXQ_API int nxq_gguf_tensor_info(nxq_gguf_t h, int64_t i, char* name, size_t name_len, int* type, int* n_dims,
                                 int64_t dims[4], uint64_t* offset, uint64_t* bytes) {
    GgufFile* g = nxq::handle(h);
    if (!g) return fail(NXQ_ERR_ARG, "gguf_tensor_info: not an open file handle");
    if (i < 0 || i >= (int64_t)g->tensors.size()) return fail(NXQ_ERR_ARG, "gguf_tensor_info: index %lld", (long long)i);
    const nxq::TensorInfo& t = g->tensors[i];
    nxq::copy_str(t.name, name, name_len);
    if (type) *type = (int)t.type;
    if (n_dims) *n_dims = t.n_dims;
    if (dims)
        for (int d = 0; d < 4; ++d) dims[d] = t.dims[d];
    if (offset) *offset = t.offset;
    if (bytes) *bytes = t.bytes;
    return NXQ_OK;
}

NXQ_API int nxq_gguf_find(nxq_gguf_t h, const char* name, int64_t* index) {
    GgufFile* g = nxq::handle(h);
    if (!g || !name || !index) return fail(NXQ_ERR_ARG, "gguf_find: bad argument");
    auto it = g->tensor_by_name.find(name);
    if (it == g->tensor_by_name.end()) return fail(NXQ_ERR_ARG, "gguf_find: no tensor '%s'", name);
    *index = it->second;
    return NXQ_OK;
}

NXQ_API int nxq_gguf_tensor_data(nxq_gguf_t h, int64_t i, const void** data, uint64_t* bytes) {
    GgufFile* g = nxq::handle(h);
    if (!g || !data) return fail(NXQ_ERR_ARG, "gguf_tensor_data: bad argument");
    if (i < 0 || i >= (int64_t)g->tensors.size()) return fail(NXQ_ERR_ARG, "gguf_tensor_data: index %lld", (long long)i);
    const nxq::TensorInfo& t = g->tensors[i];
    *data = g->bytes() + g->data_start + t.offset;
    if (bytes) *bytes = t.bytes;
    return NXQ_OK;
}

NXQ_API int nxq_gguf_meta_count(nxq_gguf_t h, int64_t* n) {
    GgufFile* g = nxq::handle(h);
    if (!g || !n) return fail(NXQ_ERR_ARG, "gguf_meta_count: bad argument");
    *n = (int64_t)g->meta.size();
    return NXQ_OK;
}

NXQ_API int nxq_gguf_meta_key(nxq_gguf_t h, int64_t i, char* key, size_t n, int* value_type) {
    GgufFile* g = nxq::handle(h);
    if (!g) return fail(NXQ_ERR_ARG, "gguf_meta_key: not an open file handle");
    if (i < 0 || i >= (int64_t)g->meta.size()) return fail(NXQ_ERR_ARG, "gguf_meta_key: index %lld", (long long)i);
    nxq::copy_str(g->meta[i].key, key, n);
    if (value_type) *value_type = (int)g->meta[i].type;
    return NXQ_OK;
}

static int meta_number(nxq_gguf_t h, const char* key, const char* fn, const nxq::MetaKV** out, bool want_float) {
    GgufFile* g = nxq::handle(h);
    if (!g) return fail(NXQ_ERR_ARG, "%s: not an open file handle", fn);
    const nxq::MetaKV* kv = nxq::meta_of(g, key);
    if (!kv) return fail(NXQ_ERR_ARG, "%s: no key '%s'", fn, key ? key : "(null)");
    const bool is_float = kv->type == NXQ_GGUF_F32 || kv->type == NXQ_GGUF_F64;
    if (kv->type == NXQ_GGUF_STRING || kv->type == NXQ_GGUF_ARRAY || is_float != want_float)
        return fail(NXQ_ERR_ARG, "%s: key '%s' holds value type %u", fn, key, kv->type);
    *out = kv;
    return NXQ_OK;
}

NXQ_API int nxq_gguf_meta_uint(nxq_gguf_t h, const char* key, uint64_t* v) {
    const nxq::MetaKV* kv;
    if (!v) return fail(NXQ_ERR_ARG, "gguf_meta_uint: null output");
    if (int rc = meta_number(h, key, "gguf_meta_uint", &kv, false)) return rc;
    if ((kv->type == NXQ_GGUF_I8 || kv->type == NXQ_GGUF_I16 || kv->type == NXQ_GGUF_I32 || kv->type == NXQ_GGUF_I64) &&
        kv->i < 0)
        return fail(NXQ_ERR_ARG, "gguf_meta_uint: key '%s' is negative", key);
    *v = kv->u;
    return NXQ_OK;
}

NXQ_API int nxq_gguf_meta_int(nxq_gguf_t h, const char* key, int64_t* v) {
    const nxq::MetaKV* kv;
    if (!v) return fail(NXQ_ERR_ARG, "gguf_meta_int: null output");
    if (int rc = meta_number(h, key, "gguf_meta_int", &kv, false)) return rc;
    if (kv->type == NXQ_GGUF_U64 && kv->u > (uint64_t)INT64_MAX)
        return fail(NXQ_ERR_ARG, "gguf_meta_int: key '%s' does not fit int64", key);
    *v = kv->i;
    return NXQ_OK;
}

NXQ_API int nxq_gguf_meta_float(nxq_gguf_t h, const char* key, double* v) {
    const nxq::MetaKV* kv;
    if (!v) return fail(NXQ_ERR_ARG, "gguf_meta_float: null output");
    if (int rc = meta_number(h, key, "gguf_meta_float", &kv, true)) return rc;
    *v = kv->f;
    return NXQ_OK;
}

NXQ_API int nxq_gguf_meta_string(nxq_gguf_t h, const char* key, char* buf, size_t n) {
    GgufFile* g = nxq::handle(h);
    if (!g || !buf || n == 0) return fail(NXQ_ERR_ARG, "gguf_meta_string: bad argument");
    const nxq::MetaKV* kv = nxq::meta_of(g, key);
    if (!kv || kv->type != NXQ_GGUF_STRING)
        return fail(NXQ_ERR_ARG, "gguf_meta_string: no string key '%s'", key ? key : "(null)");
    nxq::copy_str(kv->s, buf, n);
    return NXQ_OK;
}

NXQ_API int nxq_gguf_meta_array(nxq_gguf_t h, const char* key, int* elem_type, uint64_t* count) {
    GgufFile* g = nxq::handle(h);
    if (!g) return fail(NXQ_ERR_ARG, "gguf_meta_array: not an open file handle");
    const nxq::MetaKV* kv = nxq::meta_of(g, key);
    if (!kv || kv->type != NXQ_GGUF_ARRAY)
        return fail(NXQ_ERR_ARG, "gguf_meta_array: no array key '%s'", key ? key : "(null)");
    if (elem_type) *elem_type = (int)kv->arr_type;
    if (count) *count = kv->arr_count;
    return NXQ_OK;
}

NXQ_API int nxq_gguf_register(nxq_gguf_t h, int64_t i, int64_t slice, nxq_weight_t* out) {
    GgufFile* g = nxq::handle(h);
    if (!g || !out) return fail(NXQ_ERR_ARG, "gguf_register: bad argument");
    const uint8_t* data;
    size_t bytes;
    int64_t N, K;
    if (int rc = nxq::weight_view(g, i, slice, &data, &bytes, &N, &K)) return rc;
    return nxq_weight_register(data, bytes, (int)g->tensors[i].type, N, K, out);
}

NXQ_API int nxq_gguf_register_shard(nxq_gguf_t h, int64_t i, int64_t slice, int split, int rank, int world,
                                    nxq_weight_t* out) {
    GgufFile* g = nxq::handle(h);
    if (!g || !out) return fail(NXQ_ERR_ARG, "gguf_register_shard: bad argument");
    const uint8_t* data;
    size_t bytes;
    int64_t N, K;
    if (int rc = nxq::weight_view(g, i, slice, &data, &bytes, &N, &K)) return rc;
    return nxq_weight_register_shard(data, bytes, (int)g->tensors[i].type, N, K, split, rank, world, out);
}

}  // extern "C"
