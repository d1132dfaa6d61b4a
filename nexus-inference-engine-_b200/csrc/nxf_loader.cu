// Residency loader: NXF files straight into HBM (host code only).
//
// Replaces the reference's NXF read path, NXFReader::open / get_tensor /
// map_chunk (nexus/src/format/nxf_reader.cpp:166-258, 295-409; layouts in
// nexus/src/format/nxf.h:27-51), which maps chunks for the engine to stream at
// every call.  The file layout, as the reference's NXFWriter writes it
// (nxf_writer.cpp:92-330):
//   header        64 bytes at offset 0: u32 magic "NXF1", u16 version (1),
//                 u16 flags, u64 manifest offset / size, u64 tensor index
//                 offset / size, u64 data offset, u64 total file size, 8 bytes
//   chunks        each at a 16 KB boundary
//   tensor index  per tensor: u32 name length, name, u32 ndim, i64 shape[ndim]
//                 (shape[0] fastest, as GGUF dims), u8 dtype, u32 chunk count,
//                 24-byte chunk descriptors (u64 file offset, u32 stored size,
//                 u32 decoded size, u32 xxHash32 of the stored bytes, u8 codec,
//                 u8 group size, 2 bytes)
//   manifest      a flat JSON object (model metadata)
// Differences, all on the side of refusing bad input: every field and every
// chunk is checked against the file size, ndim is at most 4, and registration
// checks each chunk's xxHash32 (which the reference stores but never checks);
// a violation is NXQ_ERR_FORMAT.  Codecs registered (Codec, core/config.h:
// 21-36): INT4 - a chunk of [4-bit codes in quant/gptq.cpp's flat order][fp32
// scales][fp32 zeros], as GGUFImporter writes it (gguf_importer.cpp:1144-1170)
// -, the native passthroughs Q3K / Q4K / Q2K (GGUF blocks), and the flat
// arrays the engine decodes at load time (hybrid_model.cpp:165-255): INT8
// (w = q / 127), FP16 (subnormals read as zero) and FP32 (also any chunk of
// 4 bytes per element, the writer's passthrough), as NXQ_TYPE_NXF_I8 / F16 /
// F32.  Other codecs (BF16, GPTQ, AWQ, QuIP#, AQLM, TurboQuant) and
// entropy-coded chunks are refused with NXQ_ERR_CODEC; the reference's engine
// zero-fills the ones it does not know (hybrid_model.cpp:256-262).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "nxq_internal.h"

namespace nxq {
namespace {

constexpr uint32_t kNxfMagic = 0x3146584Eu;  // "NXF1" read as a little-endian u32
constexpr uint16_t kNxfVersion = 1;
constexpr uint32_t kNxfHandleMagic = 0x4E58464Cu;
constexpr int kMaxDims = 4;
constexpr size_t kHeaderBytes = 64;
constexpr size_t kChunkDescBytes = 24;

// Codec ids of the chunk descriptors (Codec, core/config.h:21-36).
constexpr int kCodecFp32 = 0, kCodecFp16 = 1, kCodecInt8 = 3, kCodecInt4 = 4, kCodecQ3K = 11, kCodecQ4K = 12,
              kCodecQ2K = 13;

struct Chunk {
    uint64_t offset;
    uint32_t stored, decoded, checksum;
    int codec, group;
};

struct Tensor {
    std::string name;
    int n_dims = 0;
    int64_t dims[kMaxDims] = {1, 1, 1, 1};
    int dtype = 0;
    std::vector<Chunk> chunks;
};

struct NxfFile {
    uint32_t magic = kNxfHandleMagic;
    int fd = -1;
    void* map = nullptr;
    uint64_t size = 0;
    std::string manifest;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, int64_t> by_name;
    ~NxfFile() {
        magic = 0;
        if (map) munmap(map, size);
        if (fd >= 0) close(fd);
    }
    const uint8_t* bytes() const { return static_cast<const uint8_t*>(map); }
};

NxfFile* handle(nxq_nxf_t h) {
    NxfFile* f = reinterpret_cast<NxfFile*>(h);
    return f && f->magic == kNxfHandleMagic ? f : nullptr;
}

template <typename T>
T load(const uint8_t* p) {
    T v;
    memcpy(&v, p, sizeof v);
    return v;
}

// xxHash32 with seed 0 (Yann Collet's published XXH32: four 32-bit lanes over
// 16-byte stripes, then 4-byte and 1-byte tails, then the avalanche).
uint32_t xxh32(const uint8_t* p, size_t n) {
    const uint32_t P1 = 2654435761u, P2 = 2246822519u, P3 = 3266489917u, P4 = 668265263u, P5 = 374761393u;
    auto rotl = [](uint32_t x, int r) { return (x << r) | (x >> (32 - r)); };
    const uint8_t* const end = p + n;
    uint32_t h;
    if (n >= 16) {
        uint32_t a = P1 + P2, b = P2, c = 0, d = 0u - P1;
        for (; p + 16 <= end; p += 16) {
            a = rotl(a + load<uint32_t>(p) * P2, 13) * P1;
            b = rotl(b + load<uint32_t>(p + 4) * P2, 13) * P1;
            c = rotl(c + load<uint32_t>(p + 8) * P2, 13) * P1;
            d = rotl(d + load<uint32_t>(p + 12) * P2, 13) * P1;
        }
        h = rotl(a, 1) + rotl(b, 7) + rotl(c, 12) + rotl(d, 18);
    } else {
        h = P5;
    }
    h += (uint32_t)n;
    for (; p + 4 <= end; p += 4) h = rotl(h + load<uint32_t>(p) * P3, 17) * P4;
    for (; p < end; ++p) h = rotl(h + (uint32_t)*p * P5, 11) * P1;
    h ^= h >> 15;
    h *= P2;
    h ^= h >> 13;
    h *= P3;
    h ^= h >> 16;
    return h;
}

int parse(NxfFile& f) {
    const uint8_t* b = f.bytes();
    if (f.size < kHeaderBytes) return fail(NXQ_ERR_FORMAT, "nxf: %llu bytes, shorter than the header", (unsigned long long)f.size);
    if (load<uint32_t>(b) != kNxfMagic) return fail(NXQ_ERR_FORMAT, "nxf: bad magic 0x%08x", load<uint32_t>(b));
    const uint16_t version = load<uint16_t>(b + 4);
    if (version != kNxfVersion) return fail(NXQ_ERR_FORMAT, "nxf: version %u (1 is supported)", version);
    const uint64_t man_off = load<uint64_t>(b + 8), man_size = load<uint64_t>(b + 16);
    const uint64_t idx_off = load<uint64_t>(b + 24), idx_size = load<uint64_t>(b + 32);
    const uint64_t total = load<uint64_t>(b + 48);
    if (total != f.size)
        return fail(NXQ_ERR_FORMAT, "nxf: header gives %llu bytes, the file has %llu", (unsigned long long)total,
                    (unsigned long long)f.size);
    auto inside = [&](uint64_t off, uint64_t len) { return off <= f.size && len <= f.size - off; };
    if (!inside(man_off, man_size)) return fail(NXQ_ERR_FORMAT, "nxf: manifest outside the file");
    if (!inside(idx_off, idx_size)) return fail(NXQ_ERR_FORMAT, "nxf: tensor index outside the file");
    f.manifest.assign(reinterpret_cast<const char*>(b + man_off), man_size);

    const uint8_t* p = b + idx_off;
    const uint8_t* const end = p + idx_size;
    auto need = [&](uint64_t len, const char* what) {
        if ((uint64_t)(end - p) < len) {
            fail(NXQ_ERR_FORMAT, "nxf: tensor index truncated at %s (offset %llu)", what,
                 (unsigned long long)(p - b));
            return false;
        }
        return true;
    };
    while (p < end) {
        Tensor t;
        if (!need(4, "a name length")) return NXQ_ERR_FORMAT;
        const uint32_t name_len = load<uint32_t>(p);
        p += 4;
        if (!need(name_len, "a name")) return NXQ_ERR_FORMAT;
        t.name.assign(reinterpret_cast<const char*>(p), name_len);
        p += name_len;
        if (!need(4, "ndim")) return NXQ_ERR_FORMAT;
        const uint32_t nd = load<uint32_t>(p);
        p += 4;
        if (nd > (uint32_t)kMaxDims) return fail(NXQ_ERR_FORMAT, "nxf: tensor '%s' has %u dimensions (at most 4)", t.name.c_str(), nd);
        t.n_dims = (int)nd;
        if (!need(8ull * nd, "a shape")) return NXQ_ERR_FORMAT;
        for (uint32_t d = 0; d < nd; ++d, p += 8) {
            t.dims[d] = load<int64_t>(p);
            if (t.dims[d] < 0) return fail(NXQ_ERR_FORMAT, "nxf: tensor '%s' has a negative dimension", t.name.c_str());
        }
        if (!need(5, "dtype and chunk count")) return NXQ_ERR_FORMAT;
        t.dtype = *p++;
        const uint32_t nc = load<uint32_t>(p);
        p += 4;
        if (!need((uint64_t)nc * kChunkDescBytes, "chunk descriptors")) return NXQ_ERR_FORMAT;
        t.chunks.resize(nc);
        for (uint32_t c = 0; c < nc; ++c, p += kChunkDescBytes) {
            Chunk& k = t.chunks[c];
            k.offset = load<uint64_t>(p);
            k.stored = load<uint32_t>(p + 8);
            k.decoded = load<uint32_t>(p + 12);
            k.checksum = load<uint32_t>(p + 16);
            k.codec = p[20];
            k.group = p[21];
            if (!inside(k.offset, k.stored))
                return fail(NXQ_ERR_FORMAT, "nxf: chunk %u of '%s' lies outside the file", c, t.name.c_str());
        }
        f.by_name.emplace(t.name, (int64_t)f.tensors.size());
        f.tensors.push_back(std::move(t));
    }
    return NXQ_OK;
}

void copy_str(const std::string& s, char* buf, size_t n) {
    if (!buf || n == 0) return;
    const size_t k = s.size() < n - 1 ? s.size() : n - 1;
    memcpy(buf, s.data(), k);
    buf[k] = '\0';
}

// The manifest is one flat JSON object; finds `key` and returns where its
// value starts, or null.  Strings may hold \" \\ \/ \n \t escapes.
const char* skip_ws(const char* p, const char* e) {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    return p;
}
const char* read_string(const char* p, const char* e, std::string* out) {
    if (p >= e || *p != '"') return nullptr;
    out->clear();
    for (++p; p < e && *p != '"'; ++p) {
        if (*p == '\\') {
            if (++p >= e) return nullptr;
            out->push_back(*p == 'n' ? '\n' : *p == 't' ? '\t' : *p);
        } else {
            out->push_back(*p);
        }
    }
    return p < e ? p + 1 : nullptr;
}
const char* skip_value(const char* p, const char* e) {
    if (p < e && *p == '"') {
        std::string s;
        return read_string(p, e, &s);
    }
    while (p < e && *p != ',' && *p != '}' && *p != ' ' && *p != '\n' && *p != '\r' && *p != '\t') ++p;
    return p;
}
int find_value(const NxfFile& f, const char* key, const char** value, const char** e_out) {
    const char* p = f.manifest.data();
    const char* const e = p + f.manifest.size();
    p = skip_ws(p, e);
    if (p >= e || *p != '{') return fail(NXQ_ERR_FORMAT, "nxf: the manifest is not a JSON object");
    ++p;
    std::string k;
    for (;;) {
        p = skip_ws(p, e);
        if (p < e && *p == ',') p = skip_ws(p + 1, e);
        if (p >= e) return fail(NXQ_ERR_FORMAT, "nxf: the manifest ends inside its object");
        if (*p == '}') return fail(NXQ_ERR_ARG, "nxf: no manifest key '%s'", key);
        if (!(p = read_string(p, e, &k))) return fail(NXQ_ERR_FORMAT, "nxf: bad key in the manifest");
        p = skip_ws(p, e);
        if (p >= e || *p != ':') return fail(NXQ_ERR_FORMAT, "nxf: no ':' after manifest key '%s'", k.c_str());
        p = skip_ws(p + 1, e);
        if (k == key) {
            *value = p;
            *e_out = e;
            return NXQ_OK;
        }
        if (!(p = skip_value(p, e))) return fail(NXQ_ERR_FORMAT, "nxf: bad value of manifest key '%s'", k.c_str());
    }
}

// Checks every chunk of tensor i (one codec and group size, stored = decoded
// size, xxHash32) and returns its codec and group size.
int check_chunks(const NxfFile& f, int64_t i, int* codec, int* group) {
    const Tensor& t = f.tensors[i];
    if (t.chunks.empty()) return fail(NXQ_ERR_FORMAT, "nxf: tensor '%s' has no chunks", t.name.c_str());
    for (size_t c = 0; c < t.chunks.size(); ++c) {
        const Chunk& k = t.chunks[c];
        if (k.codec != t.chunks[0].codec || k.group != t.chunks[0].group)
            return fail(NXQ_ERR_CODEC, "nxf: tensor '%s' mixes codecs or group sizes", t.name.c_str());
        if (k.stored != k.decoded)
            return fail(NXQ_ERR_CODEC, "nxf: chunk %zu of '%s' is entropy-coded (%u -> %u bytes)", c,
                        t.name.c_str(), k.stored, k.decoded);
        const uint32_t h = xxh32(f.bytes() + k.offset, k.stored);
        if (h != k.checksum)
            return fail(NXQ_ERR_FORMAT, "nxf: chunk %zu of '%s': xxHash32 0x%08x, descriptor 0x%08x", c,
                        t.name.c_str(), h, k.checksum);
    }
    *codec = t.chunks[0].codec;
    *group = t.chunks[0].group;
    return NXQ_OK;
}

// Registers slice `slice` of tensor i ([E][N][K], K = dims[0], N = dims[1]).
int register_tensor(const NxfFile& f, int64_t i, int64_t slice, bool sharded, int split, int rank, int world,
                    nxq_weight_t* out) {
    const Tensor& t = f.tensors[i];
    int codec, group;
    if (int rc = check_chunks(f, i, &codec, &group)) return rc;
    const int64_t K = t.dims[0], N = t.n_dims >= 2 ? t.dims[1] : 1;
    int64_t E = 1;
    for (int d = 2; d < t.n_dims; ++d) E *= t.dims[d];
    if (slice < 0 || slice >= E)
        return fail(NXQ_ERR_ARG, "nxf: slice %lld of '%s' (%lld slices)", (long long)slice, t.name.c_str(), (long long)E);
    if (K <= 0 || N <= 0) return fail(NXQ_ERR_SHAPE, "nxf: tensor '%s' is empty", t.name.c_str());
    const int64_t elems = E * N * K, slice_elems = N * K;
    uint64_t stored_total = 0;
    for (const Chunk& k : t.chunks) stored_total += k.stored;
    // Flat element arrays, decoded by the reference's engine at load time
    // (HybridModel::Impl::load_tensor, hybrid_model.cpp:165-255): FP32, and
    // any chunk that holds 4 bytes per element whatever its codec (the
    // writer's passthrough of small tensors, :170-176); FP16; INT8.
    if (codec == kCodecFp32 || codec == kCodecFp16 || codec == kCodecInt8 || stored_total == (uint64_t)elems * 4) {
        const bool f32 = codec == kCodecFp32 || stored_total == (uint64_t)elems * 4;
        const int type = f32 ? NXQ_TYPE_NXF_F32 : codec == kCodecFp16 ? NXQ_TYPE_NXF_F16 : NXQ_TYPE_NXF_I8;
        const int64_t bpe = f32 ? 4 : codec == kCodecFp16 ? 2 : 1;
        if (stored_total != (uint64_t)(elems * bpe))
            return fail(NXQ_ERR_SHAPE, "nxf: '%s' holds %llu bytes, its shape needs %lld", t.name.c_str(),
                        (unsigned long long)stored_total, (long long)(elems * bpe));
        if (K % 32)
            return fail(NXQ_ERR_SHAPE, "nxf: '%s': K=%lld is not a multiple of 32 (the block of the flat codecs)",
                        t.name.c_str(), (long long)K);
        std::vector<uint8_t> joined;
        const uint8_t* base = f.bytes() + t.chunks[0].offset;
        if (t.chunks.size() > 1) {
            joined.reserve(stored_total);
            for (const Chunk& k : t.chunks) joined.insert(joined.end(), f.bytes() + k.offset, f.bytes() + k.offset + k.stored);
            base = joined.data();
        }
        const size_t sb = (size_t)(slice_elems * bpe);
        const uint8_t* src = base + (size_t)slice * sb;
        return sharded ? nxq_weight_register_shard(src, sb, type, N, K, split, rank, world, out)
                       : nxq_weight_register(src, sb, type, N, K, out);
    }
    if (codec == kCodecQ3K || codec == kCodecQ4K || codec == kCodecQ2K) {
        const int type = codec == kCodecQ3K ? NXQ_TYPE_Q3_K : codec == kCodecQ4K ? NXQ_TYPE_Q4_K : NXQ_TYPE_Q2_K;
        const int64_t bb = codec == kCodecQ3K ? 110 : codec == kCodecQ4K ? 144 : 84;
        if (K % 256) return fail(NXQ_ERR_SHAPE, "nxf: '%s': K=%lld is not a multiple of 256", t.name.c_str(), (long long)K);
        uint64_t total = 0;
        for (const Chunk& k : t.chunks) total += k.stored;
        if (total != (uint64_t)(elems / 256 * bb))
            return fail(NXQ_ERR_SHAPE, "nxf: '%s' holds %llu bytes, its shape needs %lld", t.name.c_str(),
                        (unsigned long long)total, (long long)(elems / 256 * bb));
        std::vector<uint8_t> joined;
        const uint8_t* base = f.bytes() + t.chunks[0].offset;
        if (t.chunks.size() > 1) {
            joined.reserve(total);
            for (const Chunk& k : t.chunks) joined.insert(joined.end(), f.bytes() + k.offset, f.bytes() + k.offset + k.stored);
            base = joined.data();
        }
        const size_t sb = (size_t)(slice_elems / 256 * bb);
        const uint8_t* src = base + (size_t)slice * sb;
        return sharded ? nxq_weight_register_shard(src, sb, type, N, K, split, rank, world, out)
                       : nxq_weight_register(src, sb, type, N, K, out);
    }
    if (codec == kCodecInt4) {
        const int gs = group;
        if (gs != 32 && gs != 64 && gs != 128)
            return fail(NXQ_ERR_CODEC, "nxf: '%s': INT4 group size %d (32, 64, 128 are supported)", t.name.c_str(), gs);
        if (K % gs) return fail(NXQ_ERR_SHAPE, "nxf: '%s': K=%lld is not a multiple of %d", t.name.c_str(), (long long)K, gs);
        // A chunk of n elements holds n/2 code bytes and n/gs (scale, zero) pairs.
        std::vector<uint8_t> codes;
        std::vector<float> scales, zeros;
        for (size_t c = 0; c < t.chunks.size(); ++c) {
            const Chunk& k = t.chunks[c];
            const uint64_t n = (uint64_t)k.stored * 2 * gs / (gs + 16);
            if (n % gs || n / 2 + n / gs * 8 != k.stored)
                return fail(NXQ_ERR_FORMAT, "nxf: INT4 chunk %zu of '%s' has %u bytes, not whole groups of %d",
                            c, t.name.c_str(), k.stored, gs);
            const uint8_t* q = f.bytes() + k.offset;
            codes.insert(codes.end(), q, q + n / 2);
            const size_t g0 = scales.size();
            scales.resize(g0 + n / gs);
            zeros.resize(g0 + n / gs);
            memcpy(scales.data() + g0, q + n / 2, n / gs * 4);
            memcpy(zeros.data() + g0, q + n / 2 + n / gs * 4, n / gs * 4);
        }
        if ((int64_t)codes.size() * 2 != elems)
            return fail(NXQ_ERR_SHAPE, "nxf: '%s' holds %lld INT4 elements, its shape needs %lld", t.name.c_str(),
                        (long long)codes.size() * 2, (long long)elems);
        const size_t co = (size_t)(slice * slice_elems / 2), go = (size_t)(slice * slice_elems / gs);
        if (!sharded)
            return nxq_weight_register_int4(codes.data() + co, scales.data() + go, zeros.data() + go, N, K, gs,
                                            NXQ_INT4_ROWS, out);
        // A shard: the group blocks on the host, then the block shard path.
        std::vector<uint8_t> blocks((size_t)(N * (K / gs) * (8 + gs / 2)));
        if (int rc = nxq_int4_pack(codes.data() + co, scales.data() + go, zeros.data() + go, N, K, gs,
                                   NXQ_INT4_ROWS, blocks.data(), blocks.size()))
            return rc;
        return nxq_weight_register_shard(blocks.data(), blocks.size(), 100 + gs / 32, N, K, split, rank, world, out);
    }
    return fail(NXQ_ERR_CODEC, "nxf: '%s': codec %d is not a quantized-matmul weight codec", t.name.c_str(), codec);
}

}  // namespace
}  // namespace nxq

using nxq::NxfFile;
using nxq::fail;

extern "C" {

NXQ_API int nxq_nxf_open(const char* path, nxq_nxf_t* out) {
    if (!path || !out) return fail(NXQ_ERR_ARG, "nxf_open: null argument");
    *out = nullptr;
    auto* f = new (std::nothrow) NxfFile();
    if (!f) return fail(NXQ_ERR_NOMEM, "nxf_open: out of host memory");
    f->fd = open(path, O_RDONLY | O_CLOEXEC);
    if (f->fd < 0) {
        delete f;
        return fail(NXQ_ERR_ARG, "nxf_open: cannot open '%s' (%s)", path, strerror(errno));
    }
    struct stat st;
    if (fstat(f->fd, &st) != 0 || st.st_size <= 0) {
        delete f;
        return fail(NXQ_ERR_FORMAT, "nxf_open: '%s' is empty or unreadable", path);
    }
    f->size = (uint64_t)st.st_size;
    f->map = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
    if (f->map == MAP_FAILED) {
        f->map = nullptr;
        delete f;
        return fail(NXQ_ERR_NOMEM, "nxf_open: mmap of '%s' failed (%s)", path, strerror(errno));
    }
    int rc;
    try {
        rc = nxq::parse(*f);
    } catch (const std::bad_alloc&) {
        rc = fail(NXQ_ERR_NOMEM, "nxf_open: out of host memory while indexing '%s'", path);
    }
    if (rc != NXQ_OK) {
        delete f;
        return rc;
    }
    *out = reinterpret_cast<nxq_nxf_t>(f);
    return NXQ_OK;
}

NXQ_API int nxq_nxf_close(nxq_nxf_t h) {
    NxfFile* f = nxq::handle(h);
    if (!f) return fail(NXQ_ERR_ARG, "nxf_close: not an open file handle");
    delete f;
    return NXQ_OK;
}

NXQ_API int nxq_nxf_tensor_count(nxq_nxf_t h, int64_t* n) {
    NxfFile* f = nxq::handle(h);
    if (!f || !n) return fail(NXQ_ERR_ARG, "nxf_tensor_count: bad argument");
    *n = (int64_t)f->tensors.size();
    return NXQ_OK;
}

NXQ_API int nxq_nxf_tensor_info(nxq_nxf_t h, int64_t i, char* name, size_t name_len, int* dtype, int* n_dims,
                                int64_t dims[4], int64_t* n_chunks, int* codec, int* group_size, uint64_t* bytes) {
    NxfFile* f = nxq::handle(h);
    if (!f) return fail(NXQ_ERR_ARG, "nxf_tensor_info: not an open file handle");
    if (i < 0 || i >= (int64_t)f->tensors.size()) return fail(NXQ_ERR_ARG, "nxf_tensor_info: index %lld", (long long)i);
    const nxq::Tensor& t = f->tensors[i];
    nxq::copy_str(t.name, name, name_len);
    if (dtype) *dtype = t.dtype;
    if (n_dims) *n_dims = t.n_dims;
    if (dims)
        for (int d = 0; d < 4; ++d) dims[d] = t.dims[d];
    if (n_chunks) *n_chunks = (int64_t)t.chunks.size();
    if (codec) *codec = t.chunks.empty() ? -1 : t.chunks[0].codec;
    if (group_size) *group_size = t.chunks.empty() ? 0 : t.chunks[0].group;
    if (bytes) {
        uint64_t s = 0;
        for (const auto& k : t.chunks) s += k.stored;
        *bytes = s;
    }
    return NXQ_OK;
}

NXQ_API int nxq_nxf_chunk_info(nxq_nxf_t h, int64_t i, int64_t c, uint64_t* offset, uint32_t* stored,
                               uint32_t* decoded, uint32_t* checksum, int* codec, int* group_size) {
    NxfFile* f = nxq::handle(h);
    if (!f) return fail(NXQ_ERR_ARG, "nxf_chunk_info: not an open file handle");
    if (i < 0 || i >= (int64_t)f->tensors.size()) return fail(NXQ_ERR_ARG, "nxf_chunk_info: index %lld", (long long)i);
    const nxq::Tensor& t = f->tensors[i];
    if (c < 0 || c >= (int64_t)t.chunks.size()) return fail(NXQ_ERR_ARG, "nxf_chunk_info: chunk %lld", (long long)c);
    const nxq::Chunk& k = t.chunks[c];
    if (offset) *offset = k.offset;
    if (stored) *stored = k.stored;
    if (decoded) *decoded = k.decoded;
    if (checksum) *checksum = k.checksum;
    if (codec) *codec = k.codec;
    if (group_size) *group_size = k.group;
    return NXQ_OK;
}

NXQ_API int nxq_nxf_find(nxq_nxf_t h, const char* name, int64_t* index) {
    NxfFile* f = nxq::handle(h);
    if (!f || !name || !index) return fail(NXQ_ERR_ARG, "nxf_find: bad argument");
    auto it = f->by_name.find(name);
    if (it == f->by_name.end()) return fail(NXQ_ERR_ARG, "nxf_find: no tensor '%s'", name);
    *index = it->second;
    return NXQ_OK;
}

NXQ_API int nxq_nxf_verify(nxq_nxf_t h, int64_t i) {
    NxfFile* f = nxq::handle(h);
    if (!f) return fail(NXQ_ERR_ARG, "nxf_verify: not an open file handle");
    if (i < 0 || i >= (int64_t)f->tensors.size()) return fail(NXQ_ERR_ARG, "nxf_verify: index %lld", (long long)i);
    int codec, group;
    return nxq::check_chunks(*f, i, &codec, &group);
}

NXQ_API int nxq_nxf_xxh32(const void* data, size_t n, uint32_t* out) {
    if ((!data && n) || !out) return fail(NXQ_ERR_ARG, "nxf_xxh32: bad argument");
    *out = nxq::xxh32(static_cast<const uint8_t*>(data), n);
    return NXQ_OK;
}

NXQ_API int nxq_nxf_manifest(nxq_nxf_t h, char* buf, size_t n, uint64_t* size) {
    NxfFile* f = nxq::handle(h);
    if (!f) return fail(NXQ_ERR_ARG, "nxf_manifest: not an open file handle");
    if (size) *size = f->manifest.size();
    nxq::copy_str(f->manifest, buf, n);
    return NXQ_OK;
}

NXQ_API int nxq_nxf_manifest_number(nxq_nxf_t h, const char* key, double* v) {
    NxfFile* f = nxq::handle(h);
    if (!f || !key || !v) return fail(NXQ_ERR_ARG, "nxf_manifest_number: bad argument");
    const char *p, *e;
    if (int rc = nxq::find_value(*f, key, &p, &e)) return rc;
    if (p < e && *p == '"') return fail(NXQ_ERR_ARG, "nxf: manifest key '%s' is a string", key);
    const std::string s(p, nxq::skip_value(p, e));
    char* stop = nullptr;
    *v = strtod(s.c_str(), &stop);
    if (s.empty() || stop != s.c_str() + s.size()) return fail(NXQ_ERR_FORMAT, "nxf: manifest key '%s' is not a number", key);
    return NXQ_OK;
}

NXQ_API int nxq_nxf_manifest_string(nxq_nxf_t h, const char* key, char* buf, size_t n) {
    NxfFile* f = nxq::handle(h);
    if (!f || !key) return fail(NXQ_ERR_ARG, "nxf_manifest_string: bad argument");
    const char *p, *e;
    if (int rc = nxq::find_value(*f, key, &p, &e)) return rc;
    std::string s;
    if (p >= e || *p != '"') return fail(NXQ_ERR_ARG, "nxf: manifest key '%s' is not a string", key);
    if (!nxq::read_string(p, e, &s)) return fail(NXQ_ERR_FORMAT, "nxf: bad string value of '%s'", key);
    nxq::copy_str(s, buf, n);
    return NXQ_OK;
}

NXQ_API int nxq_nxf_register(nxq_nxf_t h, int64_t i, int64_t slice, nxq_weight_t* out) {
    NxfFile* f = nxq::handle(h);
    if (!f || !out) return fail(NXQ_ERR_ARG, "nxf_register: bad argument");
    if (i < 0 || i >= (int64_t)f->tensors.size()) return fail(NXQ_ERR_ARG, "nxf_register: index %lld", (long long)i);
    try {
        return nxq::register_tensor(*f, i, slice, false, 0, 0, 1, out);
    } catch (const std::bad_alloc&) {
        return fail(NXQ_ERR_NOMEM, "nxf_register: out of host memory");
    }
}

NXQ_API int nxq_nxf_register_shard(nxq_nxf_t h, int64_t i, int64_t slice, int split, int rank, int world,
                                   nxq_weight_t* out) {
    NxfFile* f = nxq::handle(h);
    if (!f || !out) return fail(NXQ_ERR_ARG, "nxf_register_shard: bad argument");
    if (i < 0 || i >= (int64_t)f->tensors.size()) return fail(NXQ_ERR_ARG, "nxf_register_shard: index %lld", (long long)i);
    try {
        return nxq::register_tensor(*f, i, slice, true, split, rank, world, out);
    } catch (const std::bad_alloc&) {
        return fail(NXQ_ERR_NOMEM, "nxf_register_shard: out of host memory");
    }
}

}  // extern "C"
