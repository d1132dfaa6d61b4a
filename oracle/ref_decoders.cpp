// Test infrastructure only: a wrapper translation unit that exposes the
// reference's own GGUF block decoders, compiled from the reference sources in
// place (see oracle/Makefile).  Nothing in the product links this file; only
// tests/, __graft_entry__.smoke() and bench.py's CPU baseline load the shared
// library it produces (oracle/_ref/libref_decoders.so).
//
// The decoders live in an anonymous namespace inside
// nexus/src/import/gguf_importer.cpp (dequant_gguf_to_fp32 :958-1000), so the
// only way to call them unchanged is to compile that file inside this TU.
#include "import/gguf_importer.cpp"
#include "quant/gptq.h"

#include <cstdint>
#include <cstring>

extern "C" {

// Calls nexus::import::dequant_gguf_to_fp32 (gguf_importer.cpp:958) on `n`
// elements of `type` (GGUFType id).  Returns 0 on success, -1 if the reference
// reports the type unsupported.  Unknown types are zero-filled by the reference
// itself (gguf_importer.cpp:993-998).
int ref_dequant(uint32_t type, const uint8_t* src, uint64_t n, float* out) {
    if (type >= 101 && type <= 108) {
        // NXF INT4 group blocks [scale f32][zero f32][gs/2 codes]: each block
        // through the reference's own nexus::quant::dequant_int4
        // (quant/gptq.cpp:9-27) with that block's scale and zero.
        const int gs = 32 * (int)(type - 100), bb = 8 + gs / 2;
        for (uint64_t b = 0; b < n / gs; ++b) {
            const uint8_t* blk = src + b * bb;
            float scale, zero;
            std::memcpy(&scale, blk, 4);
            std::memcpy(&zero, blk + 4, 4);
            nexus::quant::dequant_int4(out + b * gs, blk + 8, &scale, &zero, gs, gs);
        }
        return 0;
    }
    bool ok = nexus::import::dequant_gguf_to_fp32(
        out, src, static_cast<nexus::import::GGUFType>(type), static_cast<size_t>(n));
    return ok ? 0 : -1;
}

// nexus::quant::dequant_int4 (quant/gptq.cpp:9-27) over flat arrays.
void ref_dequant_int4(float* out, const uint8_t* data, const float* scales, const float* zeros, int n,
                      int group_size) {
    nexus::quant::dequant_int4(out, data, scales, zeros, n, group_size);
}

// The reference's fp16 -> fp32 conversion (gguf_importer.cpp:202-237).
float ref_fp16_to_fp32(uint16_t h) { return nexus::import::fp16_to_fp32(h); }

// The reference's own NXF writer (format/nxf_writer.cpp: create, set_manifest,
// begin_tensor, add_chunk, end_tensor, finalize), so that tests read files
// made by the reference itself.  ref_nxf_finish finalizes and frees the writer.
void* ref_nxf_create(const char* path) { return nexus::format::NXFWriter::create(path).release(); }

void ref_nxf_manifest(void* w, const char* architecture, const char* name, uint32_t num_layers,
                      uint32_t hidden_dim, float rope_theta, float rms_norm_eps, uint32_t default_codec,
                      uint32_t default_group_size) {
    nexus::format::ModelManifest m{};
    m.architecture = architecture;
    m.name = name;
    m.num_layers = num_layers;
    m.hidden_dim = hidden_dim;
    m.rope_theta = rope_theta;
    m.rms_norm_eps = rms_norm_eps;
    m.default_codec = static_cast<nexus::Codec>(default_codec);
    m.default_group_size = static_cast<uint8_t>(default_group_size);
    static_cast<nexus::format::NXFWriter*>(w)->set_manifest(m);
}

void ref_nxf_begin(void* w, const char* name, int ndim, const int64_t* shape, int dtype) {
    static_cast<nexus::format::NXFWriter*>(w)->begin_tensor(
        name, std::vector<int64_t>(shape, shape + ndim), static_cast<nexus::DType>(dtype));
}

void ref_nxf_chunk(void* w, const void* data, size_t size, int codec, int group_size) {
    static_cast<nexus::format::NXFWriter*>(w)->add_chunk(data, size, static_cast<nexus::Codec>(codec),
                                                         static_cast<uint8_t>(group_size));
}

void ref_nxf_end(void* w) { static_cast<nexus::format::NXFWriter*>(w)->end_tensor(); }

void ref_nxf_finish(void* w) {
    auto* writer = static_cast<nexus::format::NXFWriter*>(w);
    writer->finalize();
    delete writer;
}

}  // extern "C"
