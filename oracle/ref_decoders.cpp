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

}  // extern "C"
