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

#include <cstdint>

extern "C" {

// Calls nexus::import::dequant_gguf_to_fp32 (gguf_importer.cpp:958) on `n`
// elements of `type` (GGUFType id).  Returns 0 on success, -1 if the reference
// reports the type unsupported.  Unknown types are zero-filled by the reference
// itself (gguf_importer.cpp:993-998).
int ref_dequant(uint32_t type, const uint8_t* src, uint64_t n, float* out) {
    bool ok = nexus::import::dequant_gguf_to_fp32(
        out, src, static_cast<nexus::import::GGUFType>(type), static_cast<size_t>(n));
    return ok ? 0 : -1;
}

// The reference's fp16 -> fp32 conversion (gguf_importer.cpp:202-237).
float ref_fp16_to_fp32(uint16_t h) { return nexus::import::fp16_to_fp32(h); }

}  // extern "C"
