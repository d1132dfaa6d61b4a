// The peer-memory allreduce of the tensor-parallel layer (tp_p2p.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "nxq_internal.h"

namespace nxq {

constexpr int kP2PMaxWorld = 8;
constexpr int kP2PBlocks = 128;  // blocks (slices) of one allreduce, at most

// Layout of a rank's symmetric buffer: data [2][cap] fp32, then ready flags
// [world][kP2PBlocks] u64 (flag (r, b): rank r has written slice b of the
// current epoch), then the control pair {epoch, done-block counter}.
struct P2PParams {
    float* buf;     // this rank's partial in, the sum out (count floats, device)
    int64_t count;
    int rank, world;
    int64_t cap;    // floats per data half
    float* data[kP2PMaxWorld];                  // rank r's data (own: local pointer)
    unsigned long long* flags[kP2PMaxWorld];    // rank r's flag array
    unsigned long long* ctl;                    // this rank's control pair
    DeviceStatus* status;
};

// Bytes of one rank's symmetric buffer.
size_t p2p_bytes(int world, int64_t cap);

// ---- tile exchange of the fused row-split decode GEMV (qmm_mma.cu) ----------
// Each rank's symmetric buffer holds words [2][world][kTpxSlotWords] u64 - a
// slot per launch parity and source rank, tile t of a launch at
// [t][TILE_ROWS rows][RS tokens] (RS = the kernel's 8, 16 or 32 token
// columns) - then the control pair {epoch, done-CTA counter}.  A word carries
// one fp32 partial in its low half and the tag (epoch + 1, 32 bits) of the
// launch that wrote it in its high half: one 8-byte store, so a reader that
// sees the tag it expects sees the value with it, without a fence or flag.
constexpr int kTpxMaxTiles = 512;  // rows per call: 512 x 128 = 65536
constexpr int kTpxCtaTiles = 16;   // finished tiles one CTA can hold for the exchange
// Largest exchange a rank sends per call ((world - 1) x N x M words).  Every
// rank sends its whole partial to every peer, so the volume grows with the
// world; measured against GEMV + NCCL allreduce on B200 (405B-shaped rows,
// N = 16384): fused faster at 7.3 MB (8 ranks, M = 8) and 4.2 MB (2 ranks,
// M = 32), slower at 12.6 MB (4 ranks, M = 32) and 29 MB (8 ranks, M = 32).
constexpr int64_t kTpxMaxBytes = 8 << 20;
constexpr int64_t kTpxSlotWords = (int64_t)kTpxMaxTiles * TILE_ROWS * 32;

struct TpExchange {
    int on, rank, world;
    int owner;  // 1: owner exchange (tile t summed by rank t mod world, two hops); 0: all-to-all (one hop)
    unsigned long long* recv[kP2PMaxWorld];  // rank q's words (own: local pointer)
    unsigned long long* ctl;                 // this rank's control pair
};

// Bytes of one rank's tile-exchange buffer.
size_t tpx_bytes(int world);

// The allreduce of p.buf over the ranks, in place, on `st`.
cudaError_t launch_p2p_allreduce(const P2PParams& p, cudaStream_t st);

}  // namespace nxq
