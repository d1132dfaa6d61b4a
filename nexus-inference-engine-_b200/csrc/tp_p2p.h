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

// The allreduce of p.buf over the ranks, in place, on `st`.
cudaError_t launch_p2p_allreduce(const P2PParams& p, cudaStream_t st);

}  // namespace nxq
