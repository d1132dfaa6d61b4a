// C++ shim with the NEXUS engine's quantized-matmul operator signatures,
// forwarding to the C ABI of libnxq.so (include/nxq.h).
//
// The engine calls
//   ComputeDispatch::gemm_int4(const float* activations, const void* weights_int4,
//                              size_t weights_bytes, float* out, int M, int N, int K)
//   ComputeDispatch::gemv_int4(float* out, const float* activations,
//                              const uint8_t* weights_q, const float* scales,
//                              const float* zeros, int M, int N, int K, int group_size)
// (nexus/src/compute/compute_dispatch.h:47-61, .cpp:142-207).  This class has
// those two methods with the same signatures, plus init_gpu / has_gpu /
// gpu_name / clear_buffer_cache (compute_dispatch.h:26-35, .cpp:853-860), so a
// CUDA build of ComputeDispatch forwards each call to it unchanged.
//
// What differs from the reference, on purpose:
//   - weights are registered into HBM once per host pointer (the reference's
//     wrapped_buffer_cache_, compute_dispatch.h:311) and stay resident;
//   - every row of the activations is used (the reference's gemm_int4 ignores
//     M, compute_dispatch.cpp:156-164);
//   - a failure throws nxq::ShimError (status and message) instead of the
//     reference's silent zero-fill (compute_dispatch.cpp:174-176); calling
//     set_zero_fill_on_error(true) restores that behaviour (the output is
//     zero-filled, no exception, last_status() holds the error);
//   - the cache is guarded by a mutex (the reference's is unsynchronized).
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "nxq.h"

namespace nxq {

class ShimError : public std::runtime_error {
public:
    ShimError(int status, const std::string& msg) : std::runtime_error(msg), status_(status) {}
    int status() const { return status_; }

private:
    int status_;
};

class ComputeDispatchShim {
public:
    ComputeDispatchShim() = default;
    ~ComputeDispatchShim();
    ComputeDispatchShim(const ComputeDispatchShim&) = delete;
    ComputeDispatchShim& operator=(const ComputeDispatchShim&) = delete;

    // Initialises nxq on CUDA device `device` (the reference's argument is the
    // path of its Metal shader library; there is nothing to load here).
    // Returns false (and keeps the status) when no sm_100 GPU is usable.
    bool init_gpu(const std::string& shader_path = "", int device = 0);
    bool has_gpu() const { return ready_; }
    std::string gpu_name() const;

    // Scale-less INT4 weights in the GEMV shader's [K/2][N] byte order
    // (gemv_int4_nr8.metal:31-80: byte (k/2)*N + n holds k in the low and
    // k+1 in the high nibble, w = (q - 8) * 0.125); weights_bytes = K*N/2.
    // out[M][N] = activations[M][K] * W^T, fp32 in and out.
    void gemm_int4(const float* activations, const void* weights_int4, size_t weights_bytes, float* out,
                   int M, int N, int K);

    // NXF INT4 group weights: packed codes [K/2][N], fp32 scales and zeros
    // [K/group_size][N] (gemm_dequant.metal:29-70's K-major order; zeros may
    // be null), w = (q - zero) * scale.
    void gemv_int4(float* out, const float* activations, const uint8_t* weights_q, const float* scales,
                   const float* zeros, int M, int N, int K, int group_size);

    // Releases every registered weight (compute_dispatch.cpp:853-860).
    void clear_buffer_cache();

    void set_zero_fill_on_error(bool on) { zero_fill_on_error_ = on; }
    int last_status() const { return last_status_; }
    const std::string& last_error() const { return last_error_; }
    size_t cached_weights() const;

private:
    // Records the failure (`what`, else libnxq's last error message), then
    // zero-fills `out` (M*N floats) or throws ShimError.
    void on_error(int status, float* out, int M, int N, const char* what = nullptr);
    nxq_weight_t lookup(const void* key) const;

    bool ready_ = false;
    int device_ = -1;
    bool zero_fill_on_error_ = false;
    int last_status_ = NXQ_OK;
    std::string last_error_;
    mutable std::mutex mu_;
    std::unordered_map<const void*, nxq_weight_t> cache_;
};

}  // namespace nxq

// The engine's synchronous call pattern, timed in C++: `steps` passes over the
// n calls nxq_qmatmul_host(w[i], x[i], y[i], M[i]) (host fp32 activations and
// outputs, weights resident), one after another on the calling thread, as
// ComputeDispatch::gemm_int4 issues them (compute_dispatch.cpp:142-176).
// Stores the wall time of all passes in *seconds; returns the first failing
// call's status.  bench.py measures the host drop-in with it, so no Python
// call overhead sits between the calls.
extern "C" int nxq_dispatch_host_steps(const nxq_weight_t* w, const float* const* x, float* const* y,
                                       const int64_t* M, int n, int steps, double* seconds);
