// ComputeDispatchShim (compute_dispatch_nxq.h): the engine's gemm_int4 /
// gemv_int4 over libnxq.so.
#include "compute_dispatch_nxq.h"

#include <chrono>
#include <cstring>
#include <vector>

namespace nxq {

namespace {

std::string nxq_message() {
    char buf[512];
    nxq_last_error(buf, sizeof buf);
    return buf;
}

// The largest NXF INT4 group size that divides K: the scale-less weights of
// gemm_int4 become groups with scale 0.125 and zero 8, whose size only sets
// how many (scale, zero) pairs are stored.
int scaleless_group(int K) {
    for (int gs : {256, 128, 64, 32})
        if (K % gs == 0) return gs;
    return 0;
}

}  // namespace

ComputeDispatchShim::~ComputeDispatchShim() {
    if (ready_) clear_buffer_cache();
}

bool ComputeDispatchShim::init_gpu(const std::string&, int device) {
    const int rc = nxq_init(device);
    last_status_ = rc;
    if (rc != NXQ_OK) {
        last_error_ = nxq_message();
        ready_ = false;
        return false;
    }
    ready_ = true;
    device_ = device;
    return true;
}

std::string ComputeDispatchShim::gpu_name() const {
    return ready_ ? "CUDA device " + std::to_string(device_) + " (nxq, sm_100a)" : "";
}

void ComputeDispatchShim::on_error(int status, float* out, int M, int N, const char* what) {
    last_status_ = status;
    last_error_ = what ? std::string(what) : nxq_message();
    if (zero_fill_on_error_) {
        if (out && M > 0 && N > 0) std::memset(out, 0, sizeof(float) * (size_t)M * (size_t)N);
        return;
    }
    throw ShimError(status, "nxq: " + last_error_);
}

nxq_weight_t ComputeDispatchShim::lookup(const void* key) const {
    std::lock_guard<std::mutex> lk(mu_);
    auto it = cache_.find(key);
    return it == cache_.end() ? nullptr : it->second;
}

size_t ComputeDispatchShim::cached_weights() const {
    std::lock_guard<std::mutex> lk(mu_);
    return cache_.size();
}

void ComputeDispatchShim::gemm_int4(const float* activations, const void* weights_int4, size_t weights_bytes,
                                    float* out, int M, int N, int K) {
    if (!ready_) return on_error(NXQ_ERR_STATE, out, M, N, "gemm_int4: init_gpu has not succeeded");
    if (!activations || !weights_int4 || !out || M <= 0 || N <= 0 || K <= 0 || K % 2 ||
        weights_bytes != (size_t)K / 2 * (size_t)N)
        return on_error(NXQ_ERR_ARG, out, M, N,
                        "gemm_int4: null pointer, non-positive M/N/K, or weights_bytes != K*N/2 (scale-less INT4)");
    nxq_weight_t w = lookup(weights_int4);
    if (!w) {
        const int gs = scaleless_group(K);
        if (!gs) return on_error(NXQ_ERR_SHAPE, out, M, N, "gemm_int4: K must be a multiple of 32");
        const size_t groups = (size_t)(K / gs) * (size_t)N;
        std::vector<float> scales(groups, 0.125f), zeros(groups, 8.0f);
        const int rc = nxq_weight_register_int4(static_cast<const uint8_t*>(weights_int4), scales.data(),
                                                zeros.data(), N, K, gs, NXQ_INT4_KMAJOR, &w);
        if (rc != NXQ_OK) return on_error(rc, out, M, N);
        std::lock_guard<std::mutex> lk(mu_);
        cache_.emplace(weights_int4, w);
    }
    const int rc = nxq_qmatmul_host(w, activations, out, M);
    if (rc != NXQ_OK) return on_error(rc, out, M, N);
    last_status_ = NXQ_OK;
}

void ComputeDispatchShim::gemv_int4(float* out, const float* activations, const uint8_t* weights_q,
                                    const float* scales, const float* zeros, int M, int N, int K,
                                    int group_size) {
    if (!ready_) return on_error(NXQ_ERR_STATE, out, M, N, "gemv_int4: init_gpu has not succeeded");
    if (!out || !activations || !weights_q || !scales || M <= 0 || N <= 0 || K <= 0)
        return on_error(NXQ_ERR_ARG, out, M, N, "gemv_int4: null array or non-positive M, N, K");
    nxq_weight_t w = lookup(weights_q);
    if (!w) {
        const int rc = nxq_weight_register_int4(weights_q, scales, zeros, N, K, group_size, NXQ_INT4_KMAJOR, &w);
        if (rc != NXQ_OK) return on_error(rc, out, M, N);
        std::lock_guard<std::mutex> lk(mu_);
        cache_.emplace(weights_q, w);
    }
    const int rc = nxq_qmatmul_host(w, activations, out, M);
    if (rc != NXQ_OK) return on_error(rc, out, M, N);
    last_status_ = NXQ_OK;
}

void ComputeDispatchShim::clear_buffer_cache() {
    std::lock_guard<std::mutex> lk(mu_);
    for (auto& kv : cache_) nxq_weight_release(kv.second);
    cache_.clear();
}

}  // namespace nxq

extern "C" int nxq_dispatch_host_steps(const nxq_weight_t* w, const float* const* x, float* const* y,
                                       const int64_t* M, int n, int steps, double* seconds) {
    if (!w || !x || !y || !M || n < 0 || steps < 0 || !seconds) return NXQ_ERR_ARG;
    const auto t0 = std::chrono::steady_clock::now();
    for (int s = 0; s < steps; ++s)
        for (int i = 0; i < n; ++i)
            if (const int rc = nxq_qmatmul_host(w[i], x[i], y[i], M[i])) return rc;
    *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    return NXQ_OK;
}

