// Test driver for the C++ shim (nexus-inference-engine-_b200/shim): calls
// ComputeDispatchShim::gemm_int4 / gemv_int4 with the engine's signatures on
// inputs written by tests/test_gpu_shim.py and writes the outputs back.
//   shim_check gemm <dir>   dims "M N K", x.bin (fp32 [M][K]), w.bin ([K/2][N] bytes)
//   shim_check gemv <dir>   dims "M N K gs", x.bin, w.bin, s.bin, z.bin ([K/gs][N] fp32)
//   shim_check errors <dir> error behaviour: exception by default, zero-fill when opted in
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <iterator>
#include <string>
#include <vector>

#include "compute_dispatch_nxq.h"

template <typename T>
static std::vector<T> load(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    std::vector<char> raw((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    std::vector<T> v(raw.size() / sizeof(T));
    std::memcpy(v.data(), raw.data(), v.size() * sizeof(T));
    return v;
}

static void save(const std::string& path, const std::vector<float>& v) {
    std::ofstream f(path, std::ios::binary);
    f.write(reinterpret_cast<const char*>(v.data()), (std::streamsize)(v.size() * sizeof(float)));
}

int main(int argc, char** argv) {
    if (argc < 3) return 2;
    const std::string mode = argv[1], dir = argv[2];
    nxq::ComputeDispatchShim cd;
    if (!cd.init_gpu("unused.metallib", 0)) {
        std::cerr << "init_gpu failed: " << cd.last_error() << "\n";
        return 3;
    }
    std::ifstream dims(dir + "/dims");
    int M = 0, N = 0, K = 0, gs = 0;
    dims >> M >> N >> K >> gs;
    const auto x = load<float>(dir + "/x.bin");
    const auto w = load<uint8_t>(dir + "/w.bin");
    std::vector<float> y((size_t)M * N, -1.0f);
    if (mode == "gemm") {
        cd.gemm_int4(x.data(), w.data(), w.size(), y.data(), M, N, K);
        std::vector<float> y2((size_t)M * N, -1.0f);
        cd.gemm_int4(x.data(), w.data(), w.size(), y2.data(), M, N, K);  // the cached registration
        if (y2 != y || cd.cached_weights() != 1) {
            std::cerr << "second call differs or cache size " << cd.cached_weights() << "\n";
            return 4;
        }
        save(dir + "/y.bin", y);
    } else if (mode == "gemv") {
        const auto s = load<float>(dir + "/s.bin");
        const auto z = load<float>(dir + "/z.bin");
        cd.gemv_int4(y.data(), x.data(), w.data(), s.data(), z.data(), M, N, K, gs);
        save(dir + "/y.bin", y);
    } else if (mode == "errors") {
        try {  // weights_bytes that does not match K*N/2
            cd.gemm_int4(x.data(), w.data(), w.size() + 1, y.data(), M, N, K);
            std::cerr << "no exception\n";
            return 5;
        } catch (const nxq::ShimError& e) {
            if (e.status() != NXQ_ERR_ARG) return 6;
        }
        cd.set_zero_fill_on_error(true);  // the reference's behaviour, opted in
        cd.gemm_int4(x.data(), w.data(), w.size() + 1, y.data(), M, N, K);
        for (float v : y)
            if (v != 0.0f) return 7;
        if (cd.last_status() != NXQ_ERR_ARG) return 8;
        cd.gemv_int4(y.data(), x.data(), w.data(), nullptr, nullptr, M, N, K, 64);
        if (cd.last_status() != NXQ_ERR_ARG) return 9;
        cd.clear_buffer_cache();
        if (cd.cached_weights() != 0) return 10;
        std::cout << "errors ok\n";
    } else {
        return 2;
    }
    return 0;
}
