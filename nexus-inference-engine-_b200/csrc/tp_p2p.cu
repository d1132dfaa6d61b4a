// One-shot fp32 allreduce over NVLink peer memory for the tensor-parallel row
// split (tp.cu).  The reference runs on one device and has no counterpart.
//
// The row-split projections of a decode step end in allreduces of M x N fp32
// partial outputs of 16 KB - 2 MB, where NCCL's per-call latency (about 12 us
// measured on this B200 box) is several times the transfer time.  Here every
// rank keeps a "symmetric" device buffer - data [2][cap] floats, then ready
// flags [world][kP2PBlocks] and a control word pair - whose address every other
// rank has mapped through CUDA IPC (the handles are exchanged once, at
// nxq_tp_init, through the NCCL communicator).  One kernel per allreduce:
//   1. block b copies its slice of the local partial into the half (epoch & 1)
//      of its own data buffer;
//   2. one thread writes epoch + 1 into block b's ready flag of every peer
//      (st.release.sys, after a system-scope fence);
//   3. threads 0 .. world-1 wait (bounded) until every peer's flag for block b
//      reads epoch + 1 (ld.acquire.sys);
//   4. block b sums its slice over ranks 0 .. world-1 in rank order, reading
//      the peers' halves over NVLink, and stores it in place: every rank gets
//      the same bits;
//   5. the last block to finish advances the epoch (a device counter, so a
//      call replayed from a CUDA graph sees the next epoch).
// Reuse of a half is safe without a second barrier: a peer signals epoch e + 1
// only after its epoch-e kernel (which read my half e & 1) has completed, and
// I overwrite that half at epoch e + 2 only after seeing its epoch-(e + 1)
// signal.  Every wait is bounded by the context's wait limit; a wait that runs
// out records NXQ_ERR_TIMEOUT in the status word.  No multicast: plain peer
// loads and stores only.
#include <cuda_runtime.h>

#include "nxq_internal.h"
#include "sm100_ptx.cuh"
#include "tp_p2p.h"

namespace nxq {

namespace {

constexpr int kThreads = 512;

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void __launch_bounds__(kThreads) p2p_allreduce_kernel(const P2PParams p) {
    __shared__ int s_ok;
    const int b = blockIdx.x, nb = gridDim.x, tid = threadIdx.x;
    const unsigned long long e = *reinterpret_cast<volatile const unsigned long long*>(p.ctl);
    const int64_t per = ((p.count + nb - 1) / nb + 3) & ~(int64_t)3;  // a multiple of 4 floats
    const int64_t lo = (int64_t)b * per, hi = lo + per < p.count ? lo + per : p.count;
    const int64_t half = (int64_t)(e & 1ull) * p.cap;
    float* mine = p.data[p.rank] + half;
    // 1. the local partial into this rank's half (16-byte pieces where the
    // caller's buffer allows, the slice starts on a multiple of 4 floats).
    const bool vec = (reinterpret_cast<uintptr_t>(p.buf) & 15u) == 0;
    const int64_t n4 = vec ? (hi - lo) / 4 : 0;
    for (int64_t i = tid; i < n4; i += kThreads)
        reinterpret_cast<float4*>(mine + lo)[i] = reinterpret_cast<const float4*>(p.buf + lo)[i];
    for (int64_t i = lo + 4 * n4 + tid; i < hi; i += kThreads) mine[i] = p.buf[i];
    if (tid == 0) s_ok = 1;
    __syncthreads();
    // 2. ready: every peer learns that slice b of this rank's half is written.
    if (tid == 0) {
        __threadfence_system();
        for (int r = 0; r < p.world; ++r)
            if (r != p.rank) st_release_sys(p.flags[r] + (size_t)p.rank * kP2PBlocks + b, e + 1);
    }
    // 3. wait (bounded) for every peer's slice b.
    if (tid < p.world && tid != p.rank) {
        const unsigned long long* f = p.flags[p.rank] + (size_t)tid * kP2PBlocks + b;
        const long long t0 = clock64(), lim = ptx::wait_limit(p.status);
        while (ld_acquire_sys(f) < e + 1) {
            if (clock64() - t0 > lim) {
                if (atomicCAS(&p.status->code, 0u, kStatusTimeout) == 0u) {
                    p.status->where = 40;
                    raise_host_flag(p.status);
                }
                s_ok = 0;
                break;
            }
            __nanosleep(100);
        }
    }
    __syncthreads();
    // 4. the sum in rank order, in place: every rank's piece is requested
    // before any is added (the remote loads overlap), kU pieces per thread
    // at a time.
    if (s_ok) {
        constexpr int kU = 4;
        const float* src[kP2PMaxWorld];
#pragma unroll
        for (int r = 0; r < kP2PMaxWorld; ++r) src[r] = r < p.world ? (r == p.rank ? mine : p.data[r] + half) + lo : nullptr;
        for (int64_t i0 = tid; i0 < n4; i0 += kU * kThreads) {
            float4 v[kU][kP2PMaxWorld];
#pragma unroll
            for (int u = 0; u < kU; ++u)
#pragma unroll
                for (int r = 0; r < kP2PMaxWorld; ++r)
                    if (r < p.world && i0 + u * kThreads < n4)
                        v[u][r] = __ldcv(reinterpret_cast<const float4*>(src[r]) + i0 + u * kThreads);
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                if (i0 + u * kThreads >= n4) break;
                float4 a = v[u][0];
#pragma unroll
                for (int r = 1; r < kP2PMaxWorld; ++r)
                    if (r < p.world) {
                        a.x += v[u][r].x;
                        a.y += v[u][r].y;
                        a.z += v[u][r].z;
                        a.w += v[u][r].w;
                    }
                reinterpret_cast<float4*>(p.buf + lo)[i0 + u * kThreads] = a;
            }
        }
        for (int64_t i = lo + 4 * n4 + tid; i < hi; i += kThreads) {
            float v = 0.0f;
            for (int r = 0; r < p.world; ++r) v += (r == p.rank ? mine : p.data[r] + half)[i];
            p.buf[i] = v;
        }
    }
    // 5. the last block advances the epoch.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(reinterpret_cast<unsigned int*>(p.ctl + 1), 1u) == (unsigned)(nb - 1)) {
            *reinterpret_cast<volatile unsigned int*>(p.ctl + 1) = 0u;
            __threadfence();
            *reinterpret_cast<volatile unsigned long long*>(p.ctl) = e + 1;
        }
    }
}

}  // namespace

size_t p2p_bytes(int world, int64_t cap) {
    return (size_t)2 * cap * sizeof(float) + (size_t)world * kP2PBlocks * sizeof(unsigned long long) +
           2 * sizeof(unsigned long long);
}

size_t tpx_bytes(int world) {
    return ((size_t)2 * world * kTpxSlotWords + 2) * sizeof(unsigned long long);
}

cudaError_t launch_p2p_allreduce(const P2PParams& p, cudaStream_t st) {
    int64_t nb = (p.count + 1023) / 1024;
    if (nb < 1) nb = 1;
    if (nb > kP2PBlocks) nb = kP2PBlocks;
    p2p_allreduce_kernel<<<(unsigned)nb, kThreads, 0, st>>>(p);
    note_launches(1);
    return cudaGetLastError();
}

}  // namespace nxq
