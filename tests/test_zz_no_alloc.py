"""GPU: the allocation-free entry point nxq_qmatmul_noalloc.

Callers that cannot allocate GPU memory in the middle of their work (an
allocator or memory-pool callback, a latency-critical loop that must not pay
cudaMalloc's implicit device synchronization, a host that reserves all GPU
memory up front) use this entry point: it keeps its split-K partial sums in a
fixed device array inside the library instead of allocating per call.  Here it
must give the same result as the ordinary entry point nxq_qmatmul and as the
CPU oracle (the reference's decoders + fp32 dot products), within the matmul
tolerance of the other tests, on two calls in a row (the second call finds
the first call's leftovers in the shared array); keep that when the output is
large enough that fewer split-K slices fit in the array than the kernel
would use (the split count is then cut to what fits); and refuse an output
larger than the array with a clear error.

This file is named so that pytest collects it last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from nxq import synth
from oracle import loader

pytestmark = pytest.mark.gpu

TOL = 1e-3
ARRAY_FLOATS = 2 ** 21  # the fixed array's size in fp32 values (8 MiB)


def _noalloc(nxq, w, x, y, stream):
    return nxq.lib().nxq_qmatmul_noalloc(w.handle, x.data_ptr(), nxq._dtype_code(x.dtype), y.data_ptr(),
                                         nxq._dtype_code(y.dtype), x.shape[0], ctypes.c_void_p(stream))


def _call(nxq, w, x, N):
    import torch

    got = torch.full((x.shape[0], N), float("nan"), dtype=torch.float32, device="cuda")
    rc = _noalloc(nxq, w, x, got, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, nxq.last_error()
    torch.cuda.synchronize()
    nxq.stream_sync()
    return got.cpu().numpy()


@pytest.mark.parametrize("t,N,K,M", [(12, 4096, 4096, 4), (2, 1000, 768, 3), (11, 512, 2048, 16),
                                     (8, 2048, 4096, 1)])
def test_noalloc_matches_qmatmul_and_oracle_twice(gpu, t, N, K, M):
    import torch

    nxq = gpu
    blocks = synth.make_blocks(t, N, K, seed=N + K + M)
    w = nxq.Weight.register(blocks, t, N, K)
    try:
        for call in range(2):
            xh = synth.make_activations(M, K, seed=31 + call, dtype=np.float16)
            x = torch.from_numpy(xh).cuda()
            want = nxq.qmatmul(w, x).cpu().numpy()
            got = _call(nxq, w, x, N)
            oracle = loader.qmatmul(t, blocks, N, K, xh.astype(np.float32))
            assert synth.rel_l2(got, want) < TOL
            assert synth.rel_l2(got, oracle) < TOL
    finally:
        w.release()


def test_noalloc_split_count_cut_to_the_array(gpu):
    """A call whose kernel would use several split-K slices but whose output
    fills more than half the array (M * N = 1,105,920 > 2^20: one slice fits)
    runs with the slices that fit, right after a call that used many slices
    (N = 4096, M = 1: ten), and again after itself; each result matches the
    oracle."""
    import torch

    nxq = gpu
    t = 12
    big_N, big_K = 4096, 4096
    wide = synth.make_blocks(t, big_N, big_K, seed=77)
    w_many = nxq.Weight.register(wide, t, big_N, big_K)
    N, K, M = 128, 256, 8640  # 1 row tile, 270 token blocks of 32: the kernel wants 2 slices
    assert M * N > ARRAY_FLOATS // 2 and M * N <= ARRAY_FLOATS
    tall = synth.make_blocks(t, N, K, seed=78)
    w_cut = nxq.Weight.register(tall, t, N, K)
    try:
        x1 = synth.make_activations(1, big_K, seed=5, dtype=np.float16)
        got1 = _call(nxq, w_many, torch.from_numpy(x1).cuda(), big_N)
        assert synth.rel_l2(got1, loader.qmatmul(t, wide, big_N, big_K, x1.astype(np.float32))) < TOL
        xm = synth.make_activations(M, K, seed=6, dtype=np.float16)
        want = loader.qmatmul(t, tall, N, K, xm.astype(np.float32))
        for _ in range(2):
            got = _call(nxq, w_cut, torch.from_numpy(xm).cuda(), N)
            assert synth.rel_l2(got, want) < TOL
        got1 = _call(nxq, w_many, torch.from_numpy(x1).cuda(), big_N)
        assert synth.rel_l2(got1, loader.qmatmul(t, wide, big_N, big_K, x1.astype(np.float32))) < TOL
    finally:
        w_many.release()
        w_cut.release()


def test_noalloc_output_of_exactly_the_array(gpu):
    """M * N = 2^21, the largest output accepted, against the oracle."""
    import torch

    nxq = gpu
    t, N, K, M = 2, 128, 64, 16384
    blocks = synth.make_blocks(t, N, K, seed=79)
    w = nxq.Weight.register(blocks, t, N, K)
    try:
        xh = synth.make_activations(M, K, seed=7, dtype=np.float16)
        got = _call(nxq, w, torch.from_numpy(xh).cuda(), N)
        assert synth.rel_l2(got, loader.qmatmul(t, blocks, N, K, xh.astype(np.float32))) < TOL
    finally:
        w.release()


def test_noalloc_rejects_outputs_beyond_its_array(gpu):
    import torch

    nxq = gpu
    N, K, M = 4096, 256, 513  # M * N = 2,101,248 > 2^21
    w = nxq.Weight.register(synth.make_blocks(12, N, K, seed=5), 12, N, K)
    try:
        x = torch.zeros(M, K, dtype=torch.float16, device="cuda")
        y = torch.zeros(M, N, dtype=torch.float32, device="cuda")
        rc = _noalloc(nxq, w, x, y, torch.cuda.current_stream().cuda_stream)
        assert rc == -3
        assert "exceeds its fixed scratch" in nxq.last_error()
    finally:
        w.release()
