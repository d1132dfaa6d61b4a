"""GPU: the allocation-free entry point nxq_qmatmul_noalloc.

Callers that cannot allocate GPU memory in the middle of their work (an
allocator or memory-pool callback, a latency-critical loop that must not pay
cudaMalloc's implicit device synchronization, a host that reserves all GPU
memory up front) use this entry point: it keeps its split-K partial sums in a
fixed device array inside the library instead of allocating per call.  Here it
must give the same result as the ordinary entry point nxq_qmatmul, within the
matmul tolerance of the other tests, on two calls in a row (the second call
finds the first call's leftovers in the shared array), and must refuse an
output larger than its fixed array with a clear error.

This file is named so that pytest collects it last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from nxq import synth

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _noalloc(nxq, w, x, y, stream):
    return nxq.lib().nxq_qmatmul_noalloc(w.handle, x.data_ptr(), nxq._dtype_code(x.dtype), y.data_ptr(),
                                         nxq._dtype_code(y.dtype), x.shape[0], ctypes.c_void_p(stream))


@pytest.mark.parametrize("t,N,K,M", [(12, 4096, 4096, 4), (2, 1000, 768, 3), (11, 512, 2048, 16),
                                     (8, 2048, 4096, 1)])
def test_noalloc_matches_qmatmul_twice(gpu, t, N, K, M):
    import torch

    nxq = gpu
    blocks = synth.make_blocks(t, N, K, seed=N + K + M)
    w = nxq.Weight.register(blocks, t, N, K)
    try:
        stream = torch.cuda.current_stream().cuda_stream
        for call in range(2):
            x = torch.from_numpy(synth.make_activations(M, K, seed=31 + call, dtype=np.float16)).cuda()
            want = nxq.qmatmul(w, x)
            got = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
            rc = _noalloc(nxq, w, x, got, stream)
            assert rc == 0, nxq.last_error()
            torch.cuda.synchronize()
            nxq.stream_sync()
            assert synth.rel_l2(got.cpu().numpy(), want.cpu().numpy()) < TOL
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
