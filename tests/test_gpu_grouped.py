"""GPU: nxq_qmatmul_grouped (grouped / MoE GEMV) against the oracle and against
separate nxq_qmatmul calls.

Cases: projections sharing one input (q/k/v style), many experts with their
own inputs and batch sizes (more than one launch's 16 weights, an expert with
M = 0), and the inputs that run item by item instead (mixed block types,
prefill batch sizes, fp32 activations with M > 2).  Also checks that a group
of one block type runs as one launch per 16 weights, and that weights with
more tiles than the GPU has SMs (runs of tile-chunks that cross tiles, tiles
finished by the last of the CTAs that share them) give the same bits on every
call."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import NAMES
from oracle import loader
from nxq import synth

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _torch():
    import torch

    return torch


def _weights(gpu, t, shapes, seed):
    blocks = [synth.make_blocks(t, N, K, seed=seed + i) for i, (N, K) in enumerate(shapes)]
    return blocks, [gpu.Weight.register(b, t, N, K) for b, (N, K) in zip(blocks, shapes)]


@pytest.mark.parametrize("t", [12, 11, 8, 2], ids=lambda t: NAMES[t])
@pytest.mark.parametrize("M", [1, 5, 16, 32])
def test_shared_input_projections(gpu, t, M):
    torch = _torch()
    K = 1024
    shapes = [(512, K), (128, K), (128, K)]
    blocks, ws = _weights(gpu, t, shapes, seed=300 + M)
    try:
        x = torch.from_numpy(synth.make_activations(M, K, seed=M)).cuda()
        ys = gpu.qmatmul_grouped(ws, [x] * 3)
        sep = [gpu.qmatmul(w, x) for w in ws]
        torch.cuda.synchronize()
        xf = x.float().cpu().numpy()
        for (N, _), b, y, s in zip(shapes, blocks, ys, sep):
            want = loader.qmatmul(t, b, N, K, xf)
            assert synth.rel_l2(y.cpu().numpy(), want) < TOL
            assert synth.rel_l2(y.cpu().numpy(), s.cpu().numpy()) < 1e-5
    finally:
        for w in ws:
            w.release()


@pytest.mark.parametrize("t", [12, 8], ids=lambda t: NAMES[t])
@pytest.mark.parametrize("M", [1, 5, 32])
def test_large_group_shared_tiles(gpu, t, M):
    torch = _torch()
    K = 2048
    shapes = [(9728, K), (9728, K), (1024, K)]  # 160 tiles: no cluster split fits
    blocks, ws = _weights(gpu, t, shapes, seed=400 + M)
    try:
        x = torch.from_numpy(synth.make_activations(M, K, seed=M)).cuda()
        ys = gpu.qmatmul_grouped(ws, [x] * 3)
        torch.cuda.synchronize()
        xf = x.float().cpu().numpy()
        for (N, _), b, y in zip(shapes, blocks, ys):
            assert synth.rel_l2(y.cpu().numpy(), loader.qmatmul(t, b, N, K, xf)) < TOL
        for _ in range(3):
            again = gpu.qmatmul_grouped(ws, [x] * 3)
            torch.cuda.synchronize()
            assert all(torch.equal(a, b) for a, b in zip(ys, again))
    finally:
        for w in ws:
            w.release()


@pytest.mark.parametrize("t", [12, 11], ids=lambda t: NAMES[t])
def test_many_experts_own_inputs(gpu, t):
    torch = _torch()
    E, N, K = 20, 256, 512
    Ms = [1, 3, 0, 8, 2, 1, 7, 4, 1, 1, 6, 2, 5, 1, 3, 8, 1, 2, 1, 4]
    blocks, ws = _weights(gpu, t, [(N, K)] * E, seed=700)
    try:
        xs = [torch.from_numpy(synth.make_activations(max(m, 1), K, seed=800 + i))[:m].contiguous().cuda()
              for i, m in enumerate(Ms)]
        ys = gpu.qmatmul_grouped(ws, xs)
        torch.cuda.synchronize()
        for i, m in enumerate(Ms):
            assert tuple(ys[i].shape) == (m, N)
            if m == 0:
                continue
            want = loader.qmatmul(t, blocks[i], N, K, xs[i].float().cpu().numpy())
            assert synth.rel_l2(ys[i].cpu().numpy(), want) < TOL, i
    finally:
        for w in ws:
            w.release()


def test_one_launch_per_sixteen_weights(gpu):
    torch = _torch()
    t, N, K = 12, 256, 512
    _, ws = _weights(gpu, t, [(N, K)] * 17, seed=900)
    try:
        x = torch.from_numpy(synth.make_activations(2, K, seed=1)).cuda()
        gpu.qmatmul_grouped(ws[:3], [x] * 3)  # warm-up
        torch.cuda.synchronize()
        n0 = gpu.launch_count()
        gpu.qmatmul_grouped(ws[:16], [x] * 16)
        n1 = gpu.launch_count()
        gpu.qmatmul_grouped(ws, [x] * 17)
        n2 = gpu.launch_count()
        torch.cuda.synchronize()
        assert n1 - n0 == 1 and n2 - n1 == 2
    finally:
        for w in ws:
            w.release()


def test_fallbacks_run_item_by_item(gpu):
    torch = _torch()
    K = 512
    b4, w4 = _weights(gpu, 12, [(256, K)], seed=1000)
    b3, w3 = _weights(gpu, 11, [(128, K)], seed=1001)
    try:
        cases = [
            ([w4[0], w3[0]], [b4[0], b3[0]], [12, 11], [256, 128], 3, torch.float16),   # mixed types
            ([w4[0], w4[0]], [b4[0], b4[0]], [12, 12], [256, 256], 40, torch.float16),  # prefill M
            ([w4[0], w4[0]], [b4[0], b4[0]], [12, 12], [256, 256], 3, torch.float32),   # fp32, M > 2
            ([w4[0], w4[0]], [b4[0], b4[0]], [12, 12], [256, 256], 2, torch.float32),   # fp32, M <= 2
        ]
        for ws, bs, ts, Ns, M, dt in cases:
            x = torch.from_numpy(synth.make_activations(M, K, seed=M).astype(np.float32)).to(dt).cuda()
            ys = gpu.qmatmul_grouped(ws, [x] * len(ws))
            torch.cuda.synchronize()
            for y, b, t, N in zip(ys, bs, ts, Ns):
                want = loader.qmatmul(t, b, N, K, x.float().cpu().numpy())
                assert synth.rel_l2(y.cpu().numpy(), want) < TOL, (ts, M, dt)
    finally:
        w4[0].release()
        w3[0].release()


def test_grouped_errors(gpu):
    import ctypes

    L = gpu.lib()
    assert L.nxq_qmatmul_grouped(None, 2, None, 1, None, 0, None, None) == -1
    assert L.nxq_qmatmul_grouped(None, -1, None, 1, None, 0, None, None) == -1
    assert L.nxq_qmatmul_grouped(None, 0, None, 1, None, 0, None, None) == 0
    arr = (ctypes.c_void_p * 1)(None)
    M = (ctypes.c_int64 * 1)(1)
    assert L.nxq_qmatmul_grouped(arr, 1, arr, 1, arr, 0, M, None) == -1  # null weight handle
