"""GPU: device decode of the HBM-resident tiled copy is bit-identical to the
reference decoders (golden fixtures from the compiled reference; and the
oracle restatement, itself pinned to the reference, at benchmark sizes)."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from conftest import ALL_TYPES, MAIN_TYPES, NAMES, golden
from oracle import loader
from nxq import synth

pytestmark = pytest.mark.gpu


def _decode_gpu(nxq, blocks, t, N, K):
    w = nxq.Weight.register(blocks, t, N, K)
    try:
        y = w.dequant()
        import torch

        torch.cuda.synchronize()
        return y.cpu().numpy()
    finally:
        w.release()


@pytest.mark.parametrize("t", ALL_TYPES, ids=lambda t: NAMES[t])
def test_decode_matches_golden_kat(gpu, t):
    g = golden(t)
    qk, bb = synth.GEOMETRY[t]
    nb = g["kat_blocks"].size // bb
    # One row of all KAT blocks.
    out = _decode_gpu(gpu, g["kat_blocks"], t, 1, nb * qk)
    assert loader.same_bits(out.reshape(-1), g["kat_out"])


@pytest.mark.parametrize("t", ALL_TYPES, ids=lambda t: NAMES[t])
def test_decode_matches_golden_matrix(gpu, t):
    g = golden(t)
    N, K = int(g["mat_N"]), int(g["mat_K"])
    out = _decode_gpu(gpu, g["mat_blocks"], t, N, K)
    assert hashlib.sha256(np.ascontiguousarray(out, np.float32).tobytes()).hexdigest() == str(g["mat_w_sha256"])


@pytest.mark.parametrize("t", ALL_TYPES, ids=lambda t: NAMES[t])
@pytest.mark.parametrize("shape", [(1, 256), (3, 768), (129, 512), (300, 1024)])
def test_decode_raw_bytes_ragged(gpu, t, shape):
    N, K = shape
    blocks = synth.make_blocks(t, N, K, seed=N * 31 + K, dist="raw")
    out = _decode_gpu(gpu, blocks, t, N, K)
    assert loader.same_bits(out.reshape(-1), loader.dequant(t, blocks, N * K))


@pytest.mark.parametrize("t,N,K", [(2, 4096, 4096), (12, 14336, 4096), (12, 4096, 14336),
                                   (8, 1024, 4096), (11, 1024, 16384)])
def test_decode_benchmark_shapes(gpu, t, N, K):
    blocks = synth.make_blocks(t, N, K, seed=5)
    out = _decode_gpu(gpu, blocks, t, N, K)
    assert loader.same_bits(out.reshape(-1), loader.dequant(t, blocks, N * K))


def test_register_from_device_and_shards(gpu):
    import torch

    nxq = gpu
    t, N, K = 12, 256, 2048
    blocks = synth.make_blocks(t, N, K, seed=9)
    ref = loader.dequant(t, blocks, N * K).reshape(N, K)
    dev = torch.from_numpy(blocks).cuda()
    w = nxq.Weight.register_device(dev, t, N, K)
    assert loader.same_bits(w.dequant().cpu().numpy(), ref)
    w.release()
    for split, world in ((nxq.SPLIT_COL, 4), (nxq.SPLIT_ROW, 2), (nxq.SPLIT_ROW, 8)):
        for rank in range(world):
            s = nxq.Weight.register_shard(blocks, t, N, K, split, rank, world)
            got = s.dequant().cpu().numpy()
            if split == nxq.SPLIT_COL:
                want = ref[rank * N // world:(rank + 1) * N // world]
            else:
                want = ref[:, rank * K // world:(rank + 1) * K // world]
            assert loader.same_bits(got, want)
            s.release()


def test_register_rejects_bad_input(gpu):
    nxq = gpu
    b = synth.make_blocks(12, 4, 512, seed=1)
    with pytest.raises(nxq.NxqError) as e:
        nxq.Weight.register(b, 12, 4, 500)
    assert e.value.code == -3
    with pytest.raises(nxq.NxqError) as e:
        nxq.Weight.register(b[:-1], 12, 4, 512)
    assert e.value.code == -3
    with pytest.raises(nxq.NxqError) as e:
        nxq.Weight.register(b, 99, 4, 512)
    assert e.value.code == -2
    w = nxq.Weight.register(b, 12, 4, 512)
    h = w.handle
    w.release()
    assert nxq.lib().nxq_weight_release(h) == -1  # stale handle detected
