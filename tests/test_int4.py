"""NXF INT4 group weights (quant/gptq.cpp:9-70): w = (q - zero) * scale with
one fp32 scale and zero per group of gs elements along K, registered as
NXQ_TYPE_I4G<gs> blocks.

CPU: the oracle restatement of dequant_int4 against the golden fixtures made
by the reference's own compiled function (tests/golden/golden_I4G.npz:
special scales and zeros, codes 0 and 15, zeros omitted), the block form
against the flat form, packing from quant/gptq.cpp's flat order and from the
GEMV shader's K-major order (identical blocks), and packing errors.
GPU: registration from both orders decodes bit-exactly to the fixtures and
the reference; matmul within the parity bar on the decode GEMV and the
prefill GEMM for every group size."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import nxq
from nxq import synth
from oracle import loader

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden_I4G.npz"
GS = (32, 64, 128, 256)
TOL = 1e-3


def _g():
    return np.load(GOLDEN)


def _to_kmajor(codes, scales, zeros, N, K, gs):
    """quant/gptq.cpp flat arrays over W[N][K] -> gemv_dequant_int4's order."""
    q = np.empty((N, K), np.uint8)
    c = codes.reshape(N, K // 2)
    q[:, 0::2] = c & 15
    q[:, 1::2] = c >> 4
    km = (q.T[0::2, :] | (q.T[1::2, :] << 4)).astype(np.uint8)  # [K/2][N]
    z = None if zeros is None else zeros.reshape(N, K // gs).T.copy()
    return km, scales.reshape(N, K // gs).T.copy(), z


@pytest.mark.parametrize("gs", GS)
def test_oracle_pinned_to_reference_fixtures(gs):
    g = _g()
    codes, sc, z = g[f"g{gs}_codes"], g[f"g{gs}_scales"], g[f"g{gs}_zeros"]
    n = codes.size * 2
    assert loader.same_bits(loader.dequant_int4(codes, sc, z, n, gs), g[f"g{gs}_out"])
    assert loader.same_bits(loader.dequant_int4(codes, sc, None, n, gs), g[f"g{gs}_nozero_out"])


@pytest.mark.parametrize("gs", GS)
def test_block_form_and_layouts(gs):
    g = _g()
    codes, sc, z = g[f"g{gs}_codes"], g[f"g{gs}_scales"], g[f"g{gs}_zeros"]
    N, K = 2, codes.size  # 2 rows of K = n / 2 elements
    t = 100 + gs // 32
    blk = nxq.int4_pack(codes, sc, z, N, K, gs, nxq.INT4_ROWS)
    assert loader.same_bits(loader.dequant(t, blk, N * K), g[f"g{gs}_out"])
    km, skm, zkm = _to_kmajor(codes, sc, z, N, K, gs)
    assert np.array_equal(nxq.int4_pack(km, skm, zkm, N, K, gs, nxq.INT4_KMAJOR), blk)
    blk0 = nxq.int4_pack(codes, sc, None, N, K, gs, nxq.INT4_ROWS)
    assert loader.same_bits(loader.dequant(t, blk0, N * K), g[f"g{gs}_nozero_out"])


@pytest.mark.parametrize("gs", GS)
def test_matrix_fixture_through_oracle(gs):
    g = _g()
    t = 100 + gs // 32
    mb, N, K = g[f"g{gs}_mat_blocks"], int(g[f"g{gs}_mat_N"]), int(g[f"g{gs}_mat_K"])
    y = loader.qmatmul(t, mb, N, K, g[f"g{gs}_mat_x"], nthreads=2)
    assert np.array_equal(y, g[f"g{gs}_mat_y"])


def test_gemm_int4_scaleless_weights_map_to_groups():
    """The reference's gemm_int4 weights (gemv_int4_nr8.metal:31-80: [K/2][N]
    bytes, byte (k/2)*N + n holding k low and k+1 high, w = (q - 8) * 0.125,
    no scales) are NXF INT4 groups in the K-major order with every scale 0.125
    and every zero 8: the same bits, and the same product as the shader's
    formula."""
    rng = np.random.default_rng(11)
    N, K, gs = 48, 256, 128
    km = rng.integers(0, 256, (K // 2, N), dtype=np.uint8)
    q = np.empty((N, K), np.float32)
    q[:, 0::2] = (km & 15).T
    q[:, 1::2] = (km >> 4).T
    w_shader = (q - 8.0) * 0.125
    blocks = nxq.int4_pack(km, np.full((K // gs, N), 0.125, np.float32), np.full((K // gs, N), 8.0, np.float32),
                           N, K, gs, nxq.INT4_KMAJOR)
    t = 100 + gs // 32
    assert loader.same_bits(loader.dequant(t, blocks, N * K), w_shader.reshape(-1))
    x = rng.standard_normal((1, K)).astype(np.float32)
    y = loader.qmatmul(t, blocks, N, K, x)
    want = (x.astype(np.float64) @ w_shader.astype(np.float64).T)
    assert synth.rel_l2(y, want) < 1e-6


def test_pack_errors():
    c = np.zeros(64, np.uint8)
    s = np.ones(1, np.float32)
    out = np.zeros(72, np.uint8)
    L = nxq.lib()
    assert L.nxq_int4_pack(c.ctypes.data, s.ctypes.data, None, 1, 128, 48, 0, out.ctypes.data, 72) == -2
    assert L.nxq_int4_pack(c.ctypes.data, s.ctypes.data, None, 1, 96, 64, 0, out.ctypes.data, 72) == -3
    assert L.nxq_int4_pack(c.ctypes.data, s.ctypes.data, None, 1, 128, 128, 2, out.ctypes.data, 72) == -1
    assert L.nxq_int4_pack(c.ctypes.data, s.ctypes.data, None, 1, 128, 128, 0, out.ctypes.data, 71) == -3
    assert L.nxq_int4_pack(None, s.ctypes.data, None, 1, 128, 128, 0, out.ctypes.data, 72) == -1
    assert L.nxq_int4_pack(c.ctypes.data, s.ctypes.data, None, 1, 128, 128, 0, out.ctypes.data, 72) == 0


def _arrays(N, K, gs, seed):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 256, N * K // 2, dtype=np.uint8)
    sc = rng.uniform(1e-3, 5e-3, N * K // gs).astype(np.float32)
    z = rng.uniform(0.0, 15.0, N * K // gs).astype(np.float32)
    return codes, sc, z


@pytest.mark.gpu
@pytest.mark.parametrize("gs", GS)
@pytest.mark.parametrize("layout", ["rows", "kmajor"])
def test_register_decodes_bit_exact(gpu, gs, layout):
    N, K = 300, 1024
    codes, sc, z = _arrays(N, K, gs, seed=gs)
    ref = loader.dequant_int4(codes, sc, z, N * K, gs, which="ref" if loader.ref() else "port")
    if layout == "rows":
        w = gpu.Weight.register_int4(codes, sc, z, N, K, gs, gpu.INT4_ROWS)
    else:
        w = gpu.Weight.register_int4(*_to_kmajor(codes, sc, z, N, K, gs), N, K, gs, gpu.INT4_KMAJOR)
    try:
        assert loader.same_bits(w.dequant().cpu().numpy().reshape(-1), ref)
    finally:
        w.release()


@pytest.mark.gpu
@pytest.mark.parametrize("gs", GS)
def test_golden_matrix_on_gpu(gpu, gs):
    import torch

    g = _g()
    t = 100 + gs // 32
    mb, N, K = g[f"g{gs}_mat_blocks"], int(g[f"g{gs}_mat_N"]), int(g[f"g{gs}_mat_K"])
    w = gpu.Weight.register(mb, t, N, K)
    try:
        x = torch.from_numpy(g[f"g{gs}_mat_x"]).half().cuda()
        y = gpu.qmatmul(w, x)
        torch.cuda.synchronize()
        assert synth.rel_l2(y.cpu().numpy(), g[f"g{gs}_mat_y"]) < TOL
    finally:
        w.release()


@pytest.mark.gpu
@pytest.mark.parametrize("gs,M,kernel", [(128, 1, "mma_gemv<I4G128,m8>"), (128, 8, "mma_gemv<I4G128,m8>"),
                                          (128, 32, "mma_gemv<I4G128,m32>"), (128, 300, "tc_gemm<I4G128,n256>"),
                                          (64, 4, "mma_gemv<I4G64,m8>"), (32, 20, "mma_gemv<I4G32,m32>"),
                                          (256, 2, "mma_gemv<I4G256,m8>"), (32, 40, "tc_gemm<I4G32,n256>"),
                                          (64, 100, "tc_gemm<I4G64,n256>"), (256, 64, "tc_gemm<I4G256,n256>")])
def test_matmul_paths(gpu, gs, M, kernel):
    import torch

    N, K = 1536, 2048
    codes, sc, z = _arrays(N, K, gs, seed=100 + gs)
    w = gpu.Weight.register_int4(codes, sc, z, N, K, gs)
    try:
        assert gpu.kernel_name(w, M).startswith(kernel)
        x = torch.from_numpy(synth.make_activations(M, K, seed=M)).cuda()
        y = gpu.qmatmul(w, x)
        torch.cuda.synchronize()
        blocks = nxq.int4_pack(codes, sc, z, N, K, gs)
        want = loader.qmatmul(100 + gs // 32, blocks, N, K, x.float().cpu().numpy())
        assert synth.rel_l2(y.cpu().numpy(), want) < TOL
    finally:
        w.release()
