"""GPU: every kernel variant the benchmark times, at the full shapes of the
five BASELINE configurations, against the CPU oracle (the reference's
decoders + fp32 dot products).

The oracle runs on a sample of the output: a set of weight rows (output
columns) that includes the first and last row and both rows of several
128-row tile boundaries, for all tokens (decode), or a set of tokens for all
weight rows (prefill).  Calls are issued the way the benchmark issues them:
single calls, and CUDA graphs of back-to-back calls on different weights
(programmatic dependent launch lets a call start while the previous one
drains), on a side stream.

Bars as everywhere: rel-L2 <= 1e-3 for fp32 outputs; bf16 outputs are
compared with the unrounded oracle under rel-L2 <= 1e-3 + 2^-8 (the bf16
rounding of the stored value alone is up to 2^-9 relative per value)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import NAMES
from oracle import loader
from nxq import synth

pytestmark = pytest.mark.gpu

TOL = 1e-3
TOL_BF16 = 1e-3 + 2.0 ** -8
Q4_0, Q8_0, Q3_K, Q4_K = 2, 8, 11, 12


def _torch():
    import torch

    return torch


def sample_rows(N: int, n: int, seed: int) -> np.ndarray:
    """n weight rows: 0, N-1, the rows either side of four tile boundaries,
    and random others; sorted and unique."""
    g = synth.rng(seed)
    fixed = [0, N - 1]
    for b in (128, 256 * 3, N // 2 - N // 2 % 128, N - N % 128 - 128 if N > 256 else 128):
        if 0 < b < N:
            fixed += [b - 1, b]
    rest = g.choice(N, size=max(0, n - len(fixed)), replace=False)
    return np.unique(np.concatenate([np.array(fixed), rest]).astype(np.int64))


def oracle_rows(t: int, blocks: np.ndarray, N: int, K: int, x: np.ndarray, rows: np.ndarray) -> np.ndarray:
    """The oracle's y[:, rows] for y = x W^T: only the sampled rows' blocks
    are decoded."""
    qk, bb = synth.GEOMETRY[t]
    sub = blocks.reshape(N, (K // qk) * bb)[rows]
    return loader.qmatmul(t, sub, len(rows), K, x.astype(np.float32))


def _graph_calls(gpu, calls, stream):
    """Capture `calls` (weight, x, y) as one CUDA graph of back-to-back
    nxq_qmatmul launches on `stream` and replay it once."""
    torch = _torch()
    with torch.cuda.stream(stream):
        for w, x, y in calls:  # sizes the stream's scratch before capture
            gpu.qmatmul(w, x, out=y, stream=stream)
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for w, x, y in calls:
            gpu.qmatmul(w, x, out=y, stream=stream)
    for _, _, y in calls:
        y.fill_(float("nan"))
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize()
    gpu.stream_sync(stream)
    del g


# ---- config 2: Q4_K GEMV, Llama-3-8B MLP, M in {1, 4, 8, 16, 32} ---------------
@pytest.mark.parametrize("shape", ["gate", "down"])
def test_config2_every_batch_size(gpu, shape):
    """gate/up (K=4096, N=14336) and down (K=14336, N=4096) at M = 1, 4, 8,
    16, 32: each M as a single call and, in one graph, all five back to back
    on two weight copies (the benchmark's step)."""
    torch = _torch()
    K, N = (4096, 14336) if shape == "gate" else (14336, 4096)
    blocks = synth.make_blocks(Q4_K, N, K, seed=1000 + K + N)
    rows = sample_rows(N, 1024, seed=N)
    ws = [gpu.Weight.register(blocks, Q4_K, N, K) for _ in range(2)]
    stream = torch.cuda.Stream()
    try:
        calls, wants = [], []
        for i, M in enumerate((1, 4, 8, 16, 32)):
            xh = synth.make_activations(M, K, seed=M * 7 + K, dtype=np.float16)
            x = torch.from_numpy(xh).cuda()
            want = oracle_rows(Q4_K, blocks, N, K, xh, rows)
            y = gpu.qmatmul(ws[0], x)
            torch.cuda.synchronize()
            gpu.stream_sync()
            assert synth.rel_l2(y.cpu().numpy()[:, rows], want) < TOL, (shape, M)
            calls.append((ws[i % 2], x, torch.empty(M, N, device="cuda")))
            wants.append(want)
        _graph_calls(gpu, calls, stream)
        for (_, x, y), want in zip(calls, wants):
            assert synth.rel_l2(y.cpu().numpy()[:, rows], want) < TOL, (shape, x.shape[0], "graph")
    finally:
        for w in ws:
            w.release()


# ---- config 1: Q4_0 GEMV, M=1, 4096 x 4096, fp32 x ------------------------------
def test_config1_fp32_activations(gpu):
    torch = _torch()
    N = K = 4096
    blocks = synth.make_blocks(Q4_0, N, K, seed=1001)
    ws = [gpu.Weight.register(blocks, Q4_0, N, K) for _ in range(3)]
    stream = torch.cuda.Stream()
    try:
        x32 = torch.randn(1, K, generator=torch.Generator().manual_seed(11), dtype=torch.float32)
        want = loader.qmatmul(Q4_0, blocks, N, K, x32.numpy())
        y = gpu.qmatmul(ws[0], x32.cuda())
        torch.cuda.synchronize()
        gpu.stream_sync()
        assert synth.rel_l2(y.cpu().numpy(), want) < TOL
        calls = [(w, x32.cuda(), torch.empty(1, N, device="cuda")) for w in ws]
        _graph_calls(gpu, calls, stream)
        for _, _, y in calls:
            assert synth.rel_l2(y.cpu().numpy(), want) < TOL
    finally:
        for w in ws:
            w.release()


# ---- config 3: Q8_0 GEMV M=1 over a Llama-3-8B layer -----------------------------
CONFIG3 = [("q", 4096, 4096), ("k", 4096, 1024), ("v", 4096, 1024), ("o", 4096, 4096),
           ("gate", 4096, 14336), ("up", 4096, 14336), ("down", 14336, 4096)]  # name, K, N


@pytest.fixture(scope="module")
def config3_layer(gpu):
    layer = {}
    for i, (name, K, N) in enumerate(CONFIG3):
        blocks = synth.make_blocks(Q8_0, N, K, seed=3000 + i)
        layer[name] = (blocks, gpu.Weight.register(blocks, Q8_0, N, K), K, N)
    yield layer
    for _, w, _, _ in layer.values():
        w.release()


def test_config3_each_projection_and_the_layer_graph(gpu, config3_layer):
    """All 7 projections as single calls and as the benchmark's layer graph
    (7 launches back to back)."""
    torch = _torch()
    xs = {K: torch.randn(1, K, generator=torch.Generator().manual_seed(K), dtype=torch.float32).to(torch.float16)
          for K in (4096, 14336)}
    calls, wants = [], []
    for name, K, N in CONFIG3:
        blocks, w, _, _ = config3_layer[name]
        want = loader.qmatmul(Q8_0, blocks, N, K, xs[K].float().numpy())
        y = gpu.qmatmul(w, xs[K].cuda())
        torch.cuda.synchronize()
        gpu.stream_sync()
        assert synth.rel_l2(y.cpu().numpy(), want) < TOL, name
        calls.append((w, xs[K].cuda(), torch.empty(1, N, device="cuda")))
        wants.append(want)
    _graph_calls(gpu, calls, torch.cuda.Stream())
    for (_, _, y), want, (name, _, _) in zip(calls, wants, CONFIG3):
        assert synth.rel_l2(y.cpu().numpy(), want) < TOL, (name, "graph")


def test_config3_grouped_and_fused_layer(gpu, config3_layer):
    """The two other layer forms the benchmark times: q/k/v and gate/up as
    grouped launches; and RMSNorm + q/k/v, o + residual, gate/up + SwiGLU,
    down + residual."""
    torch = _torch()
    L = config3_layer
    x = torch.randn(1, 4096, generator=torch.Generator().manual_seed(4096), dtype=torch.float32).to(torch.float16)
    xd = x.cuda()
    ys = gpu.qmatmul_grouped([L[n][1] for n in ("q", "k", "v", "gate", "up")], [xd] * 5)
    torch.cuda.synchronize()
    gpu.stream_sync()
    for n, y in zip(("q", "k", "v", "gate", "up"), ys):
        blocks, _, K, N = L[n]
        assert synth.rel_l2(y.cpu().numpy(), loader.qmatmul(Q8_0, blocks, N, K, x.float().numpy())) < TOL, n

    # Fused forms against the oracle composed on the CPU.
    resid = torch.randn(1, 4096, generator=torch.Generator().manual_seed(7), dtype=torch.float32)
    normw = torch.rand(4096, generator=torch.Generator().manual_seed(8), dtype=torch.float32).add_(0.5)
    r = 1.0 / np.sqrt((resid.double().numpy() ** 2).mean() + 1e-5)
    xn = torch.from_numpy((resid.numpy() * np.float32(r) * normw.numpy()).astype(np.float32)).to(torch.float16)
    outs = gpu.rmsnorm_qmatmul([L[n][1] for n in ("q", "k", "v")], resid.cuda(), normw.cuda(), 1e-5)
    torch.cuda.synchronize()
    gpu.stream_sync()
    for n, y in zip(("q", "k", "v"), outs):
        blocks, _, K, N = L[n]
        assert synth.rel_l2(y.cpu().numpy(), loader.qmatmul(Q8_0, blocks, N, K, xn.float().numpy())) < TOL, n
    res_d = resid.cuda()
    y = gpu.qmatmul_residual(L["o"][1], xd, res_d)
    h = gpu.qmatmul_swiglu(L["gate"][1], L["up"][1], xd, out_dtype=torch.float32)
    torch.cuda.synchronize()
    gpu.stream_sync()
    bo, _, K, N = L["o"]
    want_o = loader.qmatmul(Q8_0, bo, N, K, x.float().numpy()) + resid.numpy()
    assert synth.rel_l2(y.cpu().numpy(), want_o) < TOL
    g = loader.qmatmul(Q8_0, L["gate"][0], 14336, 4096, x.float().numpy()).astype(np.float64)
    u = loader.qmatmul(Q8_0, L["up"][0], 14336, 4096, x.float().numpy()).astype(np.float64)
    assert synth.rel_l2(h.cpu().numpy(), g / (1.0 + np.exp(-g)) * u) < TOL
    hh = h.to(torch.float16)
    yd = gpu.qmatmul_residual(L["down"][1], hh, res_d)
    torch.cuda.synchronize()
    gpu.stream_sync()
    bd, _, K, N = L["down"]
    want_d = loader.qmatmul(Q8_0, bd, N, K, hh.float().cpu().numpy()) + resid.numpy()
    assert synth.rel_l2(yd.cpu().numpy(), want_d) < TOL


# ---- config 4: Q4_K prefill GEMM, bf16 in and out -------------------------------
@pytest.mark.parametrize("M", [512, 2048, 8192])
def test_config4_prefill_bf16_output(gpu, M):
    """The benchmarked variant: bf16 activations, bf16 output, K=4096,
    N=14336; sampled tokens (first and last of several 256-token tiles and
    random ones) against the oracle over all N columns."""
    torch = _torch()
    K, N = 4096, 14336
    blocks = synth.make_blocks(Q4_K, N, K, seed=4000)
    w = gpu.Weight.register(blocks, Q4_K, N, K)
    try:
        assert gpu.kernel_name(w, M, gpu.BF16, gpu.BF16).startswith("tc_gemm<")
        x = torch.randn(M, K, generator=torch.Generator().manual_seed(M), dtype=torch.float32).to(torch.bfloat16)
        y = gpu.qmatmul(w, x.cuda(), out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        gpu.stream_sync()
        toks = sample_rows(M, 12, seed=M)
        want = loader.qmatmul(Q4_K, blocks, N, K, x[toks].float().numpy())
        got = y.float().cpu().numpy()[toks]
        assert synth.rel_l2(got, want) < TOL_BF16
        # fp32 output of the same call: the parity bar itself.
        y32 = gpu.qmatmul(w, x.cuda(), out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert synth.rel_l2(y32.cpu().numpy()[toks], want) < TOL
        # bf16 output equals the fp32 output rounded to bf16 (same sums).
        assert torch.equal(y32.to(torch.bfloat16).cpu(), y.cpu())
    finally:
        w.release()


# ---- config 5: Q3_K 405B-shaped layer, M in {1, 8, 32} ---------------------------
CONFIG5 = [("q/o", 16384, 16384), ("k/v", 16384, 1024), ("gate/up", 16384, 53248), ("down", 53248, 16384)]


@pytest.mark.parametrize("name,K,N", CONFIG5, ids=[c[0] for c in CONFIG5])
def test_config5_projections(gpu, name, K, N):
    """Every projection shape of the 405B-shaped Q3_K layer (TP=1) at M = 1,
    8, 32, single calls and one graph of the three."""
    torch = _torch()
    blocks = synth.make_blocks(Q3_K, N, K, seed=5000 + K + N)
    rows = sample_rows(N, 512, seed=K + N)
    w = gpu.Weight.register(blocks, Q3_K, N, K)
    stream = torch.cuda.Stream()
    try:
        calls, wants = [], []
        for M in (1, 8, 32):
            xh = synth.make_activations(M, K, seed=M + K, dtype=np.float16)
            x = torch.from_numpy(xh).cuda()
            want = oracle_rows(Q3_K, blocks, N, K, xh, rows)
            y = gpu.qmatmul(w, x)
            torch.cuda.synchronize()
            gpu.stream_sync()
            assert synth.rel_l2(y.cpu().numpy()[:, rows], want) < TOL, (name, M)
            calls.append((w, x, torch.empty(M, N, device="cuda")))
            wants.append(want)
        _graph_calls(gpu, calls, stream)
        for (_, x, y), want in zip(calls, wants):
            assert synth.rel_l2(y.cpu().numpy()[:, rows], want) < TOL, (name, x.shape[0], "graph")
    finally:
        w.release()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_config5_tp_shards_on_one_gpu(gpu, world):
    """The tensor-parallel shards of the config-5 down projection (row split,
    K/world of every row) and gate projection (column split) at every TP
    degree, computed on one GPU: the column shards' outputs concatenate to
    the full product, the row shards' partial outputs sum to it."""
    torch = _torch()
    M = 8
    for name, K, N, split in (("gate", 16384, 53248, gpu.SPLIT_COL), ("down", 53248, 16384, gpu.SPLIT_ROW)):
        blocks = synth.make_blocks(Q3_K, N, K, seed=5100 + K)
        rows = sample_rows(N, 256, seed=K)
        xh = synth.make_activations(M, K, seed=K, dtype=np.float16)
        want = oracle_rows(Q3_K, blocks, N, K, xh, rows)
        x = torch.from_numpy(xh).cuda()
        parts = []
        for r in range(world):
            w = gpu.Weight.register_shard(blocks, Q3_K, N, K, split, r, world)
            try:
                if split == gpu.SPLIT_COL:
                    parts.append(gpu.qmatmul(w, x).cpu().numpy())
                else:
                    ks = K // world
                    parts.append(gpu.qmatmul(w, x[:, r * ks:(r + 1) * ks].contiguous()).cpu().numpy())
                gpu.stream_sync()
            finally:
                w.release()
        full = np.concatenate(parts, axis=1) if split == gpu.SPLIT_COL else np.sum(parts, axis=0)
        assert synth.rel_l2(full[:, rows], want) < TOL, (name, world)
