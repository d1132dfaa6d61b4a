"""GPU: the fused epilogues against the oracle.

nxq_qmatmul_swiglu: h = silu(x Wg^T) * (x Wu^T), silu(g) = g / (1 + exp(-g)),
with the oracle's fp32 products combined in float64; one launch for decode
batch sizes (a row tile's gate and up units in one run, tiles shared between
CTAs finished by one of them), otherwise gate/up then a small kernel (prefill
batch sizes).
nxq_qmatmul_residual: y = x W^T + res, fused into the decode kernel's store,
after the product otherwise; in place (y is the residual buffer) and not.
Tolerance: rel-L2 <= 1e-3 (the parity bar) for fp32 outputs.  A bf16 output
is compared with the unrounded oracle under rel-L2 <= 1e-3 + 2^-8: storing in
bf16 alone adds up to half an ulp (2^-9 relative) per value, and comparing two
bf16 roundings instead would count whole-ulp flips of values the matmul moved
by less than 1e-3 (SwiGLU multiplies two such values)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import NAMES
from oracle import loader
from nxq import synth

pytestmark = pytest.mark.gpu

TOL = 1e-3
TOL_BF16 = 1e-3 + 2.0 ** -8


def _torch():
    import torch

    return torch


def _silu_mul(g, u):
    g = g.astype(np.float64)
    return g / (1.0 + np.exp(-g)) * u.astype(np.float64)


def _pair(gpu, t, N, K, seed):
    bg = synth.make_blocks(t, N, K, seed=seed)
    bu = synth.make_blocks(t, N, K, seed=seed + 1)
    return bg, bu, gpu.Weight.register(bg, t, N, K), gpu.Weight.register(bu, t, N, K)


@pytest.mark.parametrize("t", [12, 11, 8], ids=lambda t: NAMES[t])
@pytest.mark.parametrize("M", [1, 4, 16, 32])
@pytest.mark.parametrize("N,K", [(9728, 512), (1024, 2048)])
def test_swiglu_fused_one_launch(gpu, t, M, N, K):
    torch = _torch()
    bg, bu, wg, wu = _pair(gpu, t, N, K, seed=40 + M)
    try:
        x = torch.from_numpy(synth.make_activations(M, K, seed=M)).cuda()
        gpu.qmatmul_swiglu(wg, wu, x)  # warm-up
        torch.cuda.synchronize()
        n0 = gpu.launch_count()
        h = gpu.qmatmul_swiglu(wg, wu, x)
        n1 = gpu.launch_count()
        torch.cuda.synchronize()
        assert n1 - n0 == 1
        xf = x.float().cpu().numpy()
        want = _silu_mul(loader.qmatmul(t, bg, N, K, xf), loader.qmatmul(t, bu, N, K, xf))
        assert synth.rel_l2(h.cpu().numpy(), want) < TOL
    finally:
        wg.release()
        wu.release()


@pytest.mark.parametrize("N,K,M,out", [(512, 1024, 3, "f32"), (512, 1024, 40, "f32"), (9728, 512, 2, "bf16"),
                                       (1024, 256, 1, "bf16")])
def test_swiglu_other_paths(gpu, N, K, M, out):
    torch = _torch()
    t = 12
    bg, bu, wg, wu = _pair(gpu, t, N, K, seed=60)
    try:
        x = torch.from_numpy(synth.make_activations(M, K, seed=7)).cuda()
        dt = torch.float32 if out == "f32" else torch.bfloat16
        h = gpu.qmatmul_swiglu(wg, wu, x, out_dtype=dt)
        torch.cuda.synchronize()
        xf = x.float().cpu().numpy()
        want = _silu_mul(loader.qmatmul(t, bg, N, K, xf), loader.qmatmul(t, bu, N, K, xf))
        assert synth.rel_l2(h.float().cpu().numpy(), want) < (TOL if out == "f32" else TOL_BF16)
    finally:
        wg.release()
        wu.release()


@pytest.mark.parametrize("t", [12, 11, 8, 2], ids=lambda t: NAMES[t])
@pytest.mark.parametrize("M", [1, 8, 32, 40])
@pytest.mark.parametrize("inplace", [False, True])
def test_residual(gpu, t, M, inplace):
    torch = _torch()
    N, K = 1024, 1024
    b = synth.make_blocks(t, N, K, seed=90 + M)
    w = gpu.Weight.register(b, t, N, K)
    try:
        x = torch.from_numpy(synth.make_activations(M, K, seed=M)).cuda()
        res = torch.from_numpy(synth.make_activations(M, N, seed=500 + M).astype(np.float32)).cuda()
        res0 = res.cpu().numpy().astype(np.float64)
        y = gpu.qmatmul_residual(w, x, res, out=res if inplace else None)
        torch.cuda.synchronize()
        want = loader.qmatmul(t, b, N, K, x.float().cpu().numpy()).astype(np.float64) + res0
        assert synth.rel_l2(y.cpu().numpy(), want) < TOL
    finally:
        w.release()


@pytest.mark.parametrize("M", [1, 8, 32])
def test_residual_shared_tiles(gpu, M):
    """A weight with more row tiles than SMs: tiles shared between CTAs get the
    residual once, from the CTA that finishes them."""
    torch = _torch()
    t, N, K = 12, 14336, 4096
    b = synth.make_blocks(t, N, K, seed=95)
    w = gpu.Weight.register(b, t, N, K)
    try:
        x = torch.from_numpy(synth.make_activations(M, K, seed=M)).cuda()
        res = torch.from_numpy(synth.make_activations(M, N, seed=600 + M).astype(np.float32)).cuda()
        want = loader.qmatmul(t, b, N, K, x.float().cpu().numpy()).astype(np.float64) + res.cpu().numpy()
        y = gpu.qmatmul_residual(w, x, res)
        torch.cuda.synchronize()
        assert synth.rel_l2(y.cpu().numpy(), want) < TOL
    finally:
        w.release()


def test_epilogue_errors(gpu):
    torch = _torch()
    t = 12
    wa = gpu.Weight.register(synth.make_blocks(t, 256, 512, seed=1), t, 256, 512)
    wb = gpu.Weight.register(synth.make_blocks(t, 512, 512, seed=2), t, 512, 512)
    try:
        x = torch.zeros(1, 512, dtype=torch.float16, device="cuda")
        h = torch.empty(1, 256, device="cuda")
        L = gpu.lib()
        assert L.nxq_qmatmul_swiglu(wa.handle, wb.handle, x.data_ptr(), 1, h.data_ptr(), 0, 1, None) == -3
        assert L.nxq_qmatmul_residual(wa.handle, x.data_ptr(), 1, None, h.data_ptr(), 0, 1, None) == -1
        assert L.nxq_qmatmul_swiglu(wa.handle, wa.handle, x.data_ptr(), 1, h.data_ptr(), 0, 0, None) == 0
    finally:
        wa.release()
        wb.release()


@pytest.mark.parametrize("M", [1, 4, 32, 40])
@pytest.mark.parametrize("xdt", ["f32", "bf16", "f16"])
def test_rmsnorm_prologue(gpu, M, xdt):
    """nxq_rmsnorm_qmatmul: y_i = (x * r * g) W_i^T, r = 1/sqrt(mean(x^2) + eps),
    against the normalization in float64 and the oracle matmul; two launches
    (normalization + one grouped GEMV) for decode batch sizes."""
    torch = _torch()
    t, K, eps = 11, 2048, 1e-6
    shapes = [(512, K), (128, K), (128, K)]
    blocks = [synth.make_blocks(t, N, K, seed=120 + i) for i, (N, _) in enumerate(shapes)]
    ws = [gpu.Weight.register(b, t, N, K) for b, (N, _) in zip(blocks, shapes)]
    try:
        rng = np.random.default_rng(M)
        x32 = (rng.standard_normal((M, K)) * 3.0 + 0.5).astype(np.float32)
        g32 = rng.uniform(0.5, 1.5, K).astype(np.float32)
        dt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[xdt]
        x = torch.from_numpy(x32).to(dt).cuda()
        g = torch.from_numpy(g32).cuda()
        gpu.rmsnorm_qmatmul(ws, x, g, eps)  # warm-up (scratch)
        torch.cuda.synchronize()
        n0 = gpu.launch_count()
        ys = gpu.rmsnorm_qmatmul(ws, x, g, eps)
        n1 = gpu.launch_count()
        torch.cuda.synchronize()
        if M <= 32:
            assert n1 - n0 == 2
        xin = x.float().cpu().numpy().astype(np.float64)
        xn = xin / np.sqrt((xin * xin).mean(axis=1, keepdims=True) + eps) * g32.astype(np.float64)
        for (N, _), b, y in zip(shapes, blocks, ys):
            want = loader.qmatmul(t, b, N, K, xn.astype(np.float32))
            assert synth.rel_l2(y.cpu().numpy(), want) < TOL
    finally:
        for w in ws:
            w.release()
