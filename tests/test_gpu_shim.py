"""GPU: the compiled C++ shim with the engine's operator signatures
(ComputeDispatch::gemm_int4 / gemv_int4, compute_dispatch.h:47-61) over
libnxq.so, driven by a small C++ program (tests/shim/shim_check.cpp) built
here against nxq/libnxq_dispatch.so.

gemm_int4 takes the reference's scale-less INT4 weights in the GEMV shader's
[K/2][N] byte order, w = (q - 8) * 0.125 (gemv_int4_nr8.metal:31-80);
gemv_int4 the NXF INT4 codec's codes, scales and zeros in the K-major order
(gemm_dequant.metal:29-70).  The oracle decodes those formulas exactly on the
CPU and multiplies in fp32 (loader's fp32 GEMM); bar rel-L2 <= 1e-3.  The
shim's error behaviour: an exception by default, the reference's zero-fill
(compute_dispatch.cpp:174-176) when opted in."""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

from nxq import synth

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "nexus-inference-engine-_b200"
TOL = 1e-3


@pytest.fixture(scope="module")
def shim_exe(tmp_path_factory):
    lib_dir = PKG / "nxq"
    assert (lib_dir / "libnxq_dispatch.so").exists(), "build.py builds the shim library"
    exe = tmp_path_factory.mktemp("shim") / "shim_check"
    subprocess.run(["g++", "-std=c++17", "-O1", "-o", str(exe), str(ROOT / "tests" / "shim" / "shim_check.cpp"),
                    f"-I{ROOT / 'include'}", f"-I{PKG / 'shim'}", f"-L{lib_dir}", "-lnxq_dispatch", "-lnxq",
                    f"-Wl,-rpath,{lib_dir}"], check=True)
    return exe


def _run(exe, mode, d):
    r = subprocess.run([str(exe), mode, str(d)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    return r.stdout


def _fp32_matmul(x, w):
    from oracle import loader

    M, K = x.shape
    N = w.shape[0]
    y = np.zeros((M, N), np.float32)
    loader.port().nxqo_gemm_transb(np.ascontiguousarray(x, np.float32).ctypes.data,
                                   np.ascontiguousarray(w, np.float32).ctypes.data, y.ctypes.data, M, N, K, os.cpu_count() or 1)
    return y


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (5, 1000, 768), (40, 512, 2048)])
def test_shim_gemm_int4_scaleless(gpu, shim_exe, tmp_path, M, N, K):
    g = synth.rng(M + N + K)
    wq = g.integers(0, 256, size=(K // 2, N), dtype=np.uint8)
    x = g.standard_normal((M, K), dtype=np.float32)
    lo = (wq & 15).astype(np.float32) - 8.0
    hi = (wq >> 4).astype(np.float32) - 8.0
    w = np.empty((K, N), np.float32)
    w[0::2], w[1::2] = lo * 0.125, hi * 0.125
    want = _fp32_matmul(x, w.T.copy())
    (tmp_path / "dims").write_text(f"{M} {N} {K} 0")
    x.tofile(tmp_path / "x.bin")
    wq.tofile(tmp_path / "w.bin")
    _run(shim_exe, "gemm", tmp_path)
    got = np.fromfile(tmp_path / "y.bin", np.float32).reshape(M, N)
    # fp32 activations are rounded to f16 by the tensor-core kernels.
    want16 = _fp32_matmul(x.astype(np.float16).astype(np.float32), w.T.copy())
    assert synth.rel_l2(got, want16) < TOL
    assert synth.rel_l2(got, want) < 2 * TOL


@pytest.mark.parametrize("gs", [64, 128])
def test_shim_gemv_int4_groups(gpu, shim_exe, tmp_path, gs):
    M, N, K = 3, 768, 1024
    g = synth.rng(gs)
    wq = g.integers(0, 256, size=(K // 2, N), dtype=np.uint8)
    sc = g.uniform(1e-3, 5e-3, size=(K // gs, N)).astype(np.float32)
    z = g.uniform(0.0, 15.0, size=(K // gs, N)).astype(np.float32)
    x = g.standard_normal((M, K), dtype=np.float32).astype(np.float16).astype(np.float32)
    q = np.empty((K, N), np.float32)
    q[0::2], q[1::2] = (wq & 15), (wq >> 4)
    grp = np.arange(K) // gs
    w = (q - z[grp]) * sc[grp]
    want = _fp32_matmul(x, w.T.copy())
    (tmp_path / "dims").write_text(f"{M} {N} {K} {gs}")
    x.tofile(tmp_path / "x.bin")
    wq.tofile(tmp_path / "w.bin")
    sc.tofile(tmp_path / "s.bin")
    z.tofile(tmp_path / "z.bin")
    _run(shim_exe, "gemv", tmp_path)
    got = np.fromfile(tmp_path / "y.bin", np.float32).reshape(M, N)
    assert synth.rel_l2(got, want) < TOL


def test_shim_error_behaviour(gpu, shim_exe, tmp_path):
    M, N, K = 2, 256, 512
    g = synth.rng(3)
    (tmp_path / "dims").write_text(f"{M} {N} {K} 0")
    g.standard_normal((M, K), dtype=np.float32).tofile(tmp_path / "x.bin")
    g.integers(0, 256, size=(K // 2, N), dtype=np.uint8).tofile(tmp_path / "w.bin")
    assert "errors ok" in _run(shim_exe, "errors", tmp_path)
