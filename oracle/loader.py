"""Test infrastructure: ctypes access to the CPU oracle libraries.

  port : oracle/libnxq_oracle.so, the plain-C restatement (nxq_oracle.c)
  ref  : oracle/_ref/libref_decoders.so, the reference's own decoders compiled
         from nexus/src/import/gguf_importer.cpp (oracle/Makefile); present
         where it was built (this container, and snapshots of it)

Both decode GGUF blocks to fp32; nxqo_qmatmul runs the reference CPU path
(row-streamed decode, then fp32 dot products) with either decoder.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_SO = HERE / "libnxq_oracle.so"
REF_SO = HERE / "_ref" / "libref_decoders.so"

_port: Optional[ctypes.CDLL] = None
_ref: Optional[ctypes.CDLL] = None


def build(ref: bool = True) -> None:
    """make -C oracle port [ref]; the ref target only where the reference exists."""
    targets = ["port"]
    default_ref = HERE.parent.parent / "reference" / "nexus"  # the checkout beside this repository
    if ref and Path(os.environ.get("NXQ_REFERENCE", str(default_ref)), "src").exists():
        targets.append("ref")
    env = dict(os.environ)
    if "NXQ_REFERENCE" in os.environ:
        env["REF"] = os.environ["NXQ_REFERENCE"]
    subprocess.run(["make", "-s", "-C", str(HERE), *targets], check=True, env=env)


def port() -> ctypes.CDLL:
    global _port
    if _port is None:
        if not PORT_SO.exists():
            build(ref=False)
        L = ctypes.CDLL(str(PORT_SO))
        L.nxqo_dequant.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        L.nxqo_dequant.restype = ctypes.c_int
        L.nxqo_half_to_float.argtypes = [ctypes.c_uint16]
        L.nxqo_half_to_float.restype = ctypes.c_float
        L.nxqo_qmatmul.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64,
                                   ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                   ctypes.c_int]
        L.nxqo_qmatmul.restype = ctypes.c_int
        L.nxqo_gemm_transb.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int]
        L.nxqo_gemm_transb.restype = None
        L.nxqo_dequant_int4.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_int64, ctypes.c_int]
        L.nxqo_dequant_int4.restype = None
        _port = L
    return _port


def ref() -> Optional[ctypes.CDLL]:
    """The reference's compiled decoders, or None where they were not built."""
    global _ref
    if _ref is None and REF_SO.exists():
        L = ctypes.CDLL(str(REF_SO))
        L.ref_dequant.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
        L.ref_dequant.restype = ctypes.c_int
        L.ref_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.ref_fp16_to_fp32.restype = ctypes.c_float
        L.ref_dequant_int4.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_int, ctypes.c_int]
        L.ref_dequant_int4.restype = None
        _ref = L
    return _ref


def dequant(type_id: int, blocks: np.ndarray, n: int, which: str = "port") -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.zeros(n, dtype=np.float32)
    if which == "ref":
        L = ref()
        if L is None:
            raise FileNotFoundError(REF_SO)
        rc = L.ref_dequant(type_id, blocks.ctypes.data, n, out.ctypes.data)
    else:
        rc = port().nxqo_dequant(type_id, blocks.ctypes.data, n, out.ctypes.data)
    if rc != 0:
        raise ValueError(f"oracle dequant failed for type {type_id}")
    return out


def qmatmul(type_id: int, blocks: np.ndarray, N: int, K: int, x: np.ndarray, which: str = "port",
            nthreads: int = 0) -> np.ndarray:
    """The reference CPU path: y[M][N] = x[M][K] (fp32) times decode(W)^T."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    M = x.shape[0]
    y = np.zeros((M, N), dtype=np.float32)
    dec = None
    if which == "ref":
        L = ref()
        if L is None:
            raise FileNotFoundError(REF_SO)
        dec = ctypes.cast(L.ref_dequant, ctypes.c_void_p)
    nt = nthreads or (os.cpu_count() or 1)
    rc = port().nxqo_qmatmul(dec, type_id, blocks.ctypes.data, N, K, x.ctypes.data, M,
                             y.ctypes.data, nt)
    if rc != 0:
        raise ValueError("oracle qmatmul failed")
    return y


def dequant_int4(codes: np.ndarray, scales: np.ndarray, zeros, n: int, group_size: int,
                 which: str = "port") -> np.ndarray:
    """quant/gptq.cpp:9-27 over flat arrays: the oracle's restatement ("port")
    or the reference's own compiled function ("ref")."""
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    zp = None if zeros is None else np.ascontiguousarray(zeros, dtype=np.float32)
    out = np.zeros(n, dtype=np.float32)
    if which == "ref":
        L = ref()
        if L is None:
            raise FileNotFoundError(REF_SO)
        L.ref_dequant_int4(out.ctypes.data, codes.ctypes.data, scales.ctypes.data,
                           None if zp is None else zp.ctypes.data, n, group_size)
    else:
        port().nxqo_dequant_int4(out.ctypes.data, codes.ctypes.data, scales.ctypes.data,
                                 None if zp is None else zp.ctypes.data, ctypes.c_int64(n), group_size)
    return out


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    """Bit-identical float arrays, with any NaN matching any NaN (NaN payloads
    depend on operand order chosen by the compiler, not on the decoder)."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    if not np.array_equal(na, nb):
        return False
    return bool(np.array_equal(a.view(np.uint32)[~na], b.view(np.uint32)[~nb]))
