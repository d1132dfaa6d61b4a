"""ctypes binding of libnxq.so, the C ABI declared in include/nxq.h.

This is the Python face of the drop-in boundary for NEXUS's quantized-matmul
operator (``ComputeDispatch::gemm_int4``, nexus/src/compute/compute_dispatch.h:59-61):
weights are registered once and stay resident in HBM (``Weight``), activations
and outputs are torch CUDA tensors (``qmatmul``) or host numpy arrays
(``qmatmul_host``, the synchronous drop-in).  Every call goes through the CUDA
library; there is no CPU path, and importing fails loudly if the library is
missing.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path
from typing import Optional

import numpy as np

__all__ = [
    "NxqError", "lib", "init", "shutdown", "Weight", "qmatmul", "qmatmul_host", "stream_sync",
    "kernel_name", "launch_count",
    "TYPES", "GEOMETRY", "F32", "F16", "BF16", "SPLIT_COL", "SPLIT_ROW", "declared_symbols",
    "tp_unique_id", "tp_init", "tp_shutdown", "tp_qmatmul", "tp_allreduce_f32", "GGUF", "NXF", "xxh32", "qmatmul_grouped", "qmatmul_swiglu", "qmatmul_residual", "rmsnorm_qmatmul", "int4_pack", "INT4_ROWS", "INT4_KMAJOR",
]

LIB_PATH = Path(__file__).with_name("libnxq.so")
HEADER = Path(__file__).resolve().parents[2] / "include" / "nxq.h"

# GGUF type ids (nexus/src/import/gguf_importer.h:28-57) and block geometry
# (elements per block, bytes per block; gguf_importer.cpp:679-954).
TYPES = {"Q4_0": 2, "Q4_1": 3, "Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14,
         "I4G32": 101, "I4G64": 102, "I4G128": 104, "I4G256": 108,
         "NXF_I8": 120, "NXF_F16": 121, "NXF_F32": 122}
GEOMETRY = {2: (32, 18), 3: (32, 20), 8: (32, 34), 10: (256, 84), 11: (256, 110), 12: (256, 144),
            13: (256, 176), 14: (256, 210), 101: (32, 24), 102: (64, 40), 104: (128, 72), 108: (256, 136),
            120: (32, 32), 121: (32, 64), 122: (32, 128)}
# NXF INT4 group weights: array orders accepted by register_int4 / int4_pack.
INT4_ROWS, INT4_KMAJOR = 0, 1
F32, F16, BF16 = 0, 1, 2
SPLIT_COL, SPLIT_ROW = 0, 1

STATUS = {0: "OK", -1: "ERR_ARG", -2: "ERR_CODEC", -3: "ERR_SHAPE", -4: "ERR_CUDA",
          -5: "ERR_TIMEOUT", -6: "ERR_NOMEM", -7: "ERR_STATE", -8: "ERR_NCCL", -9: "ERR_UNSUPPORTED",
          -10: "ERR_FORMAT", -11: "ERR_RANGE"}


class NxqError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"nxq {STATUS.get(code, code)}: {message}")
        self.code = code
        self.name = STATUS.get(code, str(code))


_lib: Optional[ctypes.CDLL] = None

_c = ctypes
_SIGS = {
    "nxq_init": [_c.c_int],
    "nxq_shutdown": [],
    "nxq_last_error": [_c.c_char_p, _c.c_size_t],
    "nxq_abi_version": [],
    "nxq_block_geometry": [_c.c_int, _c.POINTER(_c.c_int), _c.POINTER(_c.c_int)],
    "nxq_weight_register": [_c.c_void_p, _c.c_size_t, _c.c_int, _c.c_int64, _c.c_int64,
                            _c.POINTER(_c.c_void_p)],
    "nxq_weight_register_device": [_c.c_void_p, _c.c_size_t, _c.c_int, _c.c_int64, _c.c_int64,
                                   _c.c_void_p, _c.POINTER(_c.c_void_p)],
    "nxq_weight_register_shard": [_c.c_void_p, _c.c_size_t, _c.c_int, _c.c_int64, _c.c_int64,
                                  _c.c_int, _c.c_int, _c.c_int, _c.POINTER(_c.c_void_p)],
    "nxq_shard_extract": [_c.c_void_p, _c.c_size_t, _c.c_int, _c.c_int64, _c.c_int64, _c.c_int,
                          _c.c_int, _c.c_int, _c.c_void_p, _c.c_size_t],
    "nxq_weight_release": [_c.c_void_p],
    "nxq_int4_pack": [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int, _c.c_int,
                      _c.c_void_p, _c.c_size_t],
    "nxq_weight_register_int4": [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int, _c.c_int,
                                 _c.POINTER(_c.c_void_p)],
    "nxq_weight_info": [_c.c_void_p, _c.POINTER(_c.c_int), _c.POINTER(_c.c_int64),
                        _c.POINTER(_c.c_int64), _c.POINTER(_c.c_size_t), _c.POINTER(_c.c_size_t)],
    "nxq_dequant": [_c.c_void_p, _c.c_void_p, _c.c_void_p],
    "nxq_qmatmul": [_c.c_void_p, _c.c_void_p, _c.c_int, _c.c_void_p, _c.c_int, _c.c_int64,
                    _c.c_void_p],
    "nxq_qmatmul_host": [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int64],
    "nxq_qmatmul_grouped": [_c.POINTER(_c.c_void_p), _c.c_int, _c.POINTER(_c.c_void_p), _c.c_int,
                            _c.POINTER(_c.c_void_p), _c.c_int, _c.POINTER(_c.c_int64), _c.c_void_p],
    "nxq_qmatmul_swiglu": [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int, _c.c_void_p, _c.c_int, _c.c_int64,
                           _c.c_void_p],
    "nxq_qmatmul_residual": [_c.c_void_p, _c.c_void_p, _c.c_int, _c.c_void_p, _c.c_void_p, _c.c_int, _c.c_int64,
                             _c.c_void_p],
    "nxq_rmsnorm_qmatmul": [_c.POINTER(_c.c_void_p), _c.c_int, _c.c_void_p, _c.c_int, _c.c_void_p, _c.c_float,
                            _c.POINTER(_c.c_void_p), _c.c_int, _c.c_int64, _c.c_void_p],
    "nxq_qmatmul_noalloc": [_c.c_void_p, _c.c_void_p, _c.c_int, _c.c_void_p, _c.c_int, _c.c_int64,
                            _c.c_void_p],
    "nxq_stream_sync": [_c.c_void_p],
    "nxq_set_wait_limit": [_c.c_uint64],
    "nxq_test_hook": [_c.c_int, _c.c_int],
    "nxq_tp_wait": [_c.c_void_p, _c.c_int64],
    "nxq_tp_p2p_enabled": [_c.c_void_p],
    "nxq_tp_test_hook": [_c.c_int, _c.c_int],
    "nxq_qmatmul_kernel_name": [_c.c_void_p, _c.c_int64, _c.c_int, _c.c_int, _c.c_char_p, _c.c_size_t],
    "nxq_launch_count": [_c.POINTER(_c.c_uint64)],
    "nxq_tp_unique_id_size": [],
    "nxq_tp_unique_id": [_c.c_void_p, _c.c_size_t],
    "nxq_tp_init": [_c.c_int, _c.c_int, _c.c_void_p, _c.c_size_t],
    "nxq_tp_shutdown": [],
    "nxq_tp_qmatmul": [_c.c_void_p, _c.c_void_p, _c.c_int, _c.c_void_p, _c.c_int, _c.c_int64,
                       _c.c_int, _c.c_void_p],
    "nxq_tp_allreduce_f32": [_c.c_void_p, _c.c_int64, _c.c_void_p],
    "nxq_gguf_open": [_c.c_char_p, _c.POINTER(_c.c_void_p)],
    "nxq_gguf_close": [_c.c_void_p],
    "nxq_gguf_header": [_c.c_void_p, _c.POINTER(_c.c_uint32), _c.POINTER(_c.c_uint64), _c.POINTER(_c.c_uint64)],
    "nxq_gguf_tensor_count": [_c.c_void_p, _c.POINTER(_c.c_int64)],
    "nxq_gguf_tensor_info": [_c.c_void_p, _c.c_int64, _c.c_char_p, _c.c_size_t, _c.POINTER(_c.c_int),
                             _c.POINTER(_c.c_int), _c.POINTER(_c.c_int64), _c.POINTER(_c.c_uint64),
                             _c.POINTER(_c.c_uint64)],
    "nxq_gguf_find": [_c.c_void_p, _c.c_char_p, _c.POINTER(_c.c_int64)],
    "nxq_gguf_tensor_data": [_c.c_void_p, _c.c_int64, _c.POINTER(_c.c_void_p), _c.POINTER(_c.c_uint64)],
    "nxq_gguf_meta_count": [_c.c_void_p, _c.POINTER(_c.c_int64)],
    "nxq_gguf_meta_key": [_c.c_void_p, _c.c_int64, _c.c_char_p, _c.c_size_t, _c.POINTER(_c.c_int)],
    "nxq_gguf_meta_uint": [_c.c_void_p, _c.c_char_p, _c.POINTER(_c.c_uint64)],
    "nxq_gguf_meta_int": [_c.c_void_p, _c.c_char_p, _c.POINTER(_c.c_int64)],
    "nxq_gguf_meta_float": [_c.c_void_p, _c.c_char_p, _c.POINTER(_c.c_double)],
    "nxq_gguf_meta_string": [_c.c_void_p, _c.c_char_p, _c.c_char_p, _c.c_size_t],
    "nxq_gguf_meta_array": [_c.c_void_p, _c.c_char_p, _c.POINTER(_c.c_int), _c.POINTER(_c.c_uint64)],
    "nxq_gguf_register": [_c.c_void_p, _c.c_int64, _c.c_int64, _c.POINTER(_c.c_void_p)],
    "nxq_gguf_register_shard": [_c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int, _c.c_int, _c.c_int,
                                _c.POINTER(_c.c_void_p)],
    "nxq_nxf_open": [_c.c_char_p, _c.POINTER(_c.c_void_p)],
    "nxq_nxf_close": [_c.c_void_p],
    "nxq_nxf_tensor_count": [_c.c_void_p, _c.POINTER(_c.c_int64)],
    "nxq_nxf_tensor_info": [_c.c_void_p, _c.c_int64, _c.c_char_p, _c.c_size_t, _c.POINTER(_c.c_int),
                            _c.POINTER(_c.c_int), _c.POINTER(_c.c_int64), _c.POINTER(_c.c_int64),
                            _c.POINTER(_c.c_int), _c.POINTER(_c.c_int), _c.POINTER(_c.c_uint64)],
    "nxq_nxf_chunk_info": [_c.c_void_p, _c.c_int64, _c.c_int64, _c.POINTER(_c.c_uint64), _c.POINTER(_c.c_uint32),
                           _c.POINTER(_c.c_uint32), _c.POINTER(_c.c_uint32), _c.POINTER(_c.c_int),
                           _c.POINTER(_c.c_int)],
    "nxq_nxf_find": [_c.c_void_p, _c.c_char_p, _c.POINTER(_c.c_int64)],
    "nxq_nxf_verify": [_c.c_void_p, _c.c_int64],
    "nxq_nxf_xxh32": [_c.c_void_p, _c.c_size_t, _c.POINTER(_c.c_uint32)],
    "nxq_nxf_manifest": [_c.c_void_p, _c.c_char_p, _c.c_size_t, _c.POINTER(_c.c_uint64)],
    "nxq_nxf_manifest_number": [_c.c_void_p, _c.c_char_p, _c.POINTER(_c.c_double)],
    "nxq_nxf_manifest_string": [_c.c_void_p, _c.c_char_p, _c.c_char_p, _c.c_size_t],
    "nxq_nxf_register": [_c.c_void_p, _c.c_int64, _c.c_int64, _c.POINTER(_c.c_void_p)],
    "nxq_nxf_register_shard": [_c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int, _c.c_int, _c.c_int,
                               _c.POINTER(_c.c_void_p)],
}


def lib() -> ctypes.CDLL:
    """Load libnxq.so (built by nexus-inference-engine-_b200/build.py)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: run `python nexus-inference-engine-_b200/build.py`")
        L = ctypes.CDLL(str(LIB_PATH))
        missing = [s for s in declared_symbols() if s not in _SIGS]
        if missing:
            raise ImportError(f"binding lacks signatures for {missing}")
        for name, args in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = ctypes.c_int
        _lib = L
    return _lib


_dispatch = None


def dispatch_lib() -> ctypes.CDLL:
    """Load the engine-side shim library libnxq_dispatch.so (built by build.py
    beside libnxq.so, which it links; the same instance as lib())."""
    global _dispatch
    if _dispatch is None:
        lib()
        path = LIB_PATH.with_name("libnxq_dispatch.so")
        if not path.exists():
            raise ImportError(f"{path} is missing: run `python nexus-inference-engine-_b200/build.py`")
        _dispatch = ctypes.CDLL(str(path))
    return _dispatch


def declared_symbols() -> list[str]:
    """Entry points declared in include/nxq.h (NXQ_API functions)."""
    text = HEADER.read_text()
    return re.findall(r"NXQ_API\s+int\s+(nxq_\w+)\s*\(", text)


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().nxq_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def _check(rc: int) -> None:
    if rc != 0:
        raise NxqError(rc, last_error())


def init(device: int = 0) -> None:
    _check(lib().nxq_init(device))


def shutdown() -> None:
    _check(lib().nxq_shutdown())


def _stream_ptr(stream) -> ctypes.c_void_p:
    if stream is None:
        import torch

        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return ctypes.c_void_p(stream)
    return ctypes.c_void_p(stream.cuda_stream)


def _dtype_code(t) -> int:
    import torch

    return {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}[t]


class Weight:
    """HBM-resident packed weight [N][K] of GGUF blocks of `type`."""

    def __init__(self, handle: int, type_id: int, N: int, K: int):
        self._h = ctypes.c_void_p(handle)
        self.type = type_id
        self.N = N
        self.K = K

    @staticmethod
    def _type_id(type_) -> int:
        return TYPES[type_] if isinstance(type_, str) else int(type_)

    @classmethod
    def register(cls, blocks, type_, N: int, K: int) -> "Weight":
        t = cls._type_id(type_)
        buf = np.ascontiguousarray(np.frombuffer(memoryview(blocks).cast("B"), dtype=np.uint8))
        h = ctypes.c_void_p()
        _check(lib().nxq_weight_register(buf.ctypes.data, buf.nbytes, t, N, K, ctypes.byref(h)))
        return cls(h.value, t, N, K)

    @classmethod
    def register_device(cls, blocks_tensor, type_, N: int, K: int, stream=None) -> "Weight":
        t = cls._type_id(type_)
        h = ctypes.c_void_p()
        nbytes = blocks_tensor.numel() * blocks_tensor.element_size()
        _check(lib().nxq_weight_register_device(blocks_tensor.data_ptr(), nbytes, t, N, K,
                                                _stream_ptr(stream), ctypes.byref(h)))
        return cls(h.value, t, N, K)

    @classmethod
    def register_int4(cls, codes: np.ndarray, scales: np.ndarray, zeros, N: int, K: int, group_size: int,
                      layout: int = INT4_ROWS) -> "Weight":
        """NXF INT4 group weights from their arrays (nxq_weight_register_int4)."""
        codes = np.ascontiguousarray(codes, dtype=np.uint8)
        scales = np.ascontiguousarray(scales, dtype=np.float32)
        zp = None if zeros is None else np.ascontiguousarray(zeros, dtype=np.float32)
        h = ctypes.c_void_p()
        _check(lib().nxq_weight_register_int4(codes.ctypes.data, scales.ctypes.data,
                                              None if zp is None else zp.ctypes.data, N, K, group_size, layout,
                                              ctypes.byref(h)))
        return cls(h.value, 100 + group_size // 32, N, K)

    @classmethod
    def register_shard(cls, blocks, type_, N: int, K: int, split: int, rank: int, world: int) -> "Weight":
        t = cls._type_id(type_)
        buf = np.ascontiguousarray(np.frombuffer(memoryview(blocks).cast("B"), dtype=np.uint8))
        h = ctypes.c_void_p()
        _check(lib().nxq_weight_register_shard(buf.ctypes.data, buf.nbytes, t, N, K, split, rank,
                                               world, ctypes.byref(h)))
        n_loc = N // world if split == SPLIT_COL else N
        k_loc = K // world if split == SPLIT_ROW else K
        return cls(h.value, t, n_loc, k_loc)

    @property
    def handle(self) -> ctypes.c_void_p:
        if self._h is None or not self._h.value:
            raise NxqError(-1, "weight already released")
        return self._h

    def info(self) -> dict:
        t, n, k = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
        pb, db = ctypes.c_size_t(), ctypes.c_size_t()
        _check(lib().nxq_weight_info(self.handle, ctypes.byref(t), ctypes.byref(n), ctypes.byref(k),
                                     ctypes.byref(pb), ctypes.byref(db)))
        return {"type": t.value, "N": n.value, "K": k.value, "packed_bytes": pb.value,
                "device_bytes": db.value}

    @property
    def packed_bytes(self) -> int:
        return self.info()["packed_bytes"]

    def dequant(self, out=None, stream=None):
        import torch

        if out is None:
            out = torch.empty((self.N, self.K), dtype=torch.float32, device="cuda")
        _check(lib().nxq_dequant(self.handle, out.data_ptr(), _stream_ptr(stream)))
        return out

    def release(self) -> None:
        if self._h is not None and self._h.value:
            _check(lib().nxq_weight_release(self._h))
        self._h = None


def qmatmul(w: Weight, x, out=None, out_dtype=None, stream=None):
    """y[M][N] = x[M][K] W^T on the current (or given) stream; x is a CUDA tensor."""
    import torch

    assert x.is_cuda and x.is_contiguous() and x.shape[-1] == w.K
    M = x.numel() // w.K
    if out is None:
        out = torch.empty((M, w.N), dtype=out_dtype or torch.float32, device=x.device)
    _check(lib().nxq_qmatmul(w.handle, x.data_ptr(), _dtype_code(x.dtype), out.data_ptr(),
                             _dtype_code(out.dtype), M, _stream_ptr(stream)))
    return out


def int4_pack(codes: np.ndarray, scales: np.ndarray, zeros, N: int, K: int, group_size: int,
              layout: int = INT4_ROWS) -> np.ndarray:
    """NXF INT4 group arrays -> I4G blocks [N][K/gs] (host only, no GPU)."""
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    zp = None if zeros is None else np.ascontiguousarray(zeros, dtype=np.float32)
    out = np.zeros(N * (K // group_size) * (8 + group_size // 2), dtype=np.uint8)
    _check(lib().nxq_int4_pack(codes.ctypes.data, scales.ctypes.data, None if zp is None else zp.ctypes.data, N, K,
                               group_size, layout, out.ctypes.data, out.nbytes))
    return out


def qmatmul_grouped(ws, xs, outs=None, out_dtype=None, stream=None):
    """y_i = x_i W_i^T for every (W_i, x_i) in one decode launch per 16 weights
    when they allow it (one block type, M_i <= 32); `xs` may repeat one tensor.
    All activations share one dtype, all outputs another."""
    import torch

    ws, xs = list(ws), list(xs)
    assert len(ws) == len(xs)
    if outs is None:
        outs = [torch.empty((x.numel() // w.K, w.N), dtype=out_dtype or torch.float32, device=x.device)
                for w, x in zip(ws, xs)]
    n = len(ws)
    Ms = []
    for w, x, y in zip(ws, xs, outs):
        assert x.is_cuda and x.is_contiguous() and x.shape[-1] == w.K and x.dtype == xs[0].dtype
        assert y.dtype == outs[0].dtype and y.numel() == (x.numel() // w.K) * w.N
        Ms.append(x.numel() // w.K)
    arr = ctypes.c_void_p * max(n, 1)
    _check(lib().nxq_qmatmul_grouped(arr(*[w.handle.value for w in ws]), n, arr(*[x.data_ptr() for x in xs]),
                                     _dtype_code(xs[0].dtype) if n else F16,
                                     arr(*[y.data_ptr() for y in outs]),
                                     _dtype_code(outs[0].dtype) if n else F32,
                                     (ctypes.c_int64 * max(n, 1))(*Ms), _stream_ptr(stream)))
    return outs


def qmatmul_swiglu(w_gate: Weight, w_up: Weight, x, out=None, out_dtype=None, stream=None):
    """h = silu(x Wg^T) * (x Wu^T), silu(g) = g / (1 + exp(-g))."""
    import torch

    assert x.is_cuda and x.is_contiguous() and x.shape[-1] == w_gate.K
    M = x.numel() // w_gate.K
    if out is None:
        out = torch.empty((M, w_gate.N), dtype=out_dtype or torch.float32, device=x.device)
    _check(lib().nxq_qmatmul_swiglu(w_gate.handle, w_up.handle, x.data_ptr(), _dtype_code(x.dtype), out.data_ptr(),
                                    _dtype_code(out.dtype), M, _stream_ptr(stream)))
    return out


def qmatmul_residual(w: Weight, x, res, out=None, out_dtype=None, stream=None):
    """y = x W^T + res (res fp32 [M][N]; out may be res)."""
    import torch

    assert x.is_cuda and x.is_contiguous() and x.shape[-1] == w.K
    M = x.numel() // w.K
    assert res.dtype == torch.float32 and res.is_contiguous() and res.numel() == M * w.N
    if out is None:
        out = torch.empty((M, w.N), dtype=out_dtype or torch.float32, device=x.device)
    _check(lib().nxq_qmatmul_residual(w.handle, x.data_ptr(), _dtype_code(x.dtype), res.data_ptr(), out.data_ptr(),
                                      _dtype_code(out.dtype), M, _stream_ptr(stream)))
    return out


def rmsnorm_qmatmul(ws, x, norm, eps: float, outs=None, out_dtype=None, stream=None):
    """y_i = (x * r * norm) W_i^T, r = 1 / sqrt(mean(x^2) + eps) per token row;
    norm is an fp32 CUDA tensor [K]; all weights share K."""
    import torch

    ws = list(ws)
    K = ws[0].K
    assert x.is_cuda and x.is_contiguous() and x.shape[-1] == K
    assert norm.dtype == torch.float32 and norm.is_contiguous() and norm.numel() == K
    M = x.numel() // K
    if outs is None:
        outs = [torch.empty((M, w.N), dtype=out_dtype or torch.float32, device=x.device) for w in ws]
    n = len(ws)
    arr = ctypes.c_void_p * n
    _check(lib().nxq_rmsnorm_qmatmul(arr(*[w.handle.value for w in ws]), n, x.data_ptr(), _dtype_code(x.dtype),
                                     norm.data_ptr(), eps, arr(*[y.data_ptr() for y in outs]),
                                     _dtype_code(outs[0].dtype), M, _stream_ptr(stream)))
    return outs


def qmatmul_host(w: Weight, x: np.ndarray, out: Optional[np.ndarray] = None) -> np.ndarray:
    """Synchronous drop-in for ComputeDispatch::gemm_int4: fp32 host arrays in and out."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M = x.size // w.K
    if out is None:
        out = np.empty((M, w.N), dtype=np.float32)
    _check(lib().nxq_qmatmul_host(w.handle, x.ctypes.data, out.ctypes.data, M))
    return out


def stream_sync(stream=None) -> None:
    _check(lib().nxq_stream_sync(_stream_ptr(stream)))


def set_wait_limit(microseconds: int) -> None:
    """Limit of every bounded device-side wait (0 = the default, about 2 s)."""
    _check(lib().nxq_set_wait_limit(microseconds))


HOOK_STREAMK_SKIP_COUNT = 1


def test_hook(hook: int, on: bool) -> None:
    """Failure-detection test hooks (nxq_test_hook); off by default."""
    _check(lib().nxq_test_hook(hook, 1 if on else 0))


def kernel_name(w: Weight, M: int, x_dtype: int = F16, y_dtype: int = F32) -> str:
    """The kernel nxq_qmatmul launches for this weight, M and dtypes."""
    buf = ctypes.create_string_buffer(128)
    _check(lib().nxq_qmatmul_kernel_name(w.handle, M, x_dtype, y_dtype, buf, 128))
    return buf.value.decode()


def launch_count() -> int:
    v = ctypes.c_uint64()
    _check(lib().nxq_launch_count(ctypes.byref(v)))
    return v.value


# ---- residency loader: GGUF files --------------------------------------------

class GGUF:
    """A GGUF v2/v3 file opened by the library's loader (mapped read-only; the
    index is parsed and bounds-checked on the host, no GPU needed).  Use as a
    context manager or call close()."""

    def __init__(self, path):
        h = ctypes.c_void_p()
        _check(lib().nxq_gguf_open(str(path).encode(), ctypes.byref(h)))
        self._h = h

    @property
    def handle(self) -> ctypes.c_void_p:
        if self._h is None:
            raise NxqError(-1, "GGUF file already closed")
        return self._h

    def close(self) -> None:
        if self._h is not None:
            _check(lib().nxq_gguf_close(self._h))
            self._h = None

    def __enter__(self) -> "GGUF":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def header(self) -> dict:
        v, a, d = ctypes.c_uint32(), ctypes.c_uint64(), ctypes.c_uint64()
        _check(lib().nxq_gguf_header(self.handle, ctypes.byref(v), ctypes.byref(a), ctypes.byref(d)))
        return {"version": v.value, "alignment": a.value, "data_start": d.value}

    def tensors(self) -> list[dict]:
        n = ctypes.c_int64()
        _check(lib().nxq_gguf_tensor_count(self.handle, ctypes.byref(n)))
        return [self.tensor_info(i) for i in range(n.value)]

    def tensor_info(self, i: int) -> dict:
        name = ctypes.create_string_buffer(512)
        t, nd = ctypes.c_int(), ctypes.c_int()
        dims = (ctypes.c_int64 * 4)()
        off, nb = ctypes.c_uint64(), ctypes.c_uint64()
        _check(lib().nxq_gguf_tensor_info(self.handle, i, name, 512, ctypes.byref(t), ctypes.byref(nd), dims,
                                          ctypes.byref(off), ctypes.byref(nb)))
        return {"name": name.value.decode(), "type": t.value, "dims": list(dims)[:nd.value],
                "offset": off.value, "bytes": nb.value}

    def find(self, name: str) -> int:
        i = ctypes.c_int64()
        _check(lib().nxq_gguf_find(self.handle, name.encode(), ctypes.byref(i)))
        return i.value

    def tensor_bytes(self, i: int) -> np.ndarray:
        """The tensor's bytes in the mapping (a copy)."""
        p, nb = ctypes.c_void_p(), ctypes.c_uint64()
        _check(lib().nxq_gguf_tensor_data(self.handle, i, ctypes.byref(p), ctypes.byref(nb)))
        return np.ctypeslib.as_array((ctypes.c_uint8 * nb.value).from_address(p.value)).copy()

    def metadata(self) -> dict:
        """key -> value type id (NXQ_GGUF_*)."""
        n = ctypes.c_int64()
        _check(lib().nxq_gguf_meta_count(self.handle, ctypes.byref(n)))
        out = {}
        for i in range(n.value):
            key = ctypes.create_string_buffer(1024)
            t = ctypes.c_int()
            _check(lib().nxq_gguf_meta_key(self.handle, i, key, 1024, ctypes.byref(t)))
            out[key.value.decode()] = t.value
        return out

    def meta_uint(self, key: str) -> int:
        v = ctypes.c_uint64()
        _check(lib().nxq_gguf_meta_uint(self.handle, key.encode(), ctypes.byref(v)))
        return v.value

    def meta_int(self, key: str) -> int:
        v = ctypes.c_int64()
        _check(lib().nxq_gguf_meta_int(self.handle, key.encode(), ctypes.byref(v)))
        return v.value

    def meta_float(self, key: str) -> float:
        v = ctypes.c_double()
        _check(lib().nxq_gguf_meta_float(self.handle, key.encode(), ctypes.byref(v)))
        return v.value

    def meta_string(self, key: str, n: int = 4096) -> str:
        buf = ctypes.create_string_buffer(n)
        _check(lib().nxq_gguf_meta_string(self.handle, key.encode(), buf, n))
        return buf.value.decode()

    def meta_array(self, key: str) -> tuple[int, int]:
        t, n = ctypes.c_int(), ctypes.c_uint64()
        _check(lib().nxq_gguf_meta_array(self.handle, key.encode(), ctypes.byref(t), ctypes.byref(n)))
        return t.value, n.value

    def register(self, name_or_index, slice_: int = 0) -> "Weight":
        """Upload tensor [N][K] (expert `slice_` of a 3-D tensor) as a weight."""
        i = self.find(name_or_index) if isinstance(name_or_index, str) else int(name_or_index)
        info = self.tensor_info(i)
        h = ctypes.c_void_p()
        _check(lib().nxq_gguf_register(self.handle, i, slice_, ctypes.byref(h)))
        return Weight(h.value, info["type"], info["dims"][1], info["dims"][0])

    def register_shard(self, name_or_index, split: int, rank: int, world: int, slice_: int = 0) -> "Weight":
        i = self.find(name_or_index) if isinstance(name_or_index, str) else int(name_or_index)
        info = self.tensor_info(i)
        h = ctypes.c_void_p()
        _check(lib().nxq_gguf_register_shard(self.handle, i, slice_, split, rank, world, ctypes.byref(h)))
        N, K = info["dims"][1], info["dims"][0]
        return Weight(h.value, info["type"], N // world if split == SPLIT_COL else N,
                      K // world if split == SPLIT_ROW else K)


# ---- residency loader: NXF files ----------------------------------------------

# NXF chunk codecs (Codec, core/config.h) that register as weights, and the
# block type each becomes (INT4: the NXF INT4 group type of the chunk's group size).
NXF_CODEC_INT4, NXF_CODEC_Q3K, NXF_CODEC_Q4K, NXF_CODEC_Q2K = 4, 11, 12, 13


def xxh32(data) -> int:
    """xxHash32 (seed 0) of a bytes-like object: the NXF chunk checksum."""
    buf = np.ascontiguousarray(np.frombuffer(bytes(data), dtype=np.uint8))
    v = ctypes.c_uint32()
    _check(lib().nxq_nxf_xxh32(buf.ctypes.data if buf.size else None, buf.size, ctypes.byref(v)))
    return v.value


class NXF:
    """An NXF file opened by the library's loader (mapped read-only; header,
    manifest and tensor index parsed and bounds-checked on the host, no GPU
    needed).  Use as a context manager or call close()."""

    def __init__(self, path):
        h = ctypes.c_void_p()
        _check(lib().nxq_nxf_open(str(path).encode(), ctypes.byref(h)))
        self._h = h

    @property
    def handle(self) -> ctypes.c_void_p:
        if self._h is None:
            raise NxqError(-1, "NXF file already closed")
        return self._h

    def close(self) -> None:
        if self._h is not None:
            _check(lib().nxq_nxf_close(self._h))
            self._h = None

    def __enter__(self) -> "NXF":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def tensors(self) -> list[dict]:
        n = ctypes.c_int64()
        _check(lib().nxq_nxf_tensor_count(self.handle, ctypes.byref(n)))
        return [self.tensor_info(i) for i in range(n.value)]

    def tensor_info(self, i: int) -> dict:
        name = ctypes.create_string_buffer(512)
        dt, nd, codec, gs = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        dims = (ctypes.c_int64 * 4)()
        nc, nb = ctypes.c_int64(), ctypes.c_uint64()
        _check(lib().nxq_nxf_tensor_info(self.handle, i, name, 512, ctypes.byref(dt), ctypes.byref(nd), dims,
                                         ctypes.byref(nc), ctypes.byref(codec), ctypes.byref(gs), ctypes.byref(nb)))
        return {"name": name.value.decode(), "dtype": dt.value, "dims": list(dims)[:nd.value],
                "chunks": nc.value, "codec": codec.value, "group_size": gs.value, "bytes": nb.value}

    def chunk_info(self, i: int, c: int) -> dict:
        off, st, de, cs = ctypes.c_uint64(), ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
        codec, gs = ctypes.c_int(), ctypes.c_int()
        _check(lib().nxq_nxf_chunk_info(self.handle, i, c, ctypes.byref(off), ctypes.byref(st), ctypes.byref(de),
                                        ctypes.byref(cs), ctypes.byref(codec), ctypes.byref(gs)))
        return {"offset": off.value, "stored": st.value, "decoded": de.value, "checksum": cs.value,
                "codec": codec.value, "group_size": gs.value}

    def find(self, name: str) -> int:
        i = ctypes.c_int64()
        _check(lib().nxq_nxf_find(self.handle, name.encode(), ctypes.byref(i)))
        return i.value

    def verify(self, name_or_index) -> None:
        i = self.find(name_or_index) if isinstance(name_or_index, str) else int(name_or_index)
        _check(lib().nxq_nxf_verify(self.handle, i))

    def manifest(self) -> str:
        n = ctypes.c_uint64()
        _check(lib().nxq_nxf_manifest(self.handle, None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(n.value + 1)
        _check(lib().nxq_nxf_manifest(self.handle, buf, n.value + 1, None))
        return buf.value.decode()

    def manifest_number(self, key: str) -> float:
        v = ctypes.c_double()
        _check(lib().nxq_nxf_manifest_number(self.handle, key.encode(), ctypes.byref(v)))
        return v.value

    def manifest_string(self, key: str, n: int = 4096) -> str:
        buf = ctypes.create_string_buffer(n)
        _check(lib().nxq_nxf_manifest_string(self.handle, key.encode(), buf, n))
        return buf.value.decode()

    @staticmethod
    def _type(info: dict) -> int:
        c = info["codec"]
        if c == NXF_CODEC_INT4:
            return 100 + info["group_size"] // 32
        return {NXF_CODEC_Q3K: TYPES["Q3_K"], NXF_CODEC_Q4K: TYPES["Q4_K"], NXF_CODEC_Q2K: TYPES["Q2_K"]}.get(c, -1)

    def register(self, name_or_index, slice_: int = 0) -> "Weight":
        """Upload tensor [N][K] (slice `slice_` of a 3-D tensor) as a weight,
        after checking every chunk's xxHash32."""
        i = self.find(name_or_index) if isinstance(name_or_index, str) else int(name_or_index)
        info = self.tensor_info(i)
        h = ctypes.c_void_p()
        _check(lib().nxq_nxf_register(self.handle, i, slice_, ctypes.byref(h)))
        w = Weight(h.value, self._type(info), info["dims"][1], info["dims"][0])
        w.type = w.info()["type"]  # the block type the library chose for the chunk's codec
        return w

    def register_shard(self, name_or_index, split: int, rank: int, world: int, slice_: int = 0) -> "Weight":
        i = self.find(name_or_index) if isinstance(name_or_index, str) else int(name_or_index)
        info = self.tensor_info(i)
        h = ctypes.c_void_p()
        _check(lib().nxq_nxf_register_shard(self.handle, i, slice_, split, rank, world, ctypes.byref(h)))
        N, K = info["dims"][1], info["dims"][0]
        w = Weight(h.value, self._type(info), N // world if split == SPLIT_COL else N,
                   K // world if split == SPLIT_ROW else K)
        w.type = w.info()["type"]
        return w


# ---- tensor parallelism ------------------------------------------------------

def tp_unique_id() -> bytes:
    n = lib().nxq_tp_unique_id_size()
    buf = ctypes.create_string_buffer(n)
    _check(lib().nxq_tp_unique_id(buf, n))
    return buf.raw


def tp_init(rank: int, world: int, uid: bytes) -> None:
    buf = ctypes.create_string_buffer(uid, len(uid))
    _check(lib().nxq_tp_init(rank, world, buf, len(uid)))


def tp_shutdown() -> None:
    _check(lib().nxq_tp_shutdown())


def tp_qmatmul(shard: Weight, x, out, split: int, stream=None):
    M = x.numel() // shard.K
    _check(lib().nxq_tp_qmatmul(shard.handle, x.data_ptr(), _dtype_code(x.dtype), out.data_ptr(),
                                _dtype_code(out.dtype), M, split, _stream_ptr(stream)))
    return out


def tp_p2p_enabled() -> int:
    """Peer-memory path of this rank: 1 = allreduces up to 8 MB over NVLink
    peer memory, 2 = decode row-split calls fused with their reduction, 0 =
    NCCL only (NXQ_TP_ALLREDUCE at nxq_tp_init)."""
    v = ctypes.c_int()
    _check(lib().nxq_tp_p2p_enabled(ctypes.byref(v)))
    return v.value


def tp_wait(stream=None, timeout_ms: int = 10000) -> None:
    """Wait for the TP work on `stream`; aborts the communicator on an NCCL
    error or when the deadline passes (nxq_tp_wait)."""
    _check(lib().nxq_tp_wait(_stream_ptr(stream), timeout_ms))


HOOK_TP_STREAM_PENDING = 2


def tp_allreduce_f32(buf, stream=None):
    _check(lib().nxq_tp_allreduce_f32(buf.data_ptr(), buf.numel(), _stream_ptr(stream)))
    return buf
