"""Writes NXF files for the loader tests: the layout of the reference's
NXFWriter (format/nxf_writer.cpp:92-330), restated.  A 16 KB region holds the
64-byte header; each chunk starts at a 16 KB boundary; the tensor index and
then the JSON manifest follow, each padded to 16 KB; the header (magic "NXF1",
version 1, manifest and index offsets and sizes, data offset 16 KB, total
size) is written last.  Chunk descriptors carry xxHash32 (seed 0) of the
chunk, computed here by the library's nxq.xxh32.  tests/test_nxf.py checks
that this writer and the reference's produce the same bytes."""
from __future__ import annotations

import struct

import numpy as np

import nxq

ALIGN = 16 * 1024
MAGIC = 0x3146584E
# Codec (core/config.h:21-36) and DType (core/config.h:39-46) ids.
CODEC_FP32, CODEC_FP16, CODEC_BF16, CODEC_INT8, CODEC_INT4 = 0, 1, 2, 3, 4
CODEC_Q3K, CODEC_Q4K, CODEC_Q2K = 11, 12, 13
DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_I8, DTYPE_I4 = 0, 1, 2, 3, 4


def _escape(s: str) -> str:
    return s.replace("\\", "\\\\").replace('"', '\\"').replace("\n", "\\n").replace("\t", "\\t")


class Writer:
    def __init__(self):
        self.buf = bytearray(ALIGN)
        self.index = bytearray()
        self.man = {"architecture": "", "name": "", "num_layers": 0, "hidden_dim": 0, "rope_theta": 0.0,
                    "rms_norm_eps": 0.0, "default_codec": 0, "default_group_size": 0}

    def manifest(self, **kv) -> None:
        self.man.update(kv)

    def _pad(self) -> None:
        r = len(self.buf) % ALIGN
        if r:
            self.buf += bytes(ALIGN - r)

    def tensor(self, name: str, shape, dtype: int, chunks) -> None:
        """chunks: [(bytes, codec, group_size)], written in order."""
        descs = bytearray()
        for data, codec, gs in chunks:
            data = bytes(data)
            self._pad()
            descs += struct.pack("<QIIIBB2x", len(self.buf), len(data), len(data), nxq.xxh32(data), codec, gs)
            self.buf += data
        nb = name.encode()
        self.index += struct.pack("<I", len(nb)) + nb + struct.pack("<I", len(shape))
        self.index += struct.pack(f"<{len(shape)}q", *shape) + struct.pack("<BI", dtype, len(chunks)) + descs

    def _manifest_json(self) -> bytes:
        m = self.man
        f32 = lambda v: float(np.float32(v))  # noqa: E731  (the manifest's fields are fp32)
        return ("{\n"
                f'  "architecture": "{_escape(m["architecture"])}",\n'
                f'  "name": "{_escape(m["name"])}",\n'
                f'  "num_layers": {m["num_layers"]},\n'
                f'  "hidden_dim": {m["hidden_dim"]},\n'
                '  "num_heads": 0,\n  "num_kv_heads": 0,\n  "head_dim": 0,\n  "vocab_size": 0,\n'
                '  "max_seq_len": 0,\n'
                f'  "rope_theta": {"%.1f" % f32(m["rope_theta"])},\n'
                f'  "rms_norm_eps": {"%.10g" % f32(m["rms_norm_eps"])},\n'
                '  "num_experts": 0,\n  "num_active_experts": 0,\n'
                f'  "default_codec": {m["default_codec"]},\n'
                f'  "default_group_size": {m["default_group_size"]}\n'
                "}").encode()

    def write(self, path) -> None:
        self._pad()
        idx_off = len(self.buf)
        self.buf += self.index
        self._pad()
        man = self._manifest_json()
        man_off = len(self.buf)
        self.buf += man
        self._pad()
        self.buf[:64] = struct.pack("<IHHQQQQQQ8x", MAGIC, 1, 0, man_off, len(man), idx_off, len(self.index), ALIGN,
                                    len(self.buf))
        with open(path, "wb") as f:
            f.write(self.buf)


def int4_chunk(codes: np.ndarray, scales: np.ndarray, zeros: np.ndarray) -> bytes:
    """An INT4 chunk as the reference's importer writes it (gguf_importer.cpp:
    1144-1170): the packed codes, then the fp32 scales, then the fp32 zeros."""
    return (np.ascontiguousarray(codes, np.uint8).tobytes() + np.ascontiguousarray(scales, np.float32).tobytes()
            + np.ascontiguousarray(zeros, np.float32).tobytes())
