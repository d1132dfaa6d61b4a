"""Test helper: writes GGUF v2/v3 files in the published layout (header, metadata
key/values, tensor index, data section aligned to general.alignment), for the
loader tests.  Not used by the library."""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
           U64: "<Q", I64: "<q", F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype in _SCALAR:
        return struct.pack(_SCALAR[vtype], v)
    if vtype == STRING:
        return _str(v)
    if vtype == ARRAY:
        etype, items = v
        return struct.pack("<IQ", etype, len(items)) + b"".join(_value(etype, x) for x in items)
    raise ValueError(vtype)


def gguf_bytes(tensors, metadata=(), version: int = 3, magic: bytes = b"GGUF") -> bytes:
    """tensors: (name, ggml type, dims with dims[0] fastest, raw bytes);
    metadata: (key, value type, value), arrays as (element type, [values])."""
    align = 32
    for key, vtype, v in metadata:
        if key == "general.alignment":
            align = v or 32
    out = bytearray(magic + struct.pack("<IQQ", version, len(tensors), len(metadata)))
    for key, vtype, v in metadata:
        out += _str(key) + struct.pack("<I", vtype) + _value(vtype, v)
    offsets, off = [], 0
    for name, t, dims, data in tensors:
        off = -(-off // align) * align
        offsets.append(off)
        off += len(data)
    for (name, t, dims, data), o in zip(tensors, offsets):
        out += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", t, o)
    start = -(-len(out) // align) * align
    out += b"\0" * (start - len(out))
    for (name, t, dims, data), o in zip(tensors, offsets):
        out += b"\0" * (start + o - len(out))
        out += bytes(np.asarray(data, dtype=np.uint8).tobytes())
    return bytes(out)


def write_gguf(path, tensors, metadata=(), version: int = 3) -> None:
    with open(path, "wb") as f:
        f.write(gguf_bytes(tensors, metadata, version))
