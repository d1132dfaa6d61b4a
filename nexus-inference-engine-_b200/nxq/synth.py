"""Seeded synthetic GGUF block tensors with the value distributions of the
benchmark configurations, plus exact packers for hand-built blocks.

Codes in every format are uniform over their full range, so random bytes are
valid code fields; only the fp16 scale fields (and Q8_0's code range) are set
explicitly.  Packers are the inverse of the reference unpack
(nexus/src/import/gguf_importer.cpp:679-873) and are used for known-answer
blocks.  Seeds use numpy Generator(PCG64(seed)).
"""
from __future__ import annotations

import numpy as np

GEOMETRY = {2: (32, 18), 3: (32, 20), 8: (32, 34), 10: (256, 84), 11: (256, 110),
            12: (256, 144), 13: (256, 176), 14: (256, 210), 101: (32, 24), 102: (64, 40), 104: (128, 72), 108: (256, 136),
            120: (32, 32), 121: (32, 64), 122: (32, 128)}
# Byte offsets of the fp16 fields in each block.
HALF_FIELDS = {2: [0], 3: [0, 2], 8: [0], 10: [80, 82], 11: [108], 12: [0, 2], 13: [0, 2],
               14: [208]}
Q4_0, Q4_1, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 2, 3, 8, 10, 11, 12, 13, 14
I4G = (101, 102, 104, 108)  # NXF INT4, groups of 32 / 64 / 128 / 256
NXF_I8, NXF_F16, NXF_F32 = 120, 121, 122  # NXF INT8 / FP16 / FP32 chunks as blocks of 32


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def _block_view(buf: np.ndarray, bb: int) -> np.ndarray:
    return buf.reshape(-1, bb)


def _set_half(blocks2d: np.ndarray, off: int, vals16: np.ndarray) -> None:
    u = vals16.astype(np.float16).view(np.uint16)
    blocks2d[:, off] = (u & 0xFF).astype(np.uint8)
    blocks2d[:, off + 1] = (u >> 8).astype(np.uint8)


def make_blocks(type_id: int, N: int, K: int, seed: int, dist: str = "config") -> np.ndarray:
    """Flat uint8 array of N rows of K/QK blocks.

    dist="config": the benchmark distributions
      Q4_0: d = fp16(max|w|/8),   w ~ N(0, 0.02) per 32-block; codes uniform 0..15
      Q8_0: d = fp16(max|w|/127), w ~ N(0, 0.02);               codes uniform -127..127
      K-quants and Q4_1: every fp16 field fp16(U(1e-4, 1e-3)); codes and 6-bit
      scale codes uniform
      I4G (NXF INT4 groups): scale fp32 U(1e-3, 5e-3), zero fp32 U(0, 15),
      codes uniform
      NXF_I8: int8 codes uniform -127..127 (w = q / 127)
      NXF_F16 / NXF_F32: w ~ N(0, 0.02)
    dist="raw": every byte uniform (fp16 fields may be subnormal, Inf or NaN).
    """
    qk, bb = GEOMETRY[type_id]
    if K % qk:
        raise ValueError(f"K={K} is not a multiple of {qk}")
    nb = N * (K // qk)
    g = rng(seed)
    buf = g.integers(0, 256, size=nb * bb, dtype=np.uint8)
    if dist == "raw":
        return buf
    b2 = _block_view(buf, bb)
    if type_id in (Q4_0, Q8_0):
        # Per-block max |w| of 32 N(0, 0.02) draws, in slices to bound memory.
        d = np.empty(nb, dtype=np.float32)
        step = 1 << 20
        div = 8.0 if type_id == Q4_0 else 127.0
        for s in range(0, nb, step):
            e = min(nb, s + step)
            w = g.standard_normal((e - s, 32), dtype=np.float32) * 0.02
            d[s:e] = np.abs(w).max(axis=1) / div
        _set_half(b2, 0, d)
        if type_id == Q8_0:
            codes = g.integers(-127, 128, size=(nb, 32), dtype=np.int16).astype(np.int8)
            b2[:, 2:34] = codes.view(np.uint8)
    elif type_id == NXF_I8:
        buf[:] = g.integers(-127, 128, size=nb * bb, dtype=np.int16).astype(np.int8).view(np.uint8)
    elif type_id in (NXF_F16, NXF_F32):
        w = (g.standard_normal(nb * 32, dtype=np.float32) * 0.02).astype(np.float16 if type_id == NXF_F16 else np.float32)
        buf[:] = w.view(np.uint8)
    elif type_id in I4G:
        b2[:, 0:4] = g.uniform(1e-3, 5e-3, size=nb).astype(np.float32).view(np.uint8).reshape(nb, 4)
        b2[:, 4:8] = g.uniform(0.0, 15.0, size=nb).astype(np.float32).view(np.uint8).reshape(nb, 4)
    else:
        for off in HALF_FIELDS[type_id]:
            _set_half(b2, off, g.uniform(1e-4, 1e-3, size=nb).astype(np.float32))
    return buf


def make_activations(M: int, K: int, seed: int, dtype=np.float16) -> np.ndarray:
    """x ~ N(0, 1) of shape [M][K], rounded to `dtype` (np.float16/np.float32) or
    returned as fp32 for the caller to round (bf16)."""
    x = rng(seed).standard_normal((M, K), dtype=np.float32)
    return x.astype(dtype)


def half_bits(v) -> int:
    return int(np.array(v, dtype=np.float16).view(np.uint16))


# ---- exact packers (inverse of the reference unpack) -----------------------

def pack_q4_0(d_bits: int, q: np.ndarray) -> bytes:
    """q[32] in 0..15; byte j = q[j] | q[j+16] << 4 (gguf_importer.cpp:686-692)."""
    q = np.asarray(q, dtype=np.uint8)
    body = (q[:16] & 15) | ((q[16:] & 15) << 4)
    return int(d_bits).to_bytes(2, "little") + body.astype(np.uint8).tobytes()


def pack_q8_0(d_bits: int, q: np.ndarray) -> bytes:
    q = np.asarray(q, dtype=np.int8)
    return int(d_bits).to_bytes(2, "little") + q.tobytes()


def pack_q4_k(d_bits: int, dmin_bits: int, sc: np.ndarray, mn: np.ndarray, q: np.ndarray) -> bytes:
    """sc[8], mn[8] in 0..63, q[256] in 0..15 (inverse of gguf_importer.cpp:856-871)."""
    sc = np.asarray(sc, dtype=np.int64)
    mn = np.asarray(mn, dtype=np.int64)
    s = np.zeros(12, dtype=np.int64)
    for i in range(8):
        s[i] = sc[i] | ((mn[i] & 3) << 6)
    for i in range(4):
        s[8 + i] = (mn[i] >> 2) | ((mn[i + 4] >> 2) << 4)
    q = np.asarray(q, dtype=np.uint8)
    qs = (q[0::2] & 15) | ((q[1::2] & 15) << 4)
    return (int(d_bits).to_bytes(2, "little") + int(dmin_bits).to_bytes(2, "little")
            + s.astype(np.uint8).tobytes() + qs.astype(np.uint8).tobytes())


def pack_q3_k(d_bits: int, sc: np.ndarray, q: np.ndarray) -> bytes:
    """sc[16] in 0..63 (decoded as sc-32), q[256] in 0..7 (decoded as q-4);
    inverse of gguf_importer.cpp:806-827."""
    sc = np.asarray(sc, dtype=np.int64)
    q = np.asarray(q, dtype=np.int64)
    hmask = np.zeros(32, dtype=np.int64)
    qs = np.zeros(64, dtype=np.int64)
    for e in range(256):
        qs[e // 4] |= (q[e] & 3) << (2 * (e % 4))
        hmask[e // 8] |= ((q[e] >> 2) & 1) << (e % 8)
    s = np.zeros(12, dtype=np.int64)
    for i in range(8):
        s[i] = (sc[i] & 15) | ((sc[i + 8] & 15) << 4)
        s[8 + i // 2] |= ((sc[i] >> 4) & 3) << (4 * (i % 2))
        s[8 + i // 2] |= ((sc[i + 8] >> 4) & 3) << (4 * (i % 2) + 2)
    return (hmask.astype(np.uint8).tobytes() + qs.astype(np.uint8).tobytes()
            + s.astype(np.uint8).tobytes() + int(d_bits).to_bytes(2, "little"))


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
