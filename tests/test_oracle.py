"""CPU: the oracle restatement against the reference's own decoders (golden
fixtures made by tests/golden/make_golden.py, and the compiled reference where
it is present), and the synthetic-block packers against the decode spec."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from conftest import ALL_TYPES, NAMES, golden
from oracle import loader
from nxq import synth


@pytest.mark.parametrize("t", ALL_TYPES, ids=lambda t: NAMES[t])
def test_port_matches_golden_kat(t):
    g = golden(t)
    out = loader.dequant(t, g["kat_blocks"], int(g["kat_n"]))
    assert loader.same_bits(out, g["kat_out"])


@pytest.mark.parametrize("t", ALL_TYPES, ids=lambda t: NAMES[t])
def test_port_matches_golden_matrix(t):
    g = golden(t)
    N, K = int(g["mat_N"]), int(g["mat_K"])
    w = loader.dequant(t, g["mat_blocks"], N * K)
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(g["mat_w_sha256"])
    y = loader.qmatmul(t, g["mat_blocks"], N, K, g["mat_x"], nthreads=2)
    assert synth.rel_l2(y, g["mat_y"]) < 1e-6


@pytest.mark.parametrize("t", ALL_TYPES, ids=lambda t: NAMES[t])
def test_port_matches_compiled_reference(t):
    if loader.ref() is None:
        pytest.skip("reference decoders not built here (oracle/_ref)")
    qk, bb = synth.GEOMETRY[t]
    blocks = synth.make_blocks(t, 64, 4096, seed=123 + t, dist="raw")
    n = 64 * 4096
    assert loader.same_bits(loader.dequant(t, blocks, n), loader.dequant(t, blocks, n, which="ref"))


def test_half_conversion_all_values():
    h = np.arange(65536, dtype=np.uint16)
    out = loader.dequant(1, h.view(np.uint8), 65536)
    # numpy's half->float conversion is exact and keeps NaN payloads.
    assert np.array_equal(out.view(np.uint32), h.view(np.float16).astype(np.float32).view(np.uint32))
    if loader.ref() is not None:
        assert np.array_equal(out.view(np.uint32), loader.dequant(1, h.view(np.uint8), 65536, "ref").view(np.uint32))


def _f32(v):
    return np.float32(v)


def test_pack_q4_0_roundtrip():
    g = synth.rng(1)
    q = g.integers(0, 16, 32)
    d = synth.half_bits(0.0123)
    out = loader.dequant(2, np.frombuffer(synth.pack_q4_0(d, q), np.uint8), 32)
    dv = np.uint16(d).view(np.float16).astype(np.float32)
    assert np.array_equal(out, (q - 8).astype(np.float32) * dv)


def test_pack_q8_0_roundtrip():
    g = synth.rng(2)
    q = g.integers(-127, 128, 32)
    d = synth.half_bits(-0.0031)
    out = loader.dequant(8, np.frombuffer(synth.pack_q8_0(d, q), np.uint8), 32)
    dv = np.uint16(d).view(np.float16).astype(np.float32)
    assert np.array_equal(out, q.astype(np.float32) * dv)


def test_pack_q4_k_roundtrip():
    g = synth.rng(3)
    sc, mn, q = g.integers(0, 64, 8), g.integers(0, 64, 8), g.integers(0, 16, 256)
    d, dm = synth.half_bits(0.0007), synth.half_bits(0.0003)
    out = loader.dequant(12, np.frombuffer(synth.pack_q4_k(d, dm, sc, mn, q), np.uint8), 256)
    dv = np.uint16(d).view(np.float16).astype(np.float32)
    mv = np.uint16(dm).view(np.float16).astype(np.float32)
    grp = np.arange(256) // 32
    want = (dv * sc[grp].astype(np.float32)) * q.astype(np.float32) - mv * mn[grp].astype(np.float32)
    assert np.array_equal(out, want.astype(np.float32))


def test_pack_q3_k_roundtrip():
    g = synth.rng(4)
    sc, q = g.integers(0, 64, 16), g.integers(0, 8, 256)
    d = synth.half_bits(0.0009)
    out = loader.dequant(11, np.frombuffer(synth.pack_q3_k(d, sc, q), np.uint8), 256)
    dv = np.uint16(d).view(np.float16).astype(np.float32)
    grp = np.arange(256) // 16
    want = (dv * (sc[grp] - 32).astype(np.float32)) * (q.astype(np.float32) - np.float32(4.0))
    assert np.array_equal(out, want.astype(np.float32))


def test_synthetic_distributions():
    # Q8_0 codes stay in -127..127 and scales are positive normals.
    b = synth.make_blocks(8, 16, 4096, seed=5).reshape(-1, 34)
    codes = b[:, 2:].view(np.int8)
    assert codes.min() >= -127
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    assert (d > 0).all() and (d < 0.02).all()
    b = synth.make_blocks(12, 16, 4096, seed=6).reshape(-1, 144)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    assert (d >= 9.9e-5).all() and (d <= 1.01e-3).all()


def test_oracle_rejects_bad_shape():
    with pytest.raises(ValueError):
        loader.qmatmul(12, np.zeros(144, np.uint8), 1, 100, np.zeros((1, 100), np.float32))


def test_nxf_flat_codecs_known_answers():
    """The oracle's NXF INT8 / FP16 / FP32 decoders (hybrid_model.cpp:165-255)
    on every code: INT8 q / 127 in fp32 (numpy's correctly rounded float32
    division); FP16 all 65,536 halves, with zero/subnormal exponents read as a
    signed zero and the rest exact; FP32 unchanged."""
    q = np.arange(-128, 128, dtype=np.int16).astype(np.int8)
    got = loader.dequant(120, q.view(np.uint8), 256)
    assert np.array_equal(got.view(np.uint32), (q.astype(np.float32) / np.float32(127.0)).view(np.uint32))
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = loader.dequant(121, h.view(np.uint8), 65536)
    want = h.view(np.float16).astype(np.float32)
    flush = (h & 0x7C00) == 0
    want[flush] = np.where(h[flush] & 0x8000, np.float32(-0.0), np.float32(0.0))
    assert loader.same_bits(got, want)
    assert np.array_equal(np.signbit(got[flush]), (h[flush] & 0x8000) != 0)
    f = np.random.default_rng(1).standard_normal(96).astype(np.float32)
    assert np.array_equal(loader.dequant(122, f.view(np.uint8), 96), f)
