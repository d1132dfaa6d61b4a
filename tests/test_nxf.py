"""NXF residency loader (nxq_nxf_*): the reference's NXF files
(format/nxf.h:27-51, nxf_reader.cpp:166-409) parsed and registered into HBM.

CPU: the test writer (tests/nxf_file.py) produces the same bytes as the
reference's own NXFWriter (compiled into oracle/_ref), which pins both the
layout and the xxHash32 chunk checksums; the loader reads such a file (tensor
index, chunk descriptors, manifest values) and refuses corrupt, truncated and
inconsistent ones; a codec that is no matmul weight is NXQ_ERR_CODEC.
GPU: INT4 (groups of 32 in two chunks, 64 and 128, one slice of a 3-D
tensor), Q4K / Q3K passthrough tensors (one of them in two chunks) and the
flat codecs the engine decodes at load time - INT8 (two chunks), FP16 (with
subnormal halves, read as zero) and an fp32 passthrough stored under another
codec - register bit-exactly (device decode against the oracle) and multiply
within the parity bar; column and row shards decode to their slices of the
whole tensor."""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

import nxf_file
import nxq
from nxq import synth
from oracle import loader

TOL = 1e-3


def _int4(N, K, gs, seed):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 256, N * K // 2, dtype=np.uint8)
    scales = rng.uniform(1e-3, 5e-3, N * K // gs).astype(np.float32)
    zeros = rng.uniform(0.0, 15.0, N * K // gs).astype(np.float32)
    return codes, scales, zeros


def _content():
    """(name, shape [K, N(, E)], dtype, [(bytes, codec, group)]) of a test file."""
    c128 = _int4(256, 1024, 128, 1)
    c64 = _int4(128, 512, 64, 2)
    e3 = _int4(2 * 128, 512, 128, 3)  # two stacked [128][512] slices
    m2 = _int4(192, 256, 32, 7)  # stored in two chunks of 96 rows
    q4k = synth.make_blocks(12, 128, 512, seed=4).tobytes()
    q3k = synth.make_blocks(11, 256, 512, seed=5).tobytes()
    rng = np.random.default_rng(6)
    raw = [rng.integers(0, 256, n, dtype=np.uint8).tobytes() for n in (1, 13, 37, 100)]
    i8 = rng.integers(-128, 128, 64 * 512, dtype=np.int16).astype(np.int8).tobytes()
    f16 = (rng.standard_normal(32 * 256) * 0.02).astype(np.float16)
    f16[::97] = np.float16(3e-6)  # subnormal halves: the engine reads them as zero
    f16[5] = -np.float16(1e-7)
    f32 = (rng.standard_normal(16 * 128) * 0.02).astype(np.float32).tobytes()
    bf16 = rng.integers(0, 1 << 16, 64 * 4, dtype=np.uint16).tobytes()
    return [
        ("blk.0.ffn_gate.weight", [1024, 256], nxf_file.DTYPE_I4,
         [(nxf_file.int4_chunk(*c128), nxf_file.CODEC_INT4, 128)]),
        ("blk.0.attn_k.weight", [512, 128], nxf_file.DTYPE_I4, [(nxf_file.int4_chunk(*c64), nxf_file.CODEC_INT4, 64)]),
        ("blk.0.ffn_gate_exps.weight", [512, 128, 2], nxf_file.DTYPE_I4,
         [(nxf_file.int4_chunk(*e3), nxf_file.CODEC_INT4, 128)]),
        ("blk.0.attn_q.weight", [512, 128], nxf_file.DTYPE_I4, [(q4k, nxf_file.CODEC_Q4K, 0)]),
        ("blk.0.attn_v.weight", [256, 192], nxf_file.DTYPE_I4,
         [(nxf_file.int4_chunk(m2[0][:96 * 128], m2[1][:96 * 8], m2[2][:96 * 8]), nxf_file.CODEC_INT4, 32),
          (nxf_file.int4_chunk(m2[0][96 * 128:], m2[1][96 * 8:], m2[2][96 * 8:]), nxf_file.CODEC_INT4, 32)]),
        ("blk.0.ffn_down.weight", [512, 256], nxf_file.DTYPE_I4,
         [(q3k[: 128 * 2 * 110], nxf_file.CODEC_Q3K, 0), (q3k[128 * 2 * 110:], nxf_file.CODEC_Q3K, 0)]),
        ("raw.odd_sizes", [151], nxf_file.DTYPE_F32, [(r, nxf_file.CODEC_FP32, 0) for r in raw]),
        ("blk.0.attn_o.weight", [512, 64], nxf_file.DTYPE_I8,
         [(i8[:32 * 512], nxf_file.CODEC_INT8, 0), (i8[32 * 512:], nxf_file.CODEC_INT8, 0)]),
        ("blk.0.ffn_up.weight", [256, 32], nxf_file.DTYPE_F16, [(f16.tobytes(), nxf_file.CODEC_FP16, 0)]),
        # 4 bytes per element under another codec: the writer's fp32 passthrough
        ("blk.0.small.weight", [128, 16], nxf_file.DTYPE_F32, [(f32, nxf_file.CODEC_INT8, 0)]),
        ("raw.bf16", [64, 4], nxf_file.DTYPE_BF16, [(bf16, nxf_file.CODEC_BF16, 0)]),
    ], {"c128": c128, "c64": c64, "e3": e3, "m2": m2, "q4k": q4k, "q3k": q3k, "i8": i8, "f16": f16.tobytes(),
        "f32": f32}


MANIFEST = dict(architecture="llama", name='tiny "test"\tmodel', num_layers=2, hidden_dim=4096,
                rope_theta=500000.0, rms_norm_eps=1e-5, default_codec=4, default_group_size=128)


def _write_ours(path):
    w = nxf_file.Writer()
    w.manifest(**MANIFEST)
    for name, shape, dt, chunks in _content()[0]:
        w.tensor(name, shape, dt, chunks)
    w.write(path)


def _write_reference(path):
    ref = loader.ref()
    L = ctypes.CDLL(ref._name)
    L.ref_nxf_create.restype = ctypes.c_void_p
    L.ref_nxf_create.argtypes = [ctypes.c_char_p]
    L.ref_nxf_manifest.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_uint32,
                                   ctypes.c_uint32, ctypes.c_float, ctypes.c_float, ctypes.c_uint32, ctypes.c_uint32]
    L.ref_nxf_begin.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int64),
                                ctypes.c_int]
    L.ref_nxf_chunk.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int]
    L.ref_nxf_end.argtypes = [ctypes.c_void_p]
    L.ref_nxf_finish.argtypes = [ctypes.c_void_p]
    w = L.ref_nxf_create(str(path).encode())
    assert w
    m = MANIFEST
    L.ref_nxf_manifest(w, m["architecture"].encode(), m["name"].encode(), m["num_layers"], m["hidden_dim"],
                       m["rope_theta"], m["rms_norm_eps"], m["default_codec"], m["default_group_size"])
    for name, shape, dt, chunks in _content()[0]:
        L.ref_nxf_begin(w, name.encode(), len(shape), (ctypes.c_int64 * len(shape))(*shape), dt)
        for data, codec, gs in chunks:
            L.ref_nxf_chunk(w, data, len(data), codec, gs)
        L.ref_nxf_end(w)
    L.ref_nxf_finish(w)


def _need_ref():
    if loader.ref() is None:
        pytest.skip("the reference's NXF writer (oracle/_ref) is not built here")


def test_writer_matches_reference_bytes(tmp_path):
    _need_ref()
    _write_reference(tmp_path / "ref.nxf")
    _write_ours(tmp_path / "ours.nxf")
    assert (tmp_path / "ref.nxf").read_bytes() == (tmp_path / "ours.nxf").read_bytes()


def test_reads_reference_file(tmp_path):
    _need_ref()
    path = tmp_path / "ref.nxf"
    _write_reference(path)
    raw = path.read_bytes()
    content = _content()[0]
    with nxq.NXF(path) as f:
        ts = f.tensors()
        assert [t["name"] for t in ts] == [c[0] for c in content]
        for t, (name, shape, dt, chunks) in zip(ts, content):
            assert t["dims"] == shape and t["dtype"] == dt and t["chunks"] == len(chunks)
            assert t["codec"] == chunks[0][1] and t["group_size"] == chunks[0][2]
            assert t["bytes"] == sum(len(c[0]) for c in chunks)
            i = f.find(name)
            for c, (data, codec, gs) in enumerate(chunks):
                d = f.chunk_info(i, c)
                assert d["offset"] % nxf_file.ALIGN == 0 and d["stored"] == d["decoded"] == len(data)
                assert raw[d["offset"]:d["offset"] + d["stored"]] == data
                assert d["checksum"] == nxq.xxh32(data)  # the reference's xxHash32, our restatement
            f.verify(i)
        assert f.manifest_string("architecture") == "llama"
        assert f.manifest_string("name") == MANIFEST["name"]
        assert f.manifest_number("hidden_dim") == 4096 and f.manifest_number("num_layers") == 2
        assert f.manifest_number("rope_theta") == 500000.0
        assert abs(f.manifest_number("rms_norm_eps") - 1e-5) < 1e-12
        assert f.manifest_number("default_group_size") == 128
        assert '"architecture": "llama"' in f.manifest()
        with pytest.raises(nxq.NxqError) as e:
            f.manifest_number("no_such_key")
        assert e.value.code == -1
        with pytest.raises(nxq.NxqError) as e:
            f.find("no.such.tensor")
        assert e.value.code == -1
        with pytest.raises(nxq.NxqError) as e:
            f.register("raw.odd_sizes")  # FP32 codec, 151 bytes for 151 elements
        assert e.value.code == -3
        with pytest.raises(nxq.NxqError) as e:
            f.register("raw.bf16")  # BF16: a codec the reference's engine does not decode
        assert e.value.code == -2


def _expect_format_error(path):
    with pytest.raises(nxq.NxqError) as e:
        nxq.NXF(path)
    assert e.value.code == -10


def test_refuses_bad_files(tmp_path):
    good = tmp_path / "good.nxf"
    _write_ours(good)
    raw = bytearray(good.read_bytes())
    with nxq.NXF(good) as f:
        d = f.chunk_info(f.find("blk.0.attn_q.weight"), 0)
        idx_off = int.from_bytes(raw[24:32], "little")
    # one flipped bit inside a chunk: the index reads, the checksum does not match
    bad = bytearray(raw)
    bad[d["offset"] + 100] ^= 0x10
    (tmp_path / "flip.nxf").write_bytes(bad)
    with nxq.NXF(tmp_path / "flip.nxf") as f:
        with pytest.raises(nxq.NxqError) as e:
            f.verify("blk.0.attn_q.weight")
        assert e.value.code == -10
        f.verify("blk.0.ffn_gate.weight")  # the other tensors are intact
    # truncated file; header total size that disagrees; bad magic; bad version
    (tmp_path / "short.nxf").write_bytes(raw[: len(raw) - 4096])
    _expect_format_error(tmp_path / "short.nxf")
    (tmp_path / "tiny.nxf").write_bytes(raw[:40])
    _expect_format_error(tmp_path / "tiny.nxf")
    for off, val in ((0, b"GGUF"), (4, b"\x02\x00")):
        b = bytearray(raw)
        b[off:off + len(val)] = val
        (tmp_path / "hdr.nxf").write_bytes(b)
        _expect_format_error(tmp_path / "hdr.nxf")
    # a chunk descriptor pointing past the end of the file
    b = bytearray(raw)
    name = b"blk.0.ffn_gate.weight"
    p = idx_off + 4 + len(name) + 4 + 2 * 8 + 1 + 4  # first chunk descriptor of the first tensor
    b[p:p + 8] = (len(raw) - 8).to_bytes(8, "little")
    (tmp_path / "past.nxf").write_bytes(b)
    _expect_format_error(tmp_path / "past.nxf")
    # an index that ends inside a tensor entry
    b = bytearray(raw)
    b[32:40] = (int.from_bytes(raw[32:40], "little") - 3).to_bytes(8, "little")
    (tmp_path / "idx.nxf").write_bytes(b)
    _expect_format_error(tmp_path / "idx.nxf")


def test_xxh32_known_lengths():
    """Stripe, 4-byte and 1-byte tails all reach the hash (the reference's own
    values are pinned by test_reads_reference_file)."""
    data = bytes(range(256)) * 2
    seen = {nxq.xxh32(data[:n]) for n in range(0, 70)}
    assert len(seen) == 70


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["blk.0.ffn_gate.weight", "blk.0.attn_v.weight", "blk.0.ffn_down.weight"])
def test_register_shards(gpu, tmp_path, name):
    """Each rank's COL / ROW shard of an INT4 and a two-chunk Q3K tensor
    decodes to its slice of the whole tensor's decode (ranks registered one
    after another on one GPU)."""
    path = tmp_path / "w.nxf"
    _write_ours(path)
    world = 2
    with gpu.NXF(path) as f:
        w = f.register(name)
        full = w.dequant().cpu().numpy().reshape(w.N, w.K)
        w.release()
        for split in (gpu.SPLIT_COL, gpu.SPLIT_ROW):
            for rank in range(world):
                s = f.register_shard(name, split, rank, world)
                try:
                    got = s.dequant().cpu().numpy().reshape(s.N, s.K)
                    if split == gpu.SPLIT_COL:
                        want = full[rank * s.N:(rank + 1) * s.N]
                    else:
                        want = full[:, rank * s.K:(rank + 1) * s.K]
                    assert loader.same_bits(got.reshape(-1), want.reshape(-1)), (split, rank)
                finally:
                    s.release()


@pytest.mark.gpu
def test_register_and_matmul(gpu, tmp_path):
    import torch

    path = tmp_path / "w.nxf"
    _write_ours(path)
    _, d = _content()
    cases = [  # name, slice, type, N, K, host blocks (oracle input)
        ("blk.0.ffn_gate.weight", 0, 104, 256, 1024, gpu.int4_pack(*d["c128"], 256, 1024, 128)),
        ("blk.0.attn_k.weight", 0, 102, 128, 512, gpu.int4_pack(*d["c64"], 128, 512, 64)),
        ("blk.0.ffn_gate_exps.weight", 1, 104, 128, 512,
         gpu.int4_pack(*d["e3"], 256, 512, 128)[128 * 4 * (8 + 64):]),
        ("blk.0.attn_q.weight", 0, 12, 128, 512, np.frombuffer(d["q4k"], np.uint8)),
        ("blk.0.attn_v.weight", 0, 101, 192, 256, gpu.int4_pack(*d["m2"], 192, 256, 32)),
        ("blk.0.ffn_down.weight", 0, 11, 256, 512, np.frombuffer(d["q3k"], np.uint8)),
        ("blk.0.attn_o.weight", 0, 120, 64, 512, np.frombuffer(d["i8"], np.uint8)),
        ("blk.0.ffn_up.weight", 0, 121, 32, 256, np.frombuffer(d["f16"], np.uint8)),
        ("blk.0.small.weight", 0, 122, 16, 128, np.frombuffer(d["f32"], np.uint8)),
    ]
    with gpu.NXF(path) as f:
        for name, sl, t, N, K, blocks in cases:
            w = f.register(name, sl)
            try:
                assert (w.type, w.N, w.K) == (t, N, K)
                assert loader.same_bits(w.dequant().cpu().numpy().reshape(-1), loader.dequant(t, blocks, N * K))
                x = torch.from_numpy(synth.make_activations(3, K, seed=N)).cuda()
                y = gpu.qmatmul(w, x)
                torch.cuda.synchronize()
                want = loader.qmatmul(t, blocks, N, K, x.float().cpu().numpy())
                assert synth.rel_l2(y.cpu().numpy(), want) < TOL, name
            finally:
                w.release()


@pytest.mark.gpu
@pytest.mark.parametrize("t", [120, 121, 122], ids=["NXF_I8", "NXF_F16", "NXF_F32"])
def test_flat_codecs_on_the_kernels(gpu, t):
    """The flat NXF codecs registered from host arrays: device decode
    bit-exact against the oracle's restatement of the engine's decode, and the
    matmul within the parity bar at decode and prefill batch sizes (INT8 runs
    on the Q8_0 tensor-core kernels, FP16 / FP32 on the CUDA-core kernel)."""
    import torch

    N, K = 640, 1536
    blocks = synth.make_blocks(t, N, K, seed=t)
    if t == 121:  # a few subnormal halves, which the engine reads as zero
        h = blocks.view(np.uint16).copy()
        h[::301] = 0x0003
        blocks = h.view(np.uint8)
    w = gpu.Weight.register(blocks, t, N, K)
    try:
        assert loader.same_bits(w.dequant().cpu().numpy().reshape(-1), loader.dequant(t, blocks, N * K))
        name = gpu.kernel_name(w, 1)
        assert name.startswith("mma_gemv<NXF_I8" if t == 120 else "simt<"), name
        for M in (1, 8, 40):
            x = torch.from_numpy(synth.make_activations(M, K, seed=M)).cuda()
            y = gpu.qmatmul(w, x)
            torch.cuda.synchronize()
            gpu.stream_sync()
            want = loader.qmatmul(t, blocks, N, K, x.float().cpu().numpy())
            assert synth.rel_l2(y.cpu().numpy(), want) < TOL, M
    finally:
        w.release()
