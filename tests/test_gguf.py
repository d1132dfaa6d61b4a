"""The residency loader (nxq_gguf_*): GGUF v2/v3 parsing on the host, and
registration of file tensors into HBM (GPU tests).

CPU: header, metadata of every value type (arrays skipped with their type and
length kept, as gguf_importer.cpp read_gguf_value does), tensor index, data
alignment (default 32, general.alignment, 0 meaning 32), the tensor bytes seen
through the mapping, and refusal of malformed files with NXQ_ERR_FORMAT: bad
magic, versions other than 2/3, more than 4 dimensions, duplicate names, data
past the end, and every truncation of a valid file.
GPU: a Q4_K matrix and one expert of a stacked Q3_K tensor registered from the
file decode bit-exactly to the reference decoders and multiply within the
parity bar; a TP shard matches nxq_weight_register_shard of the same blocks."""
from __future__ import annotations

import numpy as np
import pytest

from gguf_file import (ARRAY, BOOL, F32, F64, I8, I16, I32, I64, STRING, U8, U16, U32, U64, gguf_bytes,
                       write_gguf)

import nxq
from nxq import synth

ERR_ARG, ERR_CODEC, ERR_SHAPE, ERR_FORMAT = -1, -2, -3, -10
Q3, Q4K, T_F32 = 11, 12, 0

META = [
    ("general.architecture", STRING, "llama"),
    ("u8", U8, 200), ("i8", I8, -100), ("u16", U16, 60000), ("i16", I16, -30000),
    ("u32", U32, 4000000000), ("i32", I32, -2000000000), ("u64", U64, 2**63 + 5), ("i64", I64, -2**62),
    ("f32", F32, 1.5), ("f64", F64, -2.25), ("flag", BOOL, 1),
    ("tokens", ARRAY, (STRING, ["a", "bb", "ccc"])),
    ("ids", ARRAY, (U32, [1, 2, 3, 4, 5])),
    ("nested", ARRAY, (ARRAY, [(I8, [1, 2]), (I8, [3])])),
]


def _tensors():
    q4 = synth.make_blocks(Q4K, 64, 512, seed=11)
    q3 = synth.make_blocks(Q3, 3 * 32, 256, seed=12)  # 3 experts of [32][256]
    norm = np.arange(96, dtype=np.float32).view(np.uint8)
    return [("blk.0.ffn_gate.weight", Q4K, [512, 64], q4),
            ("blk.0.ffn_down_exps.weight", Q3, [256, 32, 3], q3),
            ("blk.0.attn_norm.weight", T_F32, [96], norm)]


@pytest.fixture
def gfile(tmp_path):
    p = tmp_path / "model.gguf"
    write_gguf(p, _tensors(), META)
    return p


def _rc(fn, *a):
    with pytest.raises(nxq.NxqError) as e:
        fn(*a)
    return e.value.code


def test_parse_header_tensors_and_data(gfile):
    with nxq.GGUF(gfile) as g:
        h = g.header()
        assert h["version"] == 3 and h["alignment"] == 32 and h["data_start"] % 32 == 0
        ts = g.tensors()
        want = _tensors()
        assert [t["name"] for t in ts] == [w[0] for w in want]
        for t, (name, typ, dims, data) in zip(ts, want):
            assert t["type"] == typ and t["dims"] == dims and t["bytes"] == data.size
            assert t["offset"] % 32 == 0
            assert np.array_equal(g.tensor_bytes(g.find(name)), data)
        assert _rc(g.find, "missing.weight") == ERR_ARG


def test_metadata_values(gfile):
    with nxq.GGUF(gfile) as g:
        kinds = g.metadata()
        assert list(kinds) == [k for k, _, _ in META]
        assert kinds["tokens"] == ARRAY and kinds["f64"] == F64
        assert g.meta_string("general.architecture") == "llama"
        assert g.meta_uint("u8") == 200 and g.meta_int("i8") == -100
        assert g.meta_uint("u16") == 60000 and g.meta_int("i16") == -30000
        assert g.meta_uint("u32") == 4000000000 and g.meta_int("i32") == -2000000000
        assert g.meta_uint("u64") == 2**63 + 5 and g.meta_int("i64") == -2**62
        assert g.meta_float("f32") == 1.5 and g.meta_float("f64") == -2.25
        assert g.meta_uint("flag") == 1
        assert g.meta_array("tokens") == (STRING, 3) and g.meta_array("ids") == (U32, 5)
        assert g.meta_array("nested") == (ARRAY, 2)
        # a value read as the wrong kind, or a key that is not there
        assert _rc(g.meta_uint, "i8") == ERR_ARG          # negative
        assert _rc(g.meta_int, "u64") == ERR_ARG          # does not fit int64
        assert _rc(g.meta_float, "u32") == ERR_ARG
        assert _rc(g.meta_uint, "f32") == ERR_ARG
        assert _rc(g.meta_string, "u8") == ERR_ARG
        assert _rc(g.meta_array, "u8") == ERR_ARG
        assert _rc(g.meta_uint, "nope") == ERR_ARG


@pytest.mark.parametrize("version,align", [(2, None), (3, 64), (3, 0), (2, 128)])
def test_versions_and_alignment(tmp_path, version, align):
    meta = [] if align is None else [("general.alignment", U32, align)]
    p = tmp_path / "a.gguf"
    write_gguf(p, _tensors(), meta, version=version)
    a = 32 if not align else align
    with nxq.GGUF(p) as g:
        h = g.header()
        assert h["version"] == version and h["alignment"] == a and h["data_start"] % a == 0
        for name, typ, dims, data in _tensors():
            i = g.find(name)
            assert g.tensor_info(i)["offset"] % a == 0
            assert np.array_equal(g.tensor_bytes(i), data)


def _open_bytes(tmp_path, raw: bytes):
    p = tmp_path / "bad.gguf"
    p.write_bytes(raw)
    g = nxq.GGUF(p)
    g.close()


def test_malformed_files_are_refused(tmp_path):
    good = gguf_bytes(_tensors(), META)
    cases = {
        "magic": gguf_bytes(_tensors(), META, magic=b"GGUG"),
        "v1": gguf_bytes(_tensors(), META, version=1),
        "v4": gguf_bytes(_tensors(), META, version=4),
        "dims": gguf_bytes([("t", Q4K, [256, 1, 1, 1, 1], np.zeros(144, np.uint8))]),
        "dup": gguf_bytes([("t", T_F32, [4], np.zeros(16, np.uint8))] * 2),
        "past_end": good[:-100],
        "counts": good[:8] + (2**60).to_bytes(8, "little") + good[16:],
        "empty": b"",
    }
    for name, raw in cases.items():
        code = _rc(_open_bytes, tmp_path, raw)
        assert code == ERR_FORMAT, (name, code, nxq.last_error())
    assert _rc(nxq.GGUF, tmp_path / "does-not-exist.gguf") == ERR_ARG


def test_every_truncation_is_refused_or_complete(tmp_path):
    """Cutting a valid file anywhere gives NXQ_ERR_FORMAT, except cuts that keep
    every tensor's bytes (padding after the last tensor), which parse."""
    raw = gguf_bytes(_tensors(), META)
    end_of_data = len(raw)
    for cut in range(0, len(raw), 7):
        p = tmp_path / "t.gguf"
        p.write_bytes(raw[:cut])
        try:
            g = nxq.GGUF(p)
        except nxq.NxqError as e:
            assert e.code == ERR_FORMAT, (cut, e)
            continue
        g.close()
        assert cut >= end_of_data, cut


def test_register_without_gpu_context_fails_cleanly(gfile):
    """Parsing needs no GPU; registering a non-block tensor is refused before any
    device work, whatever the context."""
    with nxq.GGUF(gfile) as g:
        assert _rc(g.register, "blk.0.attn_norm.weight") == ERR_CODEC
        assert _rc(g.register, "blk.0.ffn_down_exps.weight", 3) == ERR_SHAPE


@pytest.mark.gpu
def test_register_from_file_matches_oracle(gpu, gfile):
    import torch

    from oracle import loader

    with nxq.GGUF(gfile) as g:
        for name, slice_, (typ, N, K) in [("blk.0.ffn_gate.weight", 0, (Q4K, 64, 512)),
                                          ("blk.0.ffn_down_exps.weight", 2, (Q3, 32, 256))]:
            raw = g.tensor_bytes(g.find(name))
            per = raw.size // (3 if slice_ else 1)
            blocks = raw[per * slice_:per * (slice_ + 1)]
            w = g.register(name, slice_)
            try:
                assert (w.N, w.K) == (N, K)
                dec = w.dequant().cpu().numpy()
                assert loader.same_bits(dec, loader.dequant(typ, blocks, N * K).reshape(N, K))
                x = torch.from_numpy(synth.make_activations(4, K, seed=5)).cuda()
                y = nxq.qmatmul(w, x)
                torch.cuda.synchronize()
                want = loader.qmatmul(typ, blocks, N, K, x.float().cpu().numpy())
                assert synth.rel_l2(y.cpu().numpy(), want) < 1e-3
            finally:
                w.release()


@pytest.mark.gpu
def test_register_shard_from_file(gpu, gfile):
    with nxq.GGUF(gfile) as g:
        blocks = g.tensor_bytes(g.find("blk.0.ffn_gate.weight"))
        for split in (nxq.SPLIT_COL, nxq.SPLIT_ROW):
            a = g.register_shard("blk.0.ffn_gate.weight", split, 1, 2)
            b = nxq.Weight.register_shard(blocks, Q4K, 64, 512, split, 1, 2)
            try:
                assert (a.N, a.K) == (b.N, b.K)
                assert np.array_equal(a.dequant().cpu().numpy(), b.dequant().cpu().numpy())
            finally:
                a.release()
                b.release()
