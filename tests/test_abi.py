"""CPU: the C-ABI library loads, exports every entry point include/nxq.h
declares, and its host-only logic (argument checks, block geometry, shard
slicing) behaves without a GPU."""
from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest

import nxq
from nxq import synth
from conftest import ALL_TYPES, NAMES


def test_library_exports_every_declared_symbol():
    L = nxq.lib()
    declared = nxq.declared_symbols()
    assert len(declared) >= 20
    missing = [s for s in declared if not hasattr(L, s)]
    assert missing == []
    assert L.nxq_abi_version() == 1


def test_shim_library_loads_into_the_same_context():
    """The engine-side shim library links libnxq.so and shares its instance:
    a call through the shim's C++ loop sees the same (uninitialised, here)
    context as a direct call, and its argument checks run without a GPU."""
    D = nxq.dispatch_lib()
    f = D.nxq_dispatch_host_steps
    f.restype = ctypes.c_int
    sec = ctypes.c_double(-1.0)
    assert f(None, None, None, None, 0, 1, ctypes.byref(sec)) == -1  # null arrays
    one = (ctypes.c_void_p * 1)(None)
    m = (ctypes.c_int64 * 1)(1)
    # A null weight handle is refused by libnxq itself: the loop forwards it.
    assert f(one, one, one, m, 1, 1, ctypes.byref(sec)) == -1
    assert "null weight handle" in nxq.last_error()
    assert f(one, one, one, m, 0, 3, ctypes.byref(sec)) == 0 and sec.value >= 0.0


def test_header_entry_points_cite_the_reference():
    text = nxq.HEADER.read_text()
    # Every declaration block carries a reference citation or states that the
    # reference has no counterpart (TP).
    assert re.search(r"compute_dispatch\.h:59-61", text)
    assert re.search(r"gguf_importer\.cpp:958-1000", text)


@pytest.mark.parametrize("t", ALL_TYPES, ids=lambda t: NAMES[t])
def test_block_geometry(t):
    qk, bb = ctypes.c_int(), ctypes.c_int()
    assert nxq.lib().nxq_block_geometry(t, ctypes.byref(qk), ctypes.byref(bb)) == 0
    assert (qk.value, bb.value) == synth.GEOMETRY[t]


def test_unknown_codec_rejected():
    rc = nxq.lib().nxq_block_geometry(99, None, None)
    assert rc == -2
    assert "unsupported block type 99" in nxq.last_error()


def test_calls_before_init_fail_cleanly():
    h = ctypes.c_void_p()
    buf = np.zeros(144, np.uint8)
    rc = nxq.lib().nxq_weight_register(buf.ctypes.data, 144, 12, 1, 256, ctypes.byref(h))
    assert rc in (-7, -9)  # not initialised (or no device)
    assert nxq.lib().nxq_weight_register(None, 144, 12, 1, 256, ctypes.byref(h)) == -1
    assert nxq.lib().nxq_qmatmul(None, None, 0, None, 0, 1, None) == -1


def test_init_without_gpu_reports_unsupported():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(nxq.NxqError) as e:
        nxq.init(0)
    assert e.value.code == -9


def _extract(blocks, t, N, K, split, rank, world):
    qk, bb = synth.GEOMETRY[t]
    out_bytes = blocks.size // world
    out = np.zeros(out_bytes, np.uint8)
    rc = nxq.lib().nxq_shard_extract(blocks.ctypes.data, blocks.size, t, N, K, split, rank, world,
                                     out.ctypes.data, out.size)
    return rc, out


@pytest.mark.parametrize("t", [2, 8, 11, 12])
def test_shard_extract_col_and_row(t):
    qk, bb = synth.GEOMETRY[t]
    N, K, world = 16, 2048, 4
    blocks = synth.make_blocks(t, N, K, seed=11)
    rows = blocks.reshape(N, -1)
    for rank in range(world):
        rc, col = _extract(blocks, t, N, K, nxq.SPLIT_COL, rank, world)
        assert rc == 0
        assert np.array_equal(col.reshape(N // world, -1), rows[rank * N // world:(rank + 1) * N // world])
        rc, row = _extract(blocks, t, N, K, nxq.SPLIT_ROW, rank, world)
        assert rc == 0
        w = rows.shape[1] // world
        assert np.array_equal(row.reshape(N, -1), rows[:, rank * w:(rank + 1) * w])


def test_shard_extract_rejects_bad_splits():
    blocks = synth.make_blocks(12, 8, 512, seed=1)
    rc, _ = _extract(blocks, 12, 8, 512, nxq.SPLIT_ROW, 0, 4)  # 512/4 = 128 not a multiple of 256
    assert rc == -3
    rc, _ = _extract(blocks, 12, 8, 512, nxq.SPLIT_COL, 0, 3)  # 8 rows / 3
    assert rc == -3
    rc, _ = _extract(blocks, 12, 8, 512, 7, 0, 2)
    assert rc == -1
    rc, _ = _extract(blocks, 12, 8, 512, nxq.SPLIT_COL, 2, 2)
    assert rc == -1


def test_tp_unique_id_size():
    assert nxq.lib().nxq_tp_unique_id_size() == 128
