"""CPU: failure detection of the tensor-parallel layer (nxq_tp_*), against a
fake libnccl (tests/fake_nccl/fake_nccl.c, loaded through NXQ_NCCL_LIB) whose
return values the test chooses - the failure is made on the host, nothing
runs on a GPU.

Checked: an asynchronous NCCL error seen by nxq_tp_wait aborts the
communicator and is reported (NXQ_ERR_NCCL); a collective that fails to
enqueue aborts it too; a wait whose stream never finishes (the TP test hook
stands in for a collective waiting on a peer that left) ends at its
deadline with NXQ_ERR_TIMEOUT and an abort; after an abort every TP call is
refused (NXQ_ERR_STATE) until nxq_tp_shutdown (which does not destroy the
aborted communicator again) and a new nxq_tp_init.  The reference has one
device and zero-fills silently on failure (compute_dispatch.cpp:174-176).
Each scenario runs in a fresh process, since NCCL is resolved once per
process."""
from __future__ import annotations

import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
FAKE_SRC = Path(__file__).resolve().parent / "fake_nccl" / "fake_nccl.c"

PRELUDE = """
import ctypes, sys, time
sys.path.insert(0, {pkg!r})
import nxq
L = nxq.lib()
F = ctypes.CDLL({fake!r})
INIT, DESTROY, ABORT, ALLREDUCE, GET_ASYNC = 0, 1, 2, 3, 4
uid = nxq.tp_unique_id()
def init():
    buf = ctypes.create_string_buffer(uid, len(uid))
    assert L.nxq_tp_init(0, 2, buf, len(uid)) == 0, nxq.last_error()
dummy = ctypes.c_void_p(0x1000)  # never dereferenced by the fake
"""


@pytest.fixture(scope="module")
def fake_lib(tmp_path_factory):
    out = tmp_path_factory.mktemp("fake_nccl") / "libfake_nccl.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-o", str(out), str(FAKE_SRC)], check=True)
    return out


def run(fake_lib, body: str) -> str:
    code = PRELUDE.format(pkg=str(ROOT / "nexus-inference-engine-_b200"), fake=str(fake_lib)) + textwrap.dedent(body)
    env = {"NXQ_NCCL_LIB": str(fake_lib), "PATH": "/usr/bin:/bin", "CUDA_VISIBLE_DEVICES": ""}
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_async_error_aborts_and_refuses_until_rejoin(fake_lib):
    out = run(fake_lib, """
        init()
        F.fake_set(6, 0)                      # ncclRemoteError
        rc = L.nxq_tp_wait(None, 1000)
        assert rc == -8, rc                   # NXQ_ERR_NCCL
        assert "asynchronous error" in nxq.last_error()
        assert F.fake_calls(ABORT) == 1
        assert L.nxq_tp_allreduce_f32(dummy, 16, None) == -7   # NXQ_ERR_STATE
        assert F.fake_calls(ALLREDUCE) == 0
        assert L.nxq_tp_wait(None, 10) == -7
        assert L.nxq_tp_shutdown() == 0
        assert F.fake_calls(DESTROY) == 0 and F.fake_calls(ABORT) == 1
        F.fake_set(0, 0)
        init()
        assert L.nxq_tp_allreduce_f32(dummy, 16, None) == 0
        assert F.fake_calls(ALLREDUCE) == 1
        assert L.nxq_tp_shutdown() == 0
        assert F.fake_calls(DESTROY) == 1
        print("ok")
    """)
    assert out.strip() == "ok"


def test_failed_enqueue_aborts(fake_lib):
    out = run(fake_lib, """
        init()
        F.fake_set(0, 1)                      # ncclUnhandledCudaError from ncclAllReduce
        assert L.nxq_tp_allreduce_f32(dummy, 16, None) == -8
        assert "ncclAllReduce failed" in nxq.last_error()
        assert F.fake_calls(ABORT) == 1
        assert L.nxq_tp_allreduce_f32(dummy, 16, None) == -7
        assert F.fake_calls(ALLREDUCE) == 1
        assert L.nxq_tp_shutdown() == 0
        print("ok")
    """)
    assert out.strip() == "ok"


def test_wait_deadline_aborts(fake_lib):
    out = run(fake_lib, """
        init()
        F.fake_set(7, 0)                      # ncclInProgress: no error yet
        assert L.nxq_tp_allreduce_f32(dummy, 16, None) == 0
        assert L.nxq_tp_test_hook(nxq.HOOK_TP_STREAM_PENDING, 1) == 0
        t0 = time.monotonic()
        rc = L.nxq_tp_wait(None, 150)
        el = time.monotonic() - t0
        assert rc == -5, rc                   # NXQ_ERR_TIMEOUT
        assert 0.14 <= el < 5.0, el
        assert "did not finish within 150 ms" in nxq.last_error()
        assert F.fake_calls(ABORT) == 1 and F.fake_calls(GET_ASYNC) >= 2
        assert L.nxq_tp_allreduce_f32(dummy, 16, None) == -7
        assert L.nxq_tp_test_hook(nxq.HOOK_TP_STREAM_PENDING, 0) == 0
        assert L.nxq_tp_test_hook(99, 1) == -1
        assert L.nxq_tp_shutdown() == 0
        print("ok")
    """)
    assert out.strip() == "ok"


def test_calls_before_init_are_refused(fake_lib):
    out = run(fake_lib, """
        assert L.nxq_tp_allreduce_f32(dummy, 16, None) == -7
        assert L.nxq_tp_wait(None, 10) == -7
        assert L.nxq_tp_wait(None, -1) == -1
        print("ok")
    """)
    assert out.strip() == "ok"
