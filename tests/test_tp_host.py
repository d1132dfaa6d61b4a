"""CPU, world_size 2 and 4 over gloo: the tensor-parallel decomposition.

Each rank slices its shard with the library's host-only nxq_shard_extract,
computes its partial output with the CPU oracle, and the ranks combine them
exactly as the GPU path does (COL: gather of disjoint row blocks; ROW: sum
allreduce).  The result must equal the unsharded oracle output.  Also checks
that a rank that fails before the collective makes the others fail fast (a
short process-group timeout) instead of hanging.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, t, N, K, M, q):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "nexus-inference-engine-_b200"))
    import datetime

    import torch
    import torch.distributed as dist

    import nxq
    from nxq import synth
    from oracle import loader

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        blocks = synth.make_blocks(t, N, K, seed=77)
        x = synth.make_activations(M, K, seed=78).astype(np.float32)
        full = loader.qmatmul(t, blocks, N, K, x, nthreads=1)
        res = {}
        for split in (nxq.SPLIT_COL, nxq.SPLIT_ROW):
            shard = np.zeros(blocks.size // world, np.uint8)
            rc = nxq.lib().nxq_shard_extract(blocks.ctypes.data, blocks.size, t, N, K, split, rank,
                                             world, shard.ctypes.data, shard.size)
            assert rc == 0, nxq.last_error()
            if split == nxq.SPLIT_COL:
                n_loc = N // world
                y_loc = torch.from_numpy(loader.qmatmul(t, shard, n_loc, K, x, nthreads=1))
                parts = [torch.zeros_like(y_loc) for _ in range(world)]
                dist.all_gather(parts, y_loc)
                y = torch.cat(parts, dim=1).numpy()
            else:
                k_loc = K // world
                xs = np.ascontiguousarray(x[:, rank * k_loc:(rank + 1) * k_loc])
                y_t = torch.from_numpy(loader.qmatmul(t, shard, N, k_loc, xs, nthreads=1))
                dist.all_reduce(y_t)
                y = y_t.numpy()
            res[split] = synth.rel_l2(y, full)
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("t", [11, 12])
@pytest.mark.parametrize("world", [2, 4])
def test_tp_decomposition_matches_full(t, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    N, K, M = 128 * world, 2048, 3
    procs = [ctx.Process(target=_worker, args=(r, world, port, t, N, K, M, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    out = dict(q.get(timeout=5) for _ in range(world))
    for rank in range(world):
        assert out[rank][0] < 1e-6  # COL: disjoint rows, exact
        assert out[rank][1] < 1e-5  # ROW: fp32 partial sums added in another order


def _dying_worker(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # leaves between steps, before the collective
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put(("no-error", rank))
    except Exception as e:  # noqa: BLE001
        q.put(("error", type(e).__name__))


def test_rank_failure_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert procs[1].exitcode == 3
    kind, _ = q.get(timeout=10)
    assert kind == "error"
