"""GPU, world_size 2 (skipped with fewer than two GPUs): the tensor-parallel
entry point nxq_tp_qmatmul against the unsharded oracle output, with the ROW
split's reduction fused into the decode GEMV (the default) or on NCCL.

Each rank registers its shard with nxq_weight_register_shard and runs the COL
split (the full x, its [M][N/2] slice of y) and the ROW split (its K/2 slice
of x; the library's fp32 reduction leaves the full [M][N] on every rank).
The COL slices are gathered over gloo; both results must be within the parity
bar (rel-L2 <= 1e-3, fp32 accumulation) of loader.qmatmul on the whole weight,
for decode (M <= 32, mma_gemv) and prefill (M > 32, tc_gemm) batch sizes.
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

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, t, N, K, Ms, q, mode):
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
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    joined = False
    try:
        os.environ["NXQ_TP_ALLREDUCE"] = mode
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        nxq.init(rank)
        uid = [nxq.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        nxq.tp_init(rank, world, uid[0])
        joined = True
        blocks = synth.make_blocks(t, N, K, seed=91)
        res = {}
        for M in Ms:
            xh = torch.from_numpy(synth.make_activations(M, K, seed=92 + M).astype(np.float32)).half()
            full = loader.qmatmul(t, blocks, N, K, xh.float().numpy(), nthreads=4)

            w = nxq.Weight.register_shard(blocks, t, N, K, nxq.SPLIT_COL, rank, world)
            y = torch.empty(M, N // world, dtype=torch.float32, device=dev)
            nxq.tp_qmatmul(w, xh.to(dev), y, nxq.SPLIT_COL)
            torch.cuda.synchronize(dev)
            w.release()
            parts = [torch.zeros(M, N // world) for _ in range(world)]
            dist.all_gather(parts, y.cpu())
            res[("col", M)] = synth.rel_l2(torch.cat(parts, dim=1).numpy(), full)

            k_loc = K // world
            w = nxq.Weight.register_shard(blocks, t, N, K, nxq.SPLIT_ROW, rank, world)
            xs = xh[:, rank * k_loc:(rank + 1) * k_loc].contiguous().to(dev)
            y = torch.empty(M, N, dtype=torch.float32, device=dev)
            nxq.tp_qmatmul(w, xs, y, nxq.SPLIT_ROW)
            torch.cuda.synchronize(dev)
            w.release()
            res[("row", M)] = synth.rel_l2(y.cpu().numpy(), full)
        q.put((rank, res))
    finally:
        if joined:
            nxq.tp_shutdown()
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["fused", "nccl"])
@pytest.mark.parametrize("t", [11, 12], ids=["Q3_K", "Q4_K"])
def test_tp_qmatmul_two_gpus_matches_full(t, mode):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world, N, K, Ms = 2, 1024, 4096, (1, 8, 40)
    procs = [ctx.Process(target=_worker, args=(r, world, port, t, N, K, Ms, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    out = dict(q.get(timeout=5) for _ in range(world))
    for rank in range(world):
        for key, err in out[rank].items():
            assert err < TOL, (rank, key, err)


def _allreduce_worker(rank, world, port, sizes, q):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "nexus-inference-engine-_b200"))
    import datetime

    import torch
    import torch.distributed as dist

    import nxq

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    joined = False
    try:
        os.environ["NXQ_TP_ALLREDUCE"] = "p2p"
        torch.cuda.set_device(rank)
        nxq.init(rank)
        uid = [nxq.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        nxq.tp_init(rank, world, uid[0])
        joined = True
        res = {"p2p": nxq.tp_p2p_enabled()}

        def data(r, n, call):
            g = np.random.default_rng(1000 * r + 7 * call + n)
            return g.standard_normal(n).astype(np.float32)

        for n in sizes:
            for call in range(3):  # three calls: both halves of the buffer, epochs advancing
                buf = torch.from_numpy(data(rank, n, call)).cuda()
                nxq.tp_allreduce_f32(buf)
                nxq.tp_wait(None, 20000)
                got = buf.cpu().numpy()
                want = np.zeros(n, np.float32)
                for r in range(world):  # fp32, in rank order
                    want = (want + data(r, n, call)).astype(np.float32)
                exact = bool(np.array_equal(got, want))
                rel = float(np.abs(got - want).max() / (np.abs(want).max() + 1e-30))
                res[(n, call)] = (exact, rel, float(np.float64(got).sum()))
        # Replayed from a CUDA graph: the epoch is a device counter.
        n = 4096
        s = torch.cuda.Stream()
        bufs = [torch.from_numpy(data(rank, n, 10 + i)).cuda() for i in range(3)]
        keep = [b.clone() for b in bufs]
        with torch.cuda.stream(s):
            nxq.tp_allreduce_f32(bufs[0], stream=s)  # outside capture first
        s.synchronize()
        for b, k in zip(bufs, keep):
            b.copy_(k)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for b in bufs:
                nxq.tp_allreduce_f32(b, stream=s)
        for rep in range(2):
            for b, k in zip(bufs, keep):
                b.copy_(k)
            torch.cuda.synchronize()
            with torch.cuda.stream(s):
                g.replay()
            s.synchronize()
            for i, b in enumerate(bufs):
                want = np.zeros(n, np.float32)
                for r in range(world):
                    want = (want + data(r, n, 10 + i)).astype(np.float32)
                res[("graph", rep, i)] = (bool(np.array_equal(b.cpu().numpy(), want)), 0.0, 0.0)
        del g
        nxq.stream_sync()
        q.put((rank, res))
    finally:
        if joined:
            nxq.tp_shutdown()
        dist.destroy_process_group()


def test_tp_allreduce_peer_memory_two_gpus():
    """nxq_tp_allreduce_f32 on two GPUs with NXQ_TP_ALLREDUCE=p2p: up to 2^21
    values over NVLink peer memory (the same bits as adding the ranks' inputs in rank order in fp32,
    on every rank), beyond that over NCCL (within fp32 rounding); three calls
    per size so both halves of the symmetric buffer and advancing epochs are
    used; and three allreduces captured in a CUDA graph and replayed twice."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 2
    sizes = (1, 1000, 4096, 131072, 524289, 2 ** 21, 2 ** 21 + 5)
    procs = [ctx.Process(target=_allreduce_worker, args=(r, world, port, sizes, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    out = dict(q.get(timeout=5) for _ in range(world))
    for rank in range(world):
        assert out[rank]["p2p"], "peer-memory allreduce not enabled on two NVLink GPUs"
        for key, val in out[rank].items():
            if key == "p2p":
                continue
            exact, rel, _ = val
            if key[0] == "graph" or key[0] <= 2 ** 21:
                assert exact, (rank, key, rel)
            else:
                assert rel < 1e-6, (rank, key, rel)
    for key in out[0]:
        if key != "p2p" and key[0] != "graph":
            assert out[0][key][2] == out[1][key][2], key  # every rank holds the same sum


def _fused_worker(rank, world, port, cases, q, exchange):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "nexus-inference-engine-_b200"))
    import datetime
    import hashlib

    import torch
    import torch.distributed as dist

    import nxq
    from nxq import synth
    from oracle import loader

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    joined = False
    try:
        os.environ["NXQ_TP_ALLREDUCE"] = "fused"
        os.environ["NXQ_TP_EXCHANGE"] = exchange
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        nxq.init(rank)
        uid = [nxq.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        nxq.tp_init(rank, world, uid[0])
        joined = True
        res = {"mode": nxq.tp_p2p_enabled()}
        digest = lambda a: hashlib.sha256(a.tobytes()).hexdigest()
        for t, N, K, Ms in cases:
            blocks = synth.make_blocks(t, N, K, seed=400 + t)
            k_loc = K // world
            w = nxq.Weight.register_shard(blocks, t, N, K, nxq.SPLIT_ROW, rank, world)
            for M in Ms:
                xh = torch.from_numpy(synth.make_activations(M, K, seed=410 + M).astype(np.float32)).half()
                full = loader.qmatmul(t, blocks, N, K, xh.float().numpy(), nthreads=4)
                xs = xh[:, rank * k_loc:(rank + 1) * k_loc].contiguous().to(dev)
                outs = []
                for call in range(3):  # both halves of the exchange buffer, advancing epochs
                    y = torch.full((M, N), float("nan"), dtype=torch.float32, device=dev)
                    nxq.tp_qmatmul(w, xs, y, nxq.SPLIT_ROW)
                    nxq.tp_wait(None, 20000)
                    outs.append(y.cpu().numpy())
                res[(t, N, K, M)] = (synth.rel_l2(outs[0], full),
                                     all(np.array_equal(o, outs[0]) for o in outs), digest(outs[0]))
            if Ms[0] <= 32:
                # Two calls captured in a CUDA graph, replayed twice: the epoch
                # is a device counter, so replays keep exchanging correctly.
                M = Ms[0]
                xh = torch.from_numpy(synth.make_activations(M, K, seed=410 + M).astype(np.float32)).half()
                xs = xh[:, rank * k_loc:(rank + 1) * k_loc].contiguous().to(dev)
                s = torch.cuda.Stream()
                ys = [torch.empty(M, N, dtype=torch.float32, device=dev) for _ in range(2)]
                with torch.cuda.stream(s):
                    nxq.tp_qmatmul(w, xs, ys[0], nxq.SPLIT_ROW, stream=s)  # outside capture first
                s.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for yy in ys:
                        nxq.tp_qmatmul(w, xs, yy, nxq.SPLIT_ROW, stream=s)
                eager = None
                for rep in range(2):
                    for yy in ys:
                        yy.fill_(float("nan"))
                    with torch.cuda.stream(s):
                        g.replay()
                    s.synchronize()
                    got = [yy.cpu().numpy() for yy in ys]
                    eager = eager if eager is not None else got[0]
                    res[("graph", t, N, K, rep)] = all(np.array_equal(a, eager) for a in got)
                del g
                nxq.stream_sync(s)
            w.release()
        q.put((rank, res))
    finally:
        if joined:
            nxq.tp_shutdown()
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["all", "owner"])
def test_tp_row_split_fused_exchange_two_gpus(exchange):
    """NXQ_TP_ALLREDUCE=fused on two GPUs: decode-size ROW calls run as one
    GEMV launch per rank that pushes its partial tiles into the peer's
    exchange buffer over NVLink and sums the ranks' tiles itself (all: every
    rank sums every tile; owner: the owner of a tile, rank t mod 2, sums it
    and sends the sum back, NXQ_TP_EXCHANGE=owner).  Within the
    parity bar of the unsharded oracle (Q4_K and Q3_K; a shape with few row
    tiles and a long K, so stream-K splits tiles across CTAs), the same bits
    on both ranks, the same bits on three consecutive calls and on CUDA-graph
    replays; a prefill-size call (M = 40) takes the GEMM and NCCL path."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 2
    cases = [(12, 1024, 4096, (1, 8, 32)), (11, 4096, 14336, (1, 8, 32)), (12, 14336, 4096, (8,)),
             (12, 1024, 4096, (40,))]
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, cases, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    out = dict(q.get(timeout=5) for _ in range(world))
    for rank in range(world):
        assert out[rank]["mode"] == 2, "fused row split not enabled on two NVLink GPUs"
        for key, val in out[rank].items():
            if key == "mode":
                continue
            if key[0] == "graph":
                assert val, (rank, key)
                continue
            err, repeat, _ = val
            assert err < TOL and repeat, (rank, key, err, repeat)
    for key, val in out[0].items():
        if key != "mode" and key[0] != "graph":
            assert val[2] == out[1][key][2], key  # every rank holds the same bits
