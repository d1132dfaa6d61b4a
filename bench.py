#!/usr/bin/env python
"""Benchmark of the dequant-fused quantized matmul (the BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl nxq|reference]
    python bench.py --case Q4_K:14336x4096:M1 [--iters 3 --copies 2 --graph R]   (profiling)

Workload (one "step"): BASELINE.json config 2 - the Q4_K GEMV over a
Llama-3-8B MLP, gate and up (K=4096, N=14336) and down (K=14336, N=4096), at
every decode batch M in {1, 4, 8, 16, 32}: 15 quantized matmuls per step,
fp16 activations, fp32 output, fp32 accumulation.  Weights are synthetic
(seeded; nxq.synth) and HBM-resident; every call of a step reads its own
weight replica and the replicas of a projection span more than 4x the
126 MB L2, so each call streams its weights from HBM.

N = 1: the step on one GPU.  N > 1 (torchrun, one process per GPU): the same
step split tensor-parallel over the N GPUs - gate/up by column, down by row,
its partial outputs summed over the ranks inside the GEMV launch (tiles
exchanged over NVLink peer memory) - so the whole job is fixed as N grows
(strong scaling); the matmuls alone and NCCL allreduces of the same sizes are
also timed on their own (tp_split).

value      = algorithmic bytes of the whole step (packed weight blocks + x + y)
             times K steps over the device time of the K timed steps (CUDA
             events, max over ranks)
e2e        = the same workload through the public host-facing calls with the
             host<->device copies inside the timed region: nxq_qmatmul_host
             (N = 1) or nxq_tp_qmatmul with pinned-host copies (N > 1)
roofline   = the dominant kernel's algorithmic GB/s against the measured HBM
             copy bandwidth in MEASURED_PEAKS.json
prefill    = BASELINE.json config 4: Q4_K GEMM at M in {512, 2048, 8192},
             K=4096, N=14336, bf16 activations and bf16 output, TFLOP/s (N = 1)
config1 / config3 = BASELINE.json configs 1 (Q4_0 GEMV M=1, 4096x4096, fp32 x)
             and 3 (Q8_0 GEMV M=1 over the 7 projections of a Llama-3-8B layer),
             one GPU
tp_config5 = BASELINE.json config 5 (Q3_K 405B-shaped layer, M in {1,8,32}),
             tensor-parallel over the launched ranks (NCCL allreduce after the
             row-split projections); max over ranks; matmuls and allreduces
             also timed on their own
cpu_baseline = the reference's CPU path (its own decoders from
             oracle/_ref when built, else the oracle restatement, plus fp32
             dot products) on a bounded row sample of the same workload

--impl reference times the reference CPU path instead, on rank 0 only.
"""
from __future__ import annotations

import argparse
import csv
import ctypes
import datetime
import io
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "nexus-inference-engine-_b200"))

METRIC = "Q4_K dequant-GEMV achieved HBM GB/s vs ~8 TB/s; prefill GEMM TFLOP/s"
GEMV_MS = [1, 4, 8, 16, 32]
PROJ = [("gate", 4096, 14336), ("up", 4096, 14336), ("down", 14336, 4096)]  # name, K, N
PREFILL_MS = [512, 2048, 8192]
Q4_K = 12
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# The result line goes to a private copy of the original stdout; file
# descriptor 1 itself is pointed at stderr, so banners that native libraries
# write there (NCCL prints its version at communicator set-up) cannot land
# next to the one JSON line.
_RESULT = None


def emit(line: dict) -> None:
    out = _RESULT if _RESULT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def weight_bytes(K: int, N: int) -> int:
    return N * (K // 256) * 144


def call_bytes(M: int, K: int, N: int, x_size: int = 2, y_size: int = 4) -> int:
    return weight_bytes(K, N) + M * K * x_size + M * N * y_size


# ---------------------------------------------------------------- distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return 0, 1, 0
    import torch
    import torch.distributed as dist

    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world <= 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of this GPU's clocks and throttle reasons while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        import torch

        self.proc = None
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            gid = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-i", gid,
                 "-lms", "100"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except Exception as e:  # noqa: BLE001
            log("clock sampling unavailable:", e)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.tmp.flush()
        self.tmp.seek(0)
        rows = [r for r in csv.reader(io.StringIO(self.tmp.read())) if len(r) >= 9]
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(s):
            try:
                return float(s.strip())
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        loaded = [v for v in sm if mx and v >= 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- CPU reference path
def cpu_reference_sample(seconds: float, rows_frac: int = 32, threads: int | None = None) -> dict:
    """The reference CPU path on a row sample of the config-2 workload:
    every projection's first N/rows_frac rows, every M, repeated for ~seconds."""
    from nxq import synth
    from oracle import loader

    kind = "reference" if loader.ref() is not None else "port"
    threads = threads or os.cpu_count() or 1
    cases = []
    for name, K, N in PROJ:
        n_s = N // rows_frac
        blocks = synth.make_blocks(Q4_K, n_s, K, seed=900 + [p[0] for p in PROJ].index(name))
        for M in GEMV_MS:
            x = synth.make_activations(M, K, seed=M, dtype=np.float16).astype(np.float32)
            cases.append((blocks, n_s, K, x, M))
    total_b = 0
    t0 = time.perf_counter()
    reps = 0
    while True:
        for blocks, n_s, K, x, M in cases:
            loader.qmatmul(Q4_K, blocks, n_s, K, x, which="ref" if kind == "reference" else "port",
                           nthreads=threads)
            total_b += call_bytes(M, K, n_s)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": total_b / el / 1e9, "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": (f"config-2 workload on the first 1/{rows_frac} of each projection's rows "
                       f"(gate/up {14336 // rows_frac} rows, down {4096 // rows_frac} rows, all K), "
                       f"M in {GEMV_MS}, {reps} pass(es), {el:.1f} s; decode by "
                       f"{'the reference decoders (gguf_importer.cpp, oracle/_ref)' if kind == 'reference' else 'the oracle restatement'}"
                       " + fp32 dot products"),
            "seconds": el}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return 0
    steps, warmup = args.steps, args.warmup
    from nxq import synth
    from oracle import loader

    kind = "reference" if loader.ref() is not None else "port"
    threads = os.cpu_count() or 1
    rows_frac = 4
    cases = []
    for name, K, N in PROJ:
        n_s = N // rows_frac
        blocks = synth.make_blocks(Q4_K, n_s, K, seed=900 + [p[0] for p in PROJ].index(name))
        for M in GEMV_MS:
            x = synth.make_activations(M, K, seed=M, dtype=np.float16).astype(np.float32)
            cases.append((blocks, n_s, K, x, M))

    def step():
        b = 0
        for blocks, n_s, K, x, M in cases:
            loader.qmatmul(Q4_K, blocks, n_s, K, x, which="ref" if kind == "reference" else "port",
                           nthreads=threads)
            b += call_bytes(M, K, n_s)
        return b

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    tb = sum(step() for _ in range(steps))
    el = time.perf_counter() - t0
    v = tb / el / 1e9
    sample = (f"each step: the config-2 workload on the first 1/{rows_frac} of each projection's rows, "
              f"all K, M in {GEMV_MS}")
    line = {"metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": el / steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "BASELINE config 2: Q4_K GEMV, Llama-3-8B MLP gate/up/down, M in {1,4,8,16,32}",
                       "sample": sample},
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)
    return 0


# ---------------------------------------------------------------- GPU arm
def traffic_lookup(kernel: str, shape_launches: dict):
    """DRAM bytes per launch of `kernel` (dram__bytes_read.sum + write.sum from
    one ncu capture per shape, profiles/dram_traffic.txt), averaged over the
    shapes it ran with in proportion to their launches; None if a shape has no
    capture."""
    p = ROOT / "profiles" / "dram_traffic.txt"
    if not p.exists():
        return None
    table = {}
    for ln in p.read_text().splitlines():
        parts = ln.split()
        if len(parts) >= 3 and not ln.startswith("#"):
            try:
                table[(parts[0], parts[1])] = float(parts[2])
            except ValueError:
                pass
    total, n = 0.0, 0
    for shape, launches in shape_launches.items():
        if (kernel, shape) not in table:
            return None
        total += table[(kernel, shape)] * launches
        n += launches
    return total / n if n else None


def graph_time_ms(issue, stream, replays: int = 3) -> float:
    """Capture `issue()` (launches on `stream`) in a CUDA graph, replay it once
    to warm up, then time `replays` replays with CUDA events on `stream`;
    returns ms per replay."""
    import torch

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        issue()
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record(stream)
        for _ in range(replays):
            g.replay()
        b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / replays
    del g
    return ms


def replicas_for(nbytes: int) -> int:
    """Weight copies whose total exceeds 4x L2, so back-to-back calls stream from HBM."""
    return max(2, -(-4 * L2_BYTES // nbytes) + 1)


def bench_config1(dev, stream, pk) -> dict:
    """Q4_0 GEMV, M=1, K=N=4096, fp32 x and y."""
    import torch

    import nxq
    from nxq import synth

    K = N = 4096
    blocks = synth.make_blocks(2, N, K, seed=1001)
    wb = N * (K // 32) * 18
    R = replicas_for(wb)
    ws = [nxq.Weight.register(blocks, 2, N, K) for _ in range(R)]
    x = torch.randn(1, K, generator=torch.Generator().manual_seed(11), dtype=torch.float32).to(dev)
    y = torch.empty(1, N, dtype=torch.float32, device=dev)

    def issue():
        for w in ws:
            nxq.qmatmul(w, x, out=y, stream=stream)

    with torch.cuda.stream(stream):
        issue()
    stream.synchronize()
    ms = graph_time_ms(issue, stream) / R
    nb = wb + K * 4 + N * 4
    out = {"workload": "BASELINE config 1: Q4_0 GEMV M=1 K=N=4096, fp32 x (converted to f16 in the call), fp32 y",
           "kernel": nxq.kernel_name(ws[0], 1, nxq.F32, nxq.F32), "us_per_call": ms * 1e3,
           "GB/s": nb / (ms / 1e3) / 1e9, "frac_of_hbm": nb / (ms / 1e3) / 1e9 / pk["hbm_gbs"],
           "replicas": R}
    for w in ws:
        w.release()
    return out


def bench_config3(dev, stream, pk) -> dict:
    """Q8_0 GEMV M=1 over the 7 projections of a Llama-3-8B layer."""
    import torch

    import nxq
    from nxq import synth

    projs = [("q", 4096, 4096), ("k", 4096, 1024), ("v", 4096, 1024), ("o", 4096, 4096),
             ("gate", 4096, 14336), ("up", 4096, 14336), ("down", 14336, 4096)]  # name, K, N
    layer_bytes = sum(N * (K // 32) * 34 for _, K, N in projs)
    L = replicas_for(layer_bytes)
    xs = {K: torch.randn(1, K, generator=torch.Generator().manual_seed(K), dtype=torch.float32)
          .to(torch.float16).to(dev) for K in (4096, 14336)}
    ys = {N: torch.empty(1, N, dtype=torch.float32, device=dev) for N in (1024, 4096, 14336)}
    per = {}
    layer = {name: [] for name, _, _ in projs}
    for i, (name, K, N) in enumerate(projs):
        blocks = synth.make_blocks(8, N, K, seed=3000 + i)
        wb = N * (K // 32) * 34
        R = max(L, replicas_for(wb))
        ws = [nxq.Weight.register(blocks, 8, N, K) for _ in range(R)]
        del blocks

        def issue(ws=ws, K=K, N=N):
            for w in ws:
                nxq.qmatmul(w, xs[K], out=ys[N], stream=stream)

        with torch.cuda.stream(stream):
            issue()
        stream.synchronize()
        ms = graph_time_ms(issue, stream) / R
        nb = wb + K * 2 + N * 4
        per[name] = {"us": round(ms * 1e3, 2), "GB/s": round(nb / (ms / 1e3) / 1e9, 1)}
        layer[name] = ws[:L]
        for w in ws[L:]:
            w.release()

    def issue_layer():
        for r in range(L):
            for name, K, N in projs:
                nxq.qmatmul(layer[name][r], xs[K], out=ys[N], stream=stream)

    ms = graph_time_ms(issue_layer, stream) / L
    nb = layer_bytes + sum(K * 2 + N * 4 for _, K, N in projs)

    # The same layer with the projections that share an input grouped:
    # q/k/v and gate/up as one launch each (nxq_qmatmul_grouped), 4 launches.
    yg = {name: torch.empty(1, N, dtype=torch.float32, device=dev) for name, _, N in projs}

    def issue_grouped():
        for r in range(L):
            nxq.qmatmul_grouped([layer[n][r] for n in ("q", "k", "v")], [xs[4096]] * 3,
                                outs=[yg[n] for n in ("q", "k", "v")], stream=stream)
            nxq.qmatmul(layer["o"][r], xs[4096], out=yg["o"], stream=stream)
            nxq.qmatmul_grouped([layer[n][r] for n in ("gate", "up")], [xs[4096]] * 2,
                                outs=[yg[n] for n in ("gate", "up")], stream=stream)
            nxq.qmatmul(layer["down"][r], xs[14336], out=yg["down"], stream=stream)

    with torch.cuda.stream(stream):
        issue_grouped()
    stream.synchronize()
    ms_g = graph_time_ms(issue_grouped, stream) / L

    # The layer with every fused prologue/epilogue: RMSNorm + q/k/v (one
    # normalization kernel + one grouped launch), o with the residual add,
    # gate/up with SwiGLU (one paired launch), down with the residual add:
    # 5 launches doing strictly more than the 7 plain GEMVs above.
    resid = torch.randn(1, 4096, generator=torch.Generator().manual_seed(7), dtype=torch.float32).to(dev)
    normw = torch.rand(4096, generator=torch.Generator().manual_seed(8), dtype=torch.float32).add_(0.5).to(dev)
    hbuf = torch.empty(1, 14336, dtype=torch.float16, device=dev)

    def issue_fused():
        for r in range(L):
            nxq.rmsnorm_qmatmul([layer[n][r] for n in ("q", "k", "v")], resid, normw, 1e-5,
                                outs=[yg[n] for n in ("q", "k", "v")], stream=stream)
            nxq.qmatmul_residual(layer["o"][r], xs[4096], resid, out=resid, stream=stream)
            nxq.qmatmul_swiglu(layer["gate"][r], layer["up"][r], xs[4096], out=hbuf, stream=stream)
            nxq.qmatmul_residual(layer["down"][r], hbuf, resid, out=resid, stream=stream)

    with torch.cuda.stream(stream):
        issue_fused()
    stream.synchronize()
    ms_f = graph_time_ms(issue_fused, stream) / L
    out = {"workload": "BASELINE config 3: Q8_0 GEMV M=1, the 7 projections of a Llama-3-8B layer "
                       "(q/o 4096x4096, k/v 4096->1024, gate/up 4096->14336, down 14336->4096), f16 x, fp32 y",
           "kernel": nxq.kernel_name(layer["q"][0], 1), "per_projection": per,
           "layer_us": ms * 1e3, "layer_GB/s": nb / (ms / 1e3) / 1e9,
           "layer_frac_of_hbm": nb / (ms / 1e3) / 1e9 / pk["hbm_gbs"], "layer_replicas": L,
           "layer_grouped": {"us": ms_g * 1e3, "GB/s": nb / (ms_g / 1e3) / 1e9,
                             "frac_of_hbm": nb / (ms_g / 1e3) / 1e9 / pk["hbm_gbs"], "launches": 4,
                             "how": "q/k/v and gate/up each one nxq_qmatmul_grouped launch"},
           "layer_fused": {"us": ms_f * 1e3, "GB/s": nb / (ms_f / 1e3) / 1e9,
                           "frac_of_hbm": nb / (ms_f / 1e3) / 1e9 / pk["hbm_gbs"], "launches": 5,
                           "how": "RMSNorm + q/k/v (nxq_rmsnorm_qmatmul), o + residual, gate/up + SwiGLU "
                                  "(nxq_qmatmul_swiglu), down + residual (nxq_qmatmul_residual)"}}
    for ws in layer.values():
        for w in ws:
            w.release()
    return out


def bench_swiglu(dev, stream, pk) -> dict:
    """Config-2 gate/up pair (Q4_K, K=4096, N=14336) with the SwiGLU epilogue:
    nxq_qmatmul_swiglu (one launch over both weights) against two plain calls
    (which leave the activation still to do), M in {1, 8, 32}."""
    import torch

    import nxq
    from nxq import synth

    K, N = 4096, 14336
    wb = weight_bytes(K, N)
    R = replicas_for(2 * wb)
    bg = synth.make_blocks(Q4_K, N, K, seed=4100)
    bu = synth.make_blocks(Q4_K, N, K, seed=4101)
    gs = [nxq.Weight.register(bg, Q4_K, N, K) for _ in range(R)]
    us = [nxq.Weight.register(bu, Q4_K, N, K) for _ in range(R)]
    del bg, bu
    cases = {}
    for M in (1, 8, 32):
        x = torch.randn(M, K, generator=torch.Generator().manual_seed(M), dtype=torch.float32).to(torch.float16).to(dev)
        h = torch.empty(M, N, dtype=torch.float16, device=dev)
        yg = torch.empty(M, N, dtype=torch.float32, device=dev)
        yu = torch.empty(M, N, dtype=torch.float32, device=dev)

        def fused(M=M, x=x, h=h):
            for r in range(R):
                nxq.qmatmul_swiglu(gs[r], us[r], x, out=h, stream=stream)

        def plain(x=x, yg=yg, yu=yu):
            for r in range(R):
                nxq.qmatmul(gs[r], x, out=yg, stream=stream)
                nxq.qmatmul(us[r], x, out=yu, stream=stream)

        res = {}
        for name, fn in (("fused", fused), ("two_calls", plain)):
            with torch.cuda.stream(stream):
                fn()
            stream.synchronize()
            ms = graph_time_ms(fn, stream) / R
            res[name] = {"us": round(ms * 1e3, 2), "GB/s": round(2 * wb / (ms / 1e3) / 1e9, 1)}
        cases[f"M{M}"] = res
    for w in gs + us:
        w.release()
    return {"workload": "config-2 gate/up pair, Q4_K K=4096 N=14336, f16 x; fused: h = silu(x Wg^T) * (x Wu^T) "
                        "stored as f16 in one launch; two_calls: the two products only",
            "cases": cases, "replicas": R}


def bench_tp_layer(dev, stream, pk, rank: int, world: int) -> dict:
    """one Llama-3.1-405B-shaped layer with Q3_K weights
    (hidden 16384, FFN 53248, 128 query / 8 KV heads of dim 128), decode M in
    {1, 8, 32}, tensor-parallel over the `world` ranks: q/k/v/gate/up split by
    column (each rank holds N/world rows), o/down split by row (K/world of every
    row) and summed over the ranks by the library (at decode sizes inside the
    GEMV launch, tiles exchanged over NVLink; NXQ_TP_ALLREDUCE=nccl: an NCCL
    allreduce).  Each rank generates its own shard (synthetic data of the
    config's distribution).  The timed step is the layer's 7 row/column-split
    matmuls (attention and SwiGLU are not part of the path), captured in one
    CUDA graph; time = max over ranks.  The 7 matmuls alone and 2 NCCL
    allreduces of the row splits' outputs alone are timed the same way.  Keys
    are flat (M<m>_...) so that records keep them."""
    import torch

    import nxq
    from nxq import synth

    Q3 = 11
    H, F, KV = 16384, 53248, 1024
    projs = [("q", H, H, 0), ("k", H, KV, 0), ("v", H, KV, 0), ("o", H, H, 1),
             ("gate", H, F, 0), ("up", H, F, 0), ("down", F, H, 1)]  # name, K, N, split (0 col, 1 row)
    loc = []
    for name, K, N, split in projs:
        n_l, k_l = (N // world, K) if split == 0 else (N, K // world)
        loc.append((name, k_l, n_l, split))
    shard_bytes = sum(n * (k // 256) * 110 for _, k, n, _ in loc)
    R = max(1, -(-4 * L2_BYTES // shard_bytes))
    if world > 1:
        import torch.distributed as dist

        uid = [nxq.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        nxq.tp_init(rank, world, uid[0])
    weights = {}
    for i, (name, k_l, n_l, split) in enumerate(loc):
        blocks = synth.make_blocks(Q3, n_l, k_l, seed=5000 + 97 * i + rank)
        weights[name] = [nxq.Weight.register(blocks, Q3, n_l, k_l) for _ in range(R)]
        del blocks
    total_b = sum(N * (K // 256) * 110 for _, K, N, _ in projs)
    out = {"workload": "BASELINE config 5: Llama-3.1-405B-shaped layer, Q3_K, decode, 7 projections + "
                       "2 allreduces per step", "tp": world, "layer_weight_bytes": total_b,
           "shard_bytes_per_gpu": shard_bytes, "replicas": R,
           "timing": "CUDA graph of R layer steps, CUDA events, max over ranks"}
    for M in (1, 8, 32):
        x = {k: torch.randn(M, k, generator=torch.Generator().manual_seed(M + k), dtype=torch.float32)
             .to(torch.float16).to(dev) for k in {k_l for _, k_l, _, _ in loc}}
        y = {(name, n_l): torch.empty(M, n_l, dtype=torch.float32, device=dev) for name, _, n_l, _ in loc}

        def issue(x=x, y=y, matmul=True, allreduce=True):
            for r in range(R):
                for name, k_l, n_l, split in loc:
                    w = weights[name][r]
                    if world > 1 and matmul and allreduce:
                        nxq.tp_qmatmul(w, x[k_l], y[(name, n_l)], nxq.SPLIT_ROW if split else nxq.SPLIT_COL,
                                       stream=stream)
                    elif matmul:
                        nxq.qmatmul(w, x[k_l], out=y[(name, n_l)], stream=stream)
                    elif split and world > 1:
                        nxq.tp_allreduce_f32(y[(name, n_l)], stream=stream)

        with torch.cuda.stream(stream):
            issue()
        stream.synchronize()
        barrier(world)
        ms = max_over_ranks(graph_time_ms(issue, stream) / R, world)
        out[f"M{M}_us"] = round(ms * 1e3, 2)
        out[f"M{M}_GBps"] = round(total_b / (ms / 1e3) / 1e9, 1)
        out[f"M{M}_frac_of_hbm_per_gpu"] = round(total_b / world / (ms / 1e3) / 1e9 / pk["hbm_gbs"], 3)
        if world > 1:
            barrier(world)
            ms_mm = max_over_ranks(graph_time_ms(lambda: issue(allreduce=False), stream) / R, world)
            barrier(world)
            ms_ar = max_over_ranks(graph_time_ms(lambda: issue(matmul=False), stream) / R, world)
            out[f"M{M}_matmul_us"] = round(ms_mm * 1e3, 2)
            out[f"M{M}_allreduce_us"] = round(ms_ar * 1e3, 2)
        del x, y
    for ws in weights.values():
        for w in ws:
            w.release()
    if world > 1:
        nxq.tp_shutdown()
    return out


def bench_prefill(dev, stream, pk, pk_kind) -> dict:
    """Q4_K GEMM K=4096 N=14336, bf16 activations and bf16
    output, M in {512, 2048, 8192}; a graph of back-to-back calls rotating
    over weight replicas that together exceed 4x L2.  Flat keys."""
    import torch

    import nxq
    from nxq import synth

    K, N = 4096, 14336
    blocks = synth.make_blocks(Q4_K, N, K, seed=4000)
    R = replicas_for(weight_bytes(K, N))
    ws = [nxq.Weight.register(blocks, Q4_K, N, K) for _ in range(R)]
    del blocks
    out = {"workload": "BASELINE config 4: Q4_K GEMM K=4096 N=14336, bf16 x, bf16 y, fp32 accumulate",
           "unit": "TFLOP/s", "peak_source": f"{pk_kind} bf16_tflops (burst; kernel timed on its own)",
           "replicas": R}
    for M in PREFILL_MS:
        x = torch.randn(M, K, generator=torch.Generator().manual_seed(M), dtype=torch.float32).to(
            torch.bfloat16).to(dev)
        y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        out["kernel"] = nxq.kernel_name(ws[0], M, nxq.BF16, nxq.BF16)
        iters = R if M <= 2048 else 4
        with torch.cuda.stream(stream):
            for i in range(3):
                nxq.qmatmul(ws[i % R], x, out=y, stream=stream)
        stream.synchronize()
        ms = graph_time_ms(lambda: [nxq.qmatmul(ws[i % R], x, out=y, stream=stream) for i in range(iters)],
                           stream) / iters
        tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
        out[f"M{M}_us"] = round(ms * 1e3, 2)
        out[f"M{M}_TFLOPs"] = round(tf, 1)
        out[f"M{M}_frac_of_bf16_burst"] = round(tf / pk["bf16_tflops"], 4)
        del x, y
    nxq.stream_sync()
    for w in ws:
        w.release()
    return out


def time_replays(graphs, stream, steps: int, world: int) -> float:
    """Barrier, then `steps` replays of graphs[s % len(graphs)] between CUDA
    events on `stream`; returns the max over ranks of the elapsed ms."""
    import torch

    barrier(world)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record(stream)
        for s_i in range(steps):
            graphs[s_i % len(graphs)].replay()
        b.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(a.elapsed_time(b), world)


def capture(fn, stream):
    import torch

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    return g


def headline_single(args, dev, stream, pk) -> dict:
    """N = 1: the config-2 step (15 calls) on one GPU.  Every call of a step
    reads its own weight replica: the j-th use of a projection in step graph r
    takes replica (5 r + j) mod R, so within a step no weight is read twice and
    a replica comes back only after R/5 steps (R x 33 MB > 4 x L2)."""
    import torch

    import nxq
    from nxq import synth

    reps = replicas_for(weight_bytes(4096, 14336))
    weights = {}
    for name, K, N in PROJ:
        blocks = synth.make_blocks(Q4_K, N, K, seed=1000 + K + N)
        weights[name] = [nxq.Weight.register(blocks, Q4_K, N, K) for _ in range(reps)]
        del blocks
    xs = {M: {K: torch.randn(M, K, generator=torch.Generator().manual_seed(M * 7 + K), dtype=torch.float32)
              .to(torch.float16).to(dev) for K in (4096, 14336)} for M in GEMV_MS}
    ys = {M: {N: torch.empty(M, N, dtype=torch.float32, device=dev) for N in (4096, 14336)} for M in GEMV_MS}
    calls = [(name, K, N, M) for M in GEMV_MS for name, K, N in PROJ]
    uses = len(GEMV_MS)  # uses of each projection per step
    step_bytes = sum(call_bytes(M, K, N) for _, K, N, M in calls)
    names = {(name, M): nxq.kernel_name(weights[name][0], M, nxq.F16, nxq.F32) for name, K, N, M in calls}

    def step_calls(r):
        for j, M in enumerate(GEMV_MS):
            for name, K, N in PROJ:
                nxq.qmatmul(weights[name][(uses * r + j) % reps], xs[M][K], out=ys[M][N], stream=stream)

    with torch.cuda.stream(stream):
        for r in range(args.warmup):
            step_calls(r)
    stream.synchronize()
    nxq.stream_sync(stream)
    step_graphs = [capture(lambda r=r: step_calls(r), stream) for r in range(reps)]
    with torch.cuda.stream(stream):
        for r in range(args.warmup):
            step_graphs[r % reps].replay()
    torch.cuda.synchronize()

    clocks = ClockSampler(torch.cuda.current_device())
    time.sleep(0.3)
    ms = time_replays(step_graphs, stream, args.steps, 1)
    clk = clocks.stop()
    nxq.stream_sync(stream)
    del step_graphs

    # Per-case device time: a graph of `reps` back-to-back launches of one
    # (projection, M), each on a different replica.
    per_kernel, per_case = {}, {}
    for name, K, N, M in calls:
        g = capture(lambda name=name, K=K, N=N, M=M: [nxq.qmatmul(weights[name][r], xs[M][K], out=ys[M][N],
                                                                  stream=stream) for r in range(reps)], stream)
        with torch.cuda.stream(stream):
            g.replay()
        torch.cuda.synchronize()
        d = time_replays([g], stream, 3, 1)
        del g
        n_l = 3 * reps
        kname = names[(name, M)]
        k = per_kernel.setdefault(kname, {"ms": 0.0, "bytes": 0, "launches": 0, "shapes": {}})
        k["ms"] += d
        k["bytes"] += call_bytes(M, K, N) * n_l
        k["launches"] += n_l
        shp = f"K{K}xN{N}xM{M}"
        k["shapes"][shp] = k["shapes"].get(shp, 0) + n_l
        c = per_case.setdefault(f"{name}_M{M}", {"ms": 0.0, "bytes": 0})
        c["ms"] += d
        c["bytes"] += call_bytes(M, K, N) * n_l
    nxq.stream_sync(stream)
    total_k = sum(k["ms"] for k in per_kernel.values())
    dom_name, dom = max(per_kernel.items(), key=lambda kv: kv[1]["ms"])
    achieved = dom["bytes"] / (dom["ms"] / 1e3) / 1e9
    roofline = {"bound": "hbm", "kernel": dom_name, "achieved": achieved, "peak": pk["hbm_gbs"],
                "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                "traffic": traffic_lookup(dom_name, dom["shapes"]),
                "peak_source": "hbm_gbs of MEASURED_PEAKS.json (burst copy)", "share_of_step": dom["ms"] / total_k,
                "algorithmic_bytes_per_launch": dom["bytes"] / dom["launches"],
                "avg_launch_us": dom["ms"] / dom["launches"] * 1e3, "shapes": sorted(dom["shapes"]),
                "timing": "CUDA events on the launching stream around graph replays of back-to-back "
                          "launches of each shape on distinct weight replicas (PDL overlap included)"}

    e2e = None
    if not args.no_e2e:
        hx = {M: {K: torch.randn(M, K, generator=torch.Generator().manual_seed(M + K)).to(torch.float16)
                  .float().pin_memory().numpy() for K in (4096, 14336)} for M in GEMV_MS}
        hy = {M: {N: torch.empty(M, N, dtype=torch.float32).pin_memory().numpy() for N in (4096, 14336)}
              for M in GEMV_MS}
        counter = [0]

        def host_step():
            r = counter[0]
            for j, M in enumerate(GEMV_MS):
                for name, K, N in PROJ:
                    nxq.qmatmul_host(weights[name][(uses * r + j) % reps], hx[M][K], out=hy[M][N])
            counter[0] += 1

        for _ in range(2):
            host_step()
        nxq.stream_sync()
        e2e_steps = max(3, min(args.steps, 20))
        e2e_bytes = sum(call_bytes(M, K, N, x_size=4) for _, K, N, M in calls)
        h2d = sum(M * K * 4 for _, K, N, M in calls)
        d2h = sum(M * N * 4 for _, K, N, M in calls)
        # Python loop (ctypes overhead between the calls), for comparison.
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            host_step()
        el_py = time.perf_counter() - t0
        # The headline: the same calls issued from C++ (the engine's side of
        # the C ABI), timed there.
        seq = [(weights[name][(uses * r + j) % reps], hx[M][K], hy[M][N], M)
               for r in range(e2e_steps) for j, M in enumerate(GEMV_MS) for name, K, N in PROJ]
        n = len(seq)
        W = (ctypes.c_void_p * n)(*[w.handle.value for w, _, _, _ in seq])
        X = (ctypes.c_void_p * n)(*[x.ctypes.data for _, x, _, _ in seq])
        Y = (ctypes.c_void_p * n)(*[y.ctypes.data for _, _, y, _ in seq])
        MS = (ctypes.c_int64 * n)(*[M for _, _, _, M in seq])
        sec = ctypes.c_double(0.0)
        hs = nxq.dispatch_lib().nxq_dispatch_host_steps
        hs.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_double)]
        hs.restype = ctypes.c_int
        rc = hs(W, X, Y, MS, n, 1, ctypes.byref(sec))
        if rc != 0:
            raise RuntimeError(f"nxq_dispatch_host_steps failed ({rc}): {nxq.last_error()}")
        el = sec.value
        e2e = {"value": e2e_bytes * e2e_steps / el / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "pcie_GBps": (h2d + d2h) * e2e_steps / el / 1e9,
               "api": "nxq_qmatmul_host (fp32 host x/y, weights resident), one synchronous call per matmul, "
                      "issued from C++ (nxq_dispatch_host_steps in the engine-side shim library)",
               "steps": e2e_steps, "ms_per_step": el / e2e_steps * 1e3,
               "python_loop_GBps": e2e_bytes * e2e_steps / el_py / 1e9,
               "timing": "wall clock around the steps (host call returns after its result is in host memory)"}

    for ws in weights.values():
        for w in ws:
            w.release()
    torch.cuda.empty_cache()
    return {"value": step_bytes * args.steps / (ms / 1e3) / 1e9, "ms": ms, "step_bytes": step_bytes,
            "launches": len(calls) * args.steps, "clocks": clk, "roofline": roofline, "e2e": e2e,
            "kernels": {k: {"launches": v["launches"], "ms": round(v["ms"], 3),
                            "GB/s": round(v["bytes"] / (v["ms"] / 1e3) / 1e9, 1),
                            "share": round(v["ms"] / total_k, 4)} for k, v in per_kernel.items()},
            "per_case_GBps": {k: round(v["bytes"] / (v["ms"] / 1e3) / 1e9, 1) for k, v in per_case.items()},
            "l2": f"inputs larger than L2: {reps} weight replicas per projection "
                  f"({reps * weight_bytes(4096, 14336) / 2**20:.0f} MiB each); every call of a step reads "
                  f"its own replica",
            "parallelism": "single GPU", "scaling": "strong"}


def headline_tp(args, dev, stream, pk, rank: int, world: int) -> dict:
    """N > 1: the same config-2 step split over the ranks the way the north
    star splits a layer: gate and up by column (rank r computes rows
    [r N/T, (r+1) N/T) of y), down by row (rank r holds K/T of every row,
    takes its K/T slice of the activations - the slice of SwiGLU(gate, up) it
    computed itself - and the partial outputs are summed by the library's NCCL
    allreduce).  Strong scaling: the whole job is the unsharded step, value =
    its bytes over the time (max over ranks).  Also timed on their own, in
    graphs of the same calls: the matmuls without the allreduces, and the five
    allreduces (one per M) without the matmuls."""
    import torch
    import torch.distributed as dist

    import nxq
    from nxq import synth

    uid = [nxq.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    nxq.tp_init(rank, world, uid[0])
    tp_mode = nxq.tp_p2p_enabled()
    # name, K, N, split; the shard's local K and N.
    proj = [(name, K, N, nxq.SPLIT_ROW if name == "down" else nxq.SPLIT_COL) for name, K, N in PROJ]
    loc = {name: ((K, N // world) if sp == nxq.SPLIT_COL else (K // world, N)) for name, K, N, sp in proj}
    shard_b = {name: weight_bytes(k, n) for name, (k, n) in loc.items()}
    reps = replicas_for(min(shard_b.values()))
    weights = {}
    for i, (name, K, N, sp) in enumerate(proj):
        k, n = loc[name]
        blocks = synth.make_blocks(Q4_K, n, k, seed=2000 + 97 * i + rank)
        weights[name] = [nxq.Weight.register(blocks, Q4_K, n, k) for _ in range(reps)]
        del blocks
    xs = {M: {name: torch.randn(M, loc[name][0], generator=torch.Generator().manual_seed(M * 7 + loc[name][0] + rank),
                                dtype=torch.float32).to(torch.float16).to(dev) for name, _, _, _ in proj}
          for M in GEMV_MS}
    ys = {M: {name: torch.empty(M, loc[name][1], dtype=torch.float32, device=dev) for name, _, _, _ in proj}
          for M in GEMV_MS}
    uses = len(GEMV_MS)
    calls = [(name, K, N, sp, M) for M in GEMV_MS for name, K, N, sp in proj]
    step_bytes = sum(call_bytes(M, K, N) for _, K, N, _, M in calls)

    def step_calls(r, allreduce=True, matmul=True):
        for j, M in enumerate(GEMV_MS):
            for name, K, N, sp in proj:
                w = weights[name][(uses * r + j) % reps]
                if matmul and allreduce:
                    nxq.tp_qmatmul(w, xs[M][name], ys[M][name], sp, stream=stream)
                elif matmul:
                    nxq.qmatmul(w, xs[M][name], out=ys[M][name], stream=stream)
                elif sp == nxq.SPLIT_ROW:
                    nxq.tp_allreduce_f32(ys[M][name], stream=stream)

    with torch.cuda.stream(stream):
        for r in range(args.warmup):
            step_calls(r)
    stream.synchronize()
    nxq.stream_sync(stream)
    barrier(world)
    graphs = [capture(lambda r=r: step_calls(r), stream) for r in range(reps)]
    with torch.cuda.stream(stream):
        for r in range(args.warmup):
            graphs[r % reps].replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    time.sleep(0.3)
    ms = time_replays(graphs, stream, args.steps, world)
    clk = clocks.stop()
    del graphs
    mm_graphs = [capture(lambda r=r: step_calls(r, allreduce=False), stream) for r in range(reps)]
    ms_mm = time_replays(mm_graphs, stream, args.steps, world)
    del mm_graphs
    ar_graph = capture(lambda: step_calls(0, matmul=False), stream)
    with torch.cuda.stream(stream):
        ar_graph.replay()
    ms_ar = time_replays([ar_graph], stream, args.steps, world)
    del ar_graph
    nxq.stream_sync(stream)

    e2e = None
    if not args.no_e2e:
        # Through the public API as a caller would: each step copies this
        # rank's activations from pinned host memory, issues the 15
        # nxq_tp_qmatmul calls, and reads every output back to pinned host
        # memory; timed on the host, max over ranks.
        hx = {M: {name: xs[M][name].cpu().pin_memory() for name, _, _, _ in proj} for M in GEMV_MS}
        hy = {M: {name: torch.empty_like(ys[M][name], device="cpu").pin_memory() for name, _, _, _ in proj}
              for M in GEMV_MS}
        counter = [0]

        def host_step():
            r = counter[0]
            with torch.cuda.stream(stream):
                for j, M in enumerate(GEMV_MS):
                    for name, K, N, sp in proj:
                        xs[M][name].copy_(hx[M][name], non_blocking=True)
                    for name, K, N, sp in proj:
                        nxq.tp_qmatmul(weights[name][(uses * r + j) % reps], xs[M][name], ys[M][name], sp,
                                       stream=stream)
                    for name, K, N, sp in proj:
                        hy[M][name].copy_(ys[M][name], non_blocking=True)
            stream.synchronize()
            counter[0] += 1

        for _ in range(2):
            host_step()
        nxq.stream_sync(stream)
        e2e_steps = max(3, min(args.steps, 20))
        barrier(world)
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            host_step()
        el = max_over_ranks(time.perf_counter() - t0, world)
        h2d = sum(xs[M][name].numel() * 2 for M in GEMV_MS for name, _, _, _ in proj)
        d2h = sum(ys[M][name].numel() * 4 for M in GEMV_MS for name, _, _, _ in proj)
        e2e = {"value": step_bytes * e2e_steps / el / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
               "api": "nxq_tp_qmatmul per projection (f16 activations copied from pinned host memory, "
                      "fp32 outputs copied back), all ranks", "steps": e2e_steps,
               "ms_per_step": el / e2e_steps * 1e3,
               "timing": "wall clock around the steps, max over ranks"}

    for ws in weights.values():
        for w in ws:
            w.release()
    nxq.tp_shutdown()
    torch.cuda.empty_cache()
    return {"value": step_bytes * args.steps / (ms / 1e3) / 1e9, "ms": ms, "step_bytes": step_bytes,
            "launches": len(calls) * args.steps, "clocks": clk, "e2e": e2e,
            "roofline": {"bound": "hbm", "kernel": "mma_gemv (tensor-parallel shards)",
                         "achieved": step_bytes / world * args.steps / (ms_mm / 1e3) / 1e9,
                         "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": step_bytes / world * args.steps / (ms_mm / 1e3) / 1e9 / pk["hbm_gbs"],
                         "traffic": None,
                         "timing": "per-GPU bytes of the step's matmuls over their time without the allreduces"},
            "tp_split": {"matmul_us_per_step": round(ms_mm / args.steps * 1e3, 2),
                         "allreduce_us_per_step": round(ms_ar / args.steps * 1e3, 2),
                         "step_us": round(ms / args.steps * 1e3, 2), "allreduces_per_step": len(GEMV_MS),
                         "allreduce_bytes": [M * 4096 * 4 for M in GEMV_MS],
                         "row_reduction": tp_mode_name(tp_mode),
                         "reduction_us_per_step": round((ms - ms_mm) / args.steps * 1e3, 2),
                         "how": "matmul_us: the step's matmuls alone; allreduce_us: NCCL allreduces of the "
                                "down outputs alone; reduction_us = step_us - matmul_us, the cost of the "
                                "row_reduction the step used"},
            "l2": f"inputs larger than L2: {reps} replicas of each shard per rank; every call of a step reads its "
                  f"own replica",
            "parallelism": f"tp{world}: gate/up column split, down row split summed by "
                           f"{tp_mode_name(tp_mode)} (fp32)",
            "scaling": "strong"}


def tp_mode_name(mode: int) -> str:
    return {0: "NCCL allreduce", 1: "peer-memory allreduce",
            2: "the fused GEMV tile exchange over NVLink (NCCL allreduce for prefill sizes)"}.get(mode, str(mode))


def run_gpu_arm(args, rank, world, local):
    import torch

    import nxq

    torch.cuda.set_device(local)
    nxq.init(local)
    pk, pk_kind = peaks()
    dev = torch.device("cuda", local)
    stream = torch.cuda.Stream(device=dev)

    head = headline_single(args, dev, stream, pk) if world == 1 else headline_tp(args, dev, stream, pk, rank, world)

    # --- prefill GEMM (config 4) ------------------------------------------------
    prefill = None
    if not args.no_prefill and world == 1:
        prefill = bench_prefill(dev, stream, pk, pk_kind)

    # --- configs 1 and 3 (one GPU), config 5 (tensor parallel over the ranks) -------
    extra = {}
    if not args.no_configs:
        if world == 1:
            extra["config1"] = bench_config1(dev, stream, pk)
            extra["config3"] = bench_config3(dev, stream, pk)
            extra["swiglu_gate_up"] = bench_swiglu(dev, stream, pk)
        extra["tp_config5"] = bench_tp_layer(dev, stream, pk, rank, world)
        torch.cuda.empty_cache()

    # --- CPU baseline (rank 0, N=1) -------------------------------------------------
    cpu = None
    if world == 1 and not args.no_cpu:
        cpu = cpu_reference_sample(args.cpu_seconds)

    if rank == 0:
        workload = ("BASELINE config 2: Q4_K GEMV over a Llama-3-8B MLP, gate/up K=4096 N=14336 and down "
                    "K=14336 N=4096, M in {1,4,8,16,32}; 15 calls per step")
        if world > 1:
            workload += f", tensor-parallel over {world} GPUs (the whole step is the unit of work)"
        line = {
            "metric": METRIC, "value": head["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms"] / args.steps, "higher_is_better": True,
            "scaling": head["scaling"], "vs_baseline": None, "dtype": "f16", "accumulate": "f32",
            "data": "synthetic",
            "config": {"workload": workload,
                       "weights": "Q4_K, d/dmin fp16 U(1e-4,1e-3), codes uniform (seeded)",
                       "x": "fp16 N(0,1)", "y": "fp32", "l2": head["l2"], "parallelism": head["parallelism"]},
            "roofline": head["roofline"], "gpu_launches": head["launches"], "clocks": head["clocks"],
            "e2e": head["e2e"], "prefill": prefill, "cpu_baseline": cpu,
            "nominal_hbm_frac": head["value"] / world / 8000.0,
        }
        for k in ("kernels", "per_case_GBps", "tp_split"):
            if k in head:
                line[k] = head[k]
        line.update(extra)
        emit(line)
    return 0


# ---------------------------------------------------------------- one case (profiling)
def run_case(args) -> int:
    """One quantized-matmul configuration run a few times, small enough for an
    ncu capture: --case TYPE:NxK:M (e.g. Q4_K:14336x4096:M1).  Registers
    --copies replicas of a seeded synthetic weight (a capture then sees cold
    L2), calls nxq_qmatmul --iters times rotating through them and prints the
    kernel name and the CUDA-event time of each call; with --graph R it also
    replays a CUDA graph of R back-to-back calls (no host launch overhead).
    Prints to stderr; the one JSON line is not emitted in this mode."""
    import torch

    import nxq
    from nxq import synth

    try:
        tname, shape, mtxt = args.case.split(":")
        N, K = (int(v) for v in shape.lower().split("x"))
        M = int(mtxt.lstrip("Mm"))
    except ValueError:
        log(f"--case wants TYPE:NxK:M, e.g. Q4_K:14336x4096:M1 (got {args.case!r})")
        return 2
    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}
    t = nxq.TYPES[tname]
    nxq.init(0)
    blocks = synth.make_blocks(t, N, K, seed=1)
    ws = [nxq.Weight.register(blocks, t, N, K) for _ in range(args.copies)]
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(2)).to(dt[args.x_dtype]).cuda()
    y = torch.empty(M, N, dtype=dt[args.y_dtype], device="cuda")
    name = nxq.kernel_name(ws[0], M, nxq._dtype_code(x.dtype), nxq._dtype_code(y.dtype))
    times = []
    for i in range(args.iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        nxq.qmatmul(ws[i % len(ws)], x, out=y)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    nxq.stream_sync()
    nbytes = ws[0].packed_bytes + x.numel() * x.element_size() + y.numel() * y.element_size()
    if args.graph > 0:
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            nxq.qmatmul(ws[0], x, out=y, stream=s)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(args.graph):
                nxq.qmatmul(ws[i % len(ws)], x, out=y, stream=s)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * args.graph)
        log(f"graph: {us:.2f} us/call, {nbytes / (us * 1e-6) / 1e9:.0f} GB/s over {reps}x{args.graph} calls")
        del g
        nxq.stream_sync()
    gbs = [nbytes / (us * 1e-6) / 1e9 for us in times]
    log(f"{name} {tname} N={N} K={K} M={M}: " + ", ".join(f"{u:.1f}us {g:.0f}GB/s" for u, g in zip(times, gbs)))
    for w in ws:
        w.release()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["nxq", "reference"], default="nxq")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip configs 1, 3 and 5")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--case", default=None,
                    help="profiling mode: run one TYPE:NxK:M case (e.g. Q4_K:14336x4096:M1) and exit")
    ap.add_argument("--iters", type=int, default=3, help="--case: timed single calls")
    ap.add_argument("--copies", type=int, default=4, help="--case: weight replicas")
    ap.add_argument("--x-dtype", default="f16", choices=["f16", "bf16", "f32"], help="--case: activations")
    ap.add_argument("--y-dtype", default="f32", choices=["f16", "bf16", "f32"], help="--case: output")
    ap.add_argument("--graph", type=int, default=0, help="--case: launches per replayed CUDA graph (0 = off)")
    args = ap.parse_args()
    if args.case:
        return run_case(args)
    global _RESULT
    sys.stdout.flush()
    _RESULT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.warmup < 3:
        log("warmup raised to 3 (minimum)")
        args.warmup = 3
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        return run_reference_arm(args, rank, world)
    rank, world, local = dist_setup()
    try:
        return run_gpu_arm(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
