"""Run one quantized-matmul configuration a few times (for ncu captures).

    python nexus-inference-engine-_b200/profile_case.py --type Q4_K --N 14336 --K 4096 --M 1 --iters 3

Registers `--copies` replicas of a seeded synthetic weight (so a capture can
see cold-L2 behaviour) and calls nxq_qmatmul `--iters` times, rotating through
them; prints the kernel name and the CUDA-event time per call.  With --graph R
it also replays a CUDA graph of R back-to-back calls, which removes host launch
overhead from the timing (the per-call events above include it).  Small enough
to be captured with ncu --set full in a minute.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

import numpy as np  # noqa: E402
import torch  # noqa: E402

import nxq  # noqa: E402
from nxq import synth  # noqa: E402


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--type", default="Q4_K")
    ap.add_argument("--N", type=int, default=14336)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--M", type=int, default=1)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--copies", type=int, default=4)
    ap.add_argument("--x-dtype", default="f16", choices=["f16", "bf16", "f32"])
    ap.add_argument("--y-dtype", default="f32", choices=["f16", "bf16", "f32"])
    ap.add_argument("--graph", type=int, default=0, help="launches per replayed CUDA graph (0 = off)")
    a = ap.parse_args()
    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}
    t = nxq.TYPES[a.type]
    nxq.init(0)
    blocks = synth.make_blocks(t, a.N, a.K, seed=1)
    ws = [nxq.Weight.register(blocks, t, a.N, a.K) for _ in range(a.copies)]
    x = torch.randn(a.M, a.K, generator=torch.Generator().manual_seed(2)).to(dt[a.x_dtype]).cuda()
    y = torch.empty(a.M, a.N, dtype=dt[a.y_dtype], device="cuda")
    name = nxq.kernel_name(ws[0], a.M, nxq._dtype_code(x.dtype), nxq._dtype_code(y.dtype))
    times = []
    for i in range(a.iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        nxq.qmatmul(ws[i % len(ws)], x, out=y)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    nxq.stream_sync()
    wb = ws[0].packed_bytes
    nbytes = wb + x.numel() * x.element_size() + y.numel() * y.element_size()
    if a.graph > 0:
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            nxq.qmatmul(ws[0], x, out=y, stream=s)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(a.graph):
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
        us = e0.elapsed_time(e1) * 1e3 / (reps * a.graph)
        print(f"graph: {us:.2f} us/call, {nbytes / (us * 1e-6) / 1e9:.0f} GB/s over {reps}x{a.graph} calls")
        nxq.stream_sync()
    gbs = [nbytes / (us * 1e-6) / 1e9 for us in times]
    print(f"{name} {a.type} N={a.N} K={a.K} M={a.M}: " + ", ".join(f"{u:.1f}us {g:.0f}GB/s" for u, g in zip(times, gbs)))
    for w in ws:
        w.release()
    return 0


if __name__ == "__main__":
    sys.exit(main())
