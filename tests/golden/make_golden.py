"""Generate the golden fixtures in tests/golden/ from the reference itself.

    make -C oracle ref && python tests/golden/make_golden.py

Every expected value here comes from the reference's own decoders,
nexus/src/import/gguf_importer.cpp compiled from the reference sources into
oracle/_ref/libref_decoders.so (oracle/Makefile), so the fixtures pin both the
oracle restatement (oracle/nxq_oracle.c) and the CUDA path.  Matmul
expectations use the reference CPU path: the reference decoders followed by
fp32 dot products (the closed Accelerate cblas_sgemm of gemm.cpp:16-41 is
restated, so that half is pinned only to its documented semantics).

Per block type golden_<TYPE>.npz holds
  kat_blocks / kat_n / kat_out   known-answer blocks: zero block, fp16 subnormal,
                                 negative and max-magnitude scales, extreme
                                 codes, Inf/NaN scales, and uniformly random
                                 bytes; with the reference's decoded floats
  mat_*                          a ragged weight (N not a multiple of 128, and
                                 for 32-element blocks K not a multiple of 256)
                                 in the benchmark distribution, x ~ N(0,1)
                                 rounded to fp16, and the reference CPU path's y;
                                 mat_w_sha256 hashes the decoded weight bytes.

golden_I4G.npz (NXF INT4 groups, quant/gptq.cpp:9-27) holds, per group size
gs in {32, 64, 128, 256}, flat known-answer arrays g<gs>_codes / _scales /
_zeros (zero, negative, fp32-subnormal, huge, Inf and NaN scales; codes 0 and
15; one set with zeros omitted, g<gs>_nozero_out) and the reference's
nexus::quant::dequant_int4 output g<gs>_out, plus a ragged matrix in the
I4G block form (g<gs>_mat_*) with the reference CPU path's y.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "nexus-inference-engine-_b200"))

from oracle import loader  # noqa: E402
from nxq import synth  # noqa: E402

NAMES = {2: "Q4_0", 3: "Q4_1", 8: "Q8_0", 10: "Q2_K", 11: "Q3_K", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}
OUT = Path(__file__).resolve().parent


def kat_blocks(t: int, seed: int) -> np.ndarray:
    qk, bb = synth.GEOMETRY[t]
    g = synth.rng(seed)
    blocks = []
    halves = [0x0000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0xBC00, 0x7BFF, 0xFBFF, 0x8001, 0x7C00,
              0x7E00, 0x1234]
    fields = synth.HALF_FIELDS[t]
    # Zero block.
    blocks.append(np.zeros(bb, dtype=np.uint8))
    # All-ones and all-0x88 code bytes with each special scale value.
    for fill in (0xFF, 0x88, 0x00, 0x0F, 0xF0):
        for h in halves:
            b = np.full(bb, fill, dtype=np.uint8)
            for off in fields:
                b[off] = h & 0xFF
                b[off + 1] = h >> 8
            blocks.append(b)
    # Random code bytes with ordinary scales, and fully random bytes.
    for i in range(16):
        b = g.integers(0, 256, bb, dtype=np.uint8)
        for off in fields:
            h = synth.half_bits(g.uniform(-2.0, 2.0))
            b[off] = h & 0xFF
            b[off + 1] = h >> 8
        blocks.append(b)
    for i in range(16):
        blocks.append(g.integers(0, 256, bb, dtype=np.uint8))
    return np.concatenate(blocks)


def make_i4g() -> None:
    out = {}
    for gs in (32, 64, 128, 256):
        g = synth.rng(7100 + gs)
        groups = 24
        n = groups * gs
        codes = g.integers(0, 256, n // 2, dtype=np.uint8)
        codes[: gs // 2] = 0x00           # group 0: codes 0
        codes[gs // 2: gs] = 0xFF         # group 1: codes 15
        scales = g.uniform(-4.0, 4.0, groups).astype(np.float32)
        zeros = g.uniform(-2.0, 17.0, groups).astype(np.float32)
        special = np.array([0.0, -0.0, 1e-40, -3.0e38, 3.4e38, np.inf, -np.inf, np.nan, 1.0, -1.0],
                           dtype=np.float32)
        scales[2:2 + special.size] = special
        zeros[12] = np.inf
        zeros[13] = np.nan
        zeros[14] = 0.0
        out[f"g{gs}_codes"] = codes
        out[f"g{gs}_scales"] = scales
        out[f"g{gs}_zeros"] = zeros
        out[f"g{gs}_out"] = loader.dequant_int4(codes, scales, zeros, n, gs, which="ref")
        out[f"g{gs}_nozero_out"] = loader.dequant_int4(codes, scales, None, n, gs, which="ref")
        t = 100 + gs // 32
        N, K = 96, (768 if gs < 256 else 512)
        mb = synth.make_blocks(t, N, K, seed=8100 + gs)
        x = synth.make_activations(4, K, seed=9100 + gs, dtype=np.float16).astype(np.float32)
        out[f"g{gs}_mat_blocks"] = mb
        out[f"g{gs}_mat_N"] = np.int64(N)
        out[f"g{gs}_mat_K"] = np.int64(K)
        out[f"g{gs}_mat_x"] = x
        out[f"g{gs}_mat_y"] = loader.qmatmul(t, mb, N, K, x, which="ref", nthreads=4)
        print(f"I4G{gs}: kat {groups} groups; mat {N} x {K}")
    np.savez_compressed(OUT / "golden_I4G.npz", **out)


def main() -> int:
    loader.build(ref=True)
    if loader.ref() is None:
        print("reference decoders not built (oracle/_ref missing)", file=sys.stderr)
        return 2
    if len(sys.argv) > 1 and sys.argv[1] == "i4g":
        make_i4g()
        return 0
    for t, name in NAMES.items():
        qk, bb = synth.GEOMETRY[t]
        kb = kat_blocks(t, 7000 + t)
        n = kb.size // bb * qk
        kout = loader.dequant(t, kb, n, which="ref")
        N = 200
        K = 544 if qk == 32 else 512
        mb = synth.make_blocks(t, N, K, seed=8000 + t)
        w = loader.dequant(t, mb, N * K, which="ref")
        x = synth.make_activations(4, K, seed=9000 + t, dtype=np.float16).astype(np.float32)
        y = loader.qmatmul(t, mb, N, K, x, which="ref", nthreads=4)
        np.savez_compressed(
            OUT / f"golden_{name}.npz",
            type_id=np.int32(t), kat_blocks=kb, kat_n=np.int64(n), kat_out=kout,
            mat_blocks=mb, mat_N=np.int64(N), mat_K=np.int64(K), mat_x=x, mat_y=y,
            mat_w_sha256=np.array(hashlib.sha256(w.tobytes()).hexdigest()),
        )
        print(name, "kat", kb.size // bb, "blocks; mat", N, "x", K)
    make_i4g()
    return 0


if __name__ == "__main__":
    sys.exit(main())
