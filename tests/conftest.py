"""Shared pytest set-up.

Markers: `gpu` tests need a B200 (sm_100a) and call libnxq.so through its C
ABI; everything else runs on the CPU.  GPU tests fail, never skip, when no GPU
is present, so a box without a working GPU cannot pass them silently.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "nexus-inference-engine-_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"
NAMES = {2: "Q4_0", 3: "Q4_1", 8: "Q8_0", 10: "Q2_K", 11: "Q3_K", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}
# The block types of the benchmark configurations.
MAIN_TYPES = [2, 8, 11, 12]
ALL_TYPES = sorted(NAMES)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built libnxq.so")


def golden(type_id: int) -> dict:
    with np.load(GOLDEN / f"golden_{NAMES[type_id]}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def gpu():
    """Initialises nxq on cuda:0 once per session; fails if that is impossible."""
    import torch
    import nxq

    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    torch.cuda.init()
    nxq.init(0)
    yield nxq
