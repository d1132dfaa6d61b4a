"""Build libnxq.so in-tree for sm_100a.

    python nexus-inference-engine-_b200/build.py [--force] [--verbose]

Compiles every csrc/*.cu with nvcc (-gencode arch=compute_100a,code=sm_100a
-lineinfo -O3) into _build/ and links nxq/libnxq.so, the C-ABI library that
include/nxq.h declares.  cudart is linked statically so the library does not
depend on which libcudart the host process loaded first; NCCL is resolved at
run time (csrc/tp.cu).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
OUT = PKG / "nxq" / "libnxq.so"
SHIM_SRC = PKG / "shim" / "compute_dispatch_nxq.cpp"
SHIM_OUT = PKG / "nxq" / "libnxq_dispatch.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _nccl_include() -> list[str]:
    """Header-only use of NCCL types; prefer the copy matching torch's NCCL."""
    cands = []
    try:
        import nvidia.nccl  # type: ignore

        cands.append(Path(list(nvidia.nccl.__path__)[0]) / "include")
    except Exception:
        pass
    cands.append(Path("/usr/include"))
    for c in cands:
        if (c / "nccl.h").exists():
            return [f"-I{c}"]
    raise RuntimeError("nccl.h not found")


def _flags() -> list[str]:
    return ARCH + [
        "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3",
        "-Xptxas", "-warn-spills",
        f"-I{ROOT / 'include'}", f"-I{CSRC}",
    ] + _nccl_include()


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "nxq.h"]


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps, Path(__file__)])


def build(force: bool = False, verbose: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    deps = _headers()
    flags = _flags()
    jobs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        if force or _stale(o, s, deps):
            jobs.append((s, o))

    def compile_one(job):
        s, o = job
        cmd = [nvcc, *flags, "-c", str(s), "-o", str(o)]
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        return s, r

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for s, r in ex.map(compile_one, jobs):
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {s.name}:\n{r.stdout}\n{r.stderr}")
            if verbose and (r.stdout or r.stderr):
                print(r.stdout, r.stderr)
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or jobs or not OUT.exists() or any(o.stat().st_mtime > OUT.stat().st_mtime for o in objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", str(OUT), *map(str, objs), "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_shim(force=force, verbose=verbose)
    return OUT


def build_shim(force: bool = False, verbose: bool = False) -> Path:
    """The C++ ComputeDispatch shim (shim/compute_dispatch_nxq.cpp) as
    nxq/libnxq_dispatch.so, linked against libnxq.so beside it."""
    deps = [SHIM_SRC, SHIM_SRC.with_suffix(".h"), ROOT / "include" / "nxq.h", OUT]
    if not force and SHIM_OUT.exists() and all(p.stat().st_mtime <= SHIM_OUT.stat().st_mtime for p in deps):
        return SHIM_OUT
    cmd = [shutil.which("g++") or "g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra",
           "-o", str(SHIM_OUT), str(SHIM_SRC), f"-I{ROOT / 'include'}", f"-L{OUT.parent}", "-lnxq",
           "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"shim build failed:\n{r.stdout}\n{r.stderr}")
    return SHIM_OUT


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
