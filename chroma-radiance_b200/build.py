"""Builds libb2g.so (the engine) in-tree with nvcc for sm_100a.

    python chroma-radiance_b200/build.py [--force]

Objects go to chroma-radiance_b200/_build/, the library to chroma-radiance_b200/lib/.
Each .cu is compiled separately (in parallel) and relinked only when a source or header
is newer than the library.
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
REPO = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libb2g.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3", "-I" + str(REPO / "include"), "-I" + str(CSRC),
]


# Per-file extra flags.  model_fastmath.cu reproduces a computation the reference compiles with
# --use_fast_math, and has to be built the same way to give the same values.
FILE_FLAGS = {"model_fastmath.cu": ["--use_fast_math"]}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((REPO / "include").glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    hdrs = headers()
    jobs = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        if force or _stale(obj, [src] + hdrs):
            cmd = [nvcc()] + NVCC_FLAGS + FILE_FLAGS.get(src.name, []) + ["-c", str(src), "-o", str(obj)]
            jobs.append((src, obj, cmd))

    def run(job):
        src, obj, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for msg in ex.map(run, jobs):
            if verbose and msg:
                print(msg, file=sys.stderr)
    objs = [BUILD / (s.stem + ".o") for s in sources()]
    if force or jobs or _stale(LIB, objs):
        # The driver API (tensor-map encoding) is reached through cudaGetDriverEntryPoint,
        # so only the (static) CUDA runtime is linked.
        cmd = [nvcc()] + ARCH + ["-shared", "-o", str(LIB)] + [str(o) for o in objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
