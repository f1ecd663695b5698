"""Builds the package's native artefacts in-tree with nvcc (no JIT cache).

    python -m kvforge_b200.build            # library + probe
    python -m kvforge_b200.build --force

Outputs (git-ignored, shipped with the working tree):
    kvforge_b200/_lib/libkvforge_b200.so   the C-ABI library (include/kvforge_b200.h)
    kvforge_b200/_bin/kvf_bw_probe         the B200 machine probe
Every CUDA source is compiled for sm_100a only.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "kvforge_b200"
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "_lib" / "libkvforge_b200.so"
PROBE = PKG / "_bin" / "kvf_bw_probe"
OBJ = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}"]
LIB_SOURCES = ["decode.cu", "registry.cu", "quantize.cu", "exchange.cu"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")


def _deps(src: Path) -> list[Path]:
    return [src] + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build_library(force: bool = False) -> Path:
    OBJ.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    objs = []
    jobs = []
    for name in LIB_SOURCES:
        src = CSRC / name
        obj = OBJ / (name + ".o")
        objs.append(obj)
        if force or _stale(obj, _deps(src)):
            jobs.append([nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=len(jobs)) as ex:
            list(ex.map(_run, jobs))
    if force or jobs or _stale(LIB, objs):
        _run([nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs)])
    return LIB


def build_probe(force: bool = False) -> Path:
    PROBE.parent.mkdir(parents=True, exist_ok=True)
    src = CSRC / "bw_probe.cu"
    if force or _stale(PROBE, _deps(src)):
        _run([nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", f"-I{INCLUDE}", str(src), "-o", str(PROBE)])
    return PROBE


def build(force: bool = False) -> None:
    build_library(force)
    build_probe(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(LIB)
    print(PROBE)
