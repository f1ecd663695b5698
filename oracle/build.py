"""Build recipe for the test oracle (test infrastructure, not the product).

    python oracle/build.py [--force]

  oracle/_build/libkvf_oracle.so  the C restatement (oracle/kvf_oracle.c), gcc
  oracle/_ref/libkvf_ref.so       the reference's own host functions
                                  (runtime/kvf_host.h, via oracle/ref_shim.cu),
                                  built only where the reference tree exists

Neither output is committed (.gitignore); both travel with the working tree
to the GPU box, where the reference tree itself is absent. The reference's
own build system (CMake, PowerShell) is not used: the one header needed is
compiled directly, unmodified, from where it lies.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REFERENCE = Path(os.environ.get("KVF_REFERENCE", "/root/reference"))
ORACLE_SO = HERE / "_build" / "libkvf_oracle.so"
REF_SO = HERE / "_ref" / "libkvf_ref.so"


def _stale(out: Path, deps) -> bool:
    return not out.exists() or any(Path(d).stat().st_mtime > out.stat().st_mtime for d in deps)


def _run(cmd) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed: {' '.join(map(str, cmd))}\n{r.stdout}\n{r.stderr}")


def build_oracle(force: bool = False) -> Path:
    src = HERE / "kvf_oracle.c"
    if force or _stale(ORACLE_SO, [src]):
        ORACLE_SO.parent.mkdir(parents=True, exist_ok=True)
        cc = "/usr/bin/gcc" if Path("/usr/bin/gcc").exists() else "gcc"
        _run([cc, "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
              "-fno-fast-math", str(src), "-o", str(ORACLE_SO), "-lm"])
    return ORACLE_SO


def reference_available() -> bool:
    return (REFERENCE / "runtime" / "kvf_host.h").exists()


def build_reference(force: bool = False) -> Path | None:
    """Compile the reference's host functions; None when the tree is absent."""
    if not reference_available():
        return REF_SO if REF_SO.exists() else None
    src = HERE / "ref_shim.cu"
    deps = [src, REFERENCE / "runtime" / "kvf_host.h", REFERENCE / "runtime" / "kvf_kernels.cuh"]
    if force or _stale(REF_SO, deps):
        REF_SO.parent.mkdir(parents=True, exist_ok=True)
        nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
        # Host code only; -ffp-contract=off keeps the quantizer's a*b+c unfused,
        # as on the reference's x86-64 (no FMA) host build.
        _run([nvcc, "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC,-ffp-contract=off",
              "-gencode", "arch=compute_100a,code=sm_100a",
              f"-I{REFERENCE / 'runtime'}", str(src), "-o", str(REF_SO)])
    return REF_SO


def build(force: bool = False) -> None:
    build_oracle(force)
    build_reference(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(ORACLE_SO)
    print(REF_SO if REF_SO.exists() else "reference tree absent: oracle/_ref not built")
