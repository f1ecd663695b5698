"""Build recipe for the test oracle (test infrastructure, not the product).

    python oracle/build.py [--force]

  oracle/_build/libkvf_oracle.so  the C restatement (oracle/kvf_oracle.c), gcc
  oracle/_ref/libkvf_ref.so       the reference's own host functions
                                  (runtime/kvf_host.h, via oracle/ref_shim.cu),
                                  built only where the reference tree exists
  oracle/_ref/harness/            the reference's own harnesses built against
                                  this library's drop-in headers (include/):
                                  kvf_driver_<plan> (runtime/kvf_driver.cu with
                                  each plan the reference's compiler emitted
                                  under results/plans/, and one plan emitted by
                                  kvforge_b200.codegen), kvf_sweep
                                  (bench/sweep.cu over the dispatch tables
                                  kvforge_b200.codegen emits) and the plans
                                  file the sweep test times
  oracle/_ref/kvf                 the reference's compiler CLI (src/*.cpp,
                                  g++), for the machine-file and planner
                                  round trip on kvforge_b200/machines/

None of the outputs is committed (.gitignore); all travel with the working
tree to the GPU box, where the reference tree itself is absent. The
reference's own build system (CMake, PowerShell) is not used: the few files
needed are compiled directly, unmodified, from where they lie.

The reference tree is found through the KVF_REFERENCE environment variable,
else BASELINE.json's "reference_path"; without either, only the restatement
is built.
"""
from __future__ import annotations

import csv
import json
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
ORACLE_SO = HERE / "_build" / "libkvf_oracle.so"
REF_SO = HERE / "_ref" / "libkvf_ref.so"
HARNESS = HERE / "_ref" / "harness"


def reference_root() -> Path | None:
    env = os.environ.get("KVF_REFERENCE")
    if env:
        return Path(env)
    baseline = REPO / "BASELINE.json"
    if baseline.exists():
        p = json.loads(baseline.read_text()).get("reference_path")
        if p:
            return Path(p)
    return None


REFERENCE = reference_root()


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
    return REFERENCE is not None and (REFERENCE / "runtime" / "kvf_host.h").exists()


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


# The sweep test times a few plans of this reference shape for every kind of
# variant id (format x order x residency), taken from the reference's own
# candidate list.
SWEEP_SHAPE = "gqa4_8k"
SWEEP_PER_KIND = 2
# A plan kvforge_b200.codegen emits (cost-model choice of splits and kernel
# path) for the reference driver: the Llama-3-70B-shape batch cut to 4
# sequences of 4096 tokens, int8 groups of 64, token-major pages of 16.
CODEGEN_PLAN = dict(name="llama3_70b_b4_n4096", B=4, H=64, Hkv=8, d=128, n=4096, fmt=1, group=64, order=1,
                    paged=True, block_tokens=16)


def _overlay(links: dict) -> Path:
    """A temporary directory of symbolic links, so that a reference source
    that includes "kvf_kernels.cuh" next to itself finds this library's
    drop-in header instead of the reference's kernels."""
    d = Path(tempfile.mkdtemp(prefix="kvf_harness_"))
    for name, target in links.items():
        (d / name).symlink_to(Path(target).resolve())
    return d


def build_harnesses(force: bool = False) -> list:
    """Compile the reference's driver and sweep harnesses, unmodified, against
    include/ and libkvforge_b200.so. Returns the binaries built (or found)."""
    if not reference_available():
        return sorted(HARNESS.glob("kvf_*")) if HARNESS.exists() else []
    lib = REPO / "kvforge_b200" / "_lib" / "libkvforge_b200.so"
    if not lib.exists():
        return []
    HARNESS.mkdir(parents=True, exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    inc = REPO / "include"
    common = {
        "kvf_kernels.cuh": inc / "kvf_kernels.cuh",
        "kvforge_b200.h": inc / "kvforge_b200.h",
        "kvf_host.h": REFERENCE / "runtime" / "kvf_host.h",
        "kvf_registry.h": REFERENCE / "runtime" / "kvf_registry.h",
    }
    cflags = [nvcc, "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler",
              "-ffp-contract=off"]
    lflags = ["-L", str(lib.parent), "-lkvforge_b200", "-Xlinker", "-rpath,$ORIGIN/../../../kvforge_b200/_lib"]
    deps_common = [lib, *common.values()]
    built = []

    # Drivers: runtime/kvf_driver.cu with one emitted plan each.
    plans = []
    for info in sorted((REFERENCE / "results" / "plans").glob("*/plan_info.h")):
        name = info.parent.name
        src = info.parent / f"decode_{name}.cu"
        if src.exists():
            plans.append((name, info, src))
    # Emitted sources are kept (written only when their text changes), so an
    # unchanged emission does not trigger a rebuild.
    gen_dir = HARNESS / "gen"
    gen_dir.mkdir(exist_ok=True)

    def emit(fname: str, text: str) -> Path:
        path = gen_dir / fname
        if not path.exists() or path.read_text() != text:
            path.write_text(text)
        return path

    sys.path.insert(0, str(REPO))
    from kvforge_b200 import codegen

    p = codegen.plan(**CODEGEN_PLAN)
    src = emit(f"decode_{p.name}.cu", codegen.emit_kernel_source(p))
    info = emit(f"plan_info_{p.name}.h", codegen.emit_plan_header(p))
    plans.append((f"codegen_{p.name}", info, src))
    for name, info, src in plans:
        out = HARNESS / f"kvf_driver_{name}"
        deps = deps_common + [REFERENCE / "runtime" / "kvf_driver.cu", info, src]
        if force or _stale(out, deps):
            ov = _overlay({**common, "kvf_driver.cu": REFERENCE / "runtime" / "kvf_driver.cu",
                           "plan_info.h": info, src.name: src})
            try:
                _run(cflags + [f"-I{ov}", f"-I{inc}", str(ov / "kvf_driver.cu"), str(ov / src.name), "-o",
                               str(out)] + lflags)
            finally:
                shutil.rmtree(ov, ignore_errors=True)
        built.append(out)

    # Sweep: bench/sweep.cu over the emitted sm_100a dispatch tables.
    tables = [emit(fname, text) for fname, text in codegen.emit_dispatch_sources()]
    out = HARNESS / "kvf_sweep"
    if force or _stale(out, deps_common + [REFERENCE / "bench" / "sweep.cu", *tables]):
        ov = _overlay({**common, "sweep.cu": REFERENCE / "bench" / "sweep.cu", **{t.name: t for t in tables}})
        try:
            _run(cflags + [f"-I{ov}", f"-I{inc}", str(ov / "sweep.cu"), *[str(ov / t.name) for t in tables],
                           "-o", str(out)] + lflags)
        finally:
            shutil.rmtree(ov, ignore_errors=True)
    built.append(out)

    # The plans the sweep test times.
    src_csv = REFERENCE / "results" / "plans" / SWEEP_SHAPE / "plans.csv"
    sel = HARNESS / f"plans_{SWEEP_SHAPE}.csv"
    if src_csv.exists() and (force or _stale(sel, [src_csv])):
        with open(src_csv, newline="") as f:
            rows = list(csv.reader(f))
        head, body = rows[0], rows[1:]
        col = {h: i for i, h in enumerate(head)}
        picked = {}  # kind -> [(split/pack/page configuration, row)], distinct configurations
        for r in body:
            kind = (r[col["fmt"]], r[col["order"]], r[col["residency"]])
            cfg = (r[col["splits"]], r[col["gqa_pack"]], r[col["block_tokens"]])
            lst = picked.setdefault(kind, [])
            if len(lst) < SWEEP_PER_KIND and all(cfg != c for c, _ in lst):
                lst.append((cfg, r))
        keep = [r for lst in picked.values() for _, r in lst]
        with open(sel, "w", newline="") as f:
            csv.writer(f, lineterminator="\n").writerows([head] + keep)
    return built


# The reference's own decode kernels (its SIMT decode_partial + decode_merge,
# runtime/kvf_kernels.cuh, compiled unmodified for sm_100a) in its driver, on
# the five benchmark shapes, two split counts each: the CUDA-core baseline on
# the same GPU. Config 3's ragged lengths become the uniform length with the
# same total tokens (the reference has one n per batch); data is the
# reference's own make_data (N(0,1)), as its driver generates it.
REFGPU_PLANS = [
    # name, B, H, Hkv, d, n, fmt, group, order, block_tokens, pack g, splits
    ("cfg1_mha_b1_n4096_f16_hm", 1, 32, 32, 128, 4096, 0, 0, 0, 0, 1, (8, 16)),
    ("cfg2_gqa_b1_n32768_int8g64_tm", 1, 32, 8, 128, 32768, 1, 64, 1, 0, 4, (64, 128)),
    ("cfg3_gqa_b8_n5637_f16_tm_p16", 8, 32, 8, 128, 5637, 0, 0, 1, 16, 4, (8, 16)),
    ("cfg4_gqa_b1_n65536_int4g32_hm", 1, 32, 8, 128, 65536, 2, 32, 0, 0, 4, (64, 128)),
    ("cfg5_gqa_b64_n16384_int8g64_tm_p16", 64, 64, 8, 128, 16384, 1, 64, 1, 16, 8, (1, 2)),
]


def build_refgpu(force: bool = False) -> list:
    """kvf_refgpu_<plan>_s<splits>: runtime/kvf_driver.cu with the reference's
    own kvf_kernels.cuh (no file of this library involved), for sm_100a."""
    if not reference_available():
        return sorted(HARNESS.glob("kvf_refgpu_*")) if HARNESS.exists() else []
    HARNESS.mkdir(parents=True, exist_ok=True)
    gen_dir = HARNESS / "gen"
    gen_dir.mkdir(exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    rt = REFERENCE / "runtime"
    fmt_enum = {0: "kvf::FMT_F16", 1: "kvf::FMT_INT8", 2: "kvf::FMT_INT4"}
    ord_enum = {0: "kvf::ORD_HEAD", 1: "kvf::ORD_TOKEN"}
    built = []
    for name, B, H, Hkv, d, n, fmt, group, order, bt, g, splits_list in REFGPU_PLANS:
        for s in splits_list:
            tag = f"{name}_s{s}"
            src = f'''// Plan launcher in the form src/codegen.cpp:67-93 emits, for the reference's kernels.
#include "kvf_kernels.cuh"
extern "C" cudaError_t kvf_launch_{tag}(const kvf::Args *in, cudaStream_t st) {{
  kvf::Args a = *in;
  a.splits = {s};
  a.warps = 4;
  return kvf::launch<{fmt_enum[fmt]}, {d}, {g}, 2, {ord_enum[order]}, {"true" if bt else "false"}>(a, st);
}}
extern "C" const char *kvf_plan_{tag}() {{ return "{tag} (reference SIMT kernel)"; }}
'''
            hdr = (f"#pragma once\n#define KVF_LAUNCH kvf_launch_{tag}\n#define KVF_PLAN kvf_plan_{tag}\n"
                   f"#define KVF_H {H}\n#define KVF_HKV {Hkv}\n#define KVF_D {d}\n#define KVF_N {n}\n"
                   f"#define KVF_BATCH {B}\n#define KVF_FMT {fmt_enum[fmt]}\n#define KVF_GROUP {group}\n"
                   f"#define KVF_ORDER {ord_enum[order]}\n#define KVF_PAGED {1 if bt else 0}\n"
                   f"#define KVF_BLOCK {bt}\n#define KVF_SPLITS {s}\n#define KVF_WARPS 4\n#define KVF_PRED_US 0.0\n")
            srcp, hdrp = gen_dir / f"refgpu_{tag}.cu", gen_dir / f"plan_info_refgpu_{tag}.h"
            for path, text in ((srcp, src), (hdrp, hdr)):
                if not path.exists() or path.read_text() != text:
                    path.write_text(text)
            out = HARNESS / f"kvf_refgpu_{tag}"
            deps = [srcp, hdrp, rt / "kvf_driver.cu", rt / "kvf_host.h", rt / "kvf_kernels.cuh"]
            if force or _stale(out, deps):
                ov = _overlay({"kvf_kernels.cuh": rt / "kvf_kernels.cuh", "kvf_host.h": rt / "kvf_host.h",
                               "kvf_driver.cu": rt / "kvf_driver.cu", "plan_info.h": hdrp, srcp.name: srcp})
                try:
                    _run([nvcc, "-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler",
                          "-ffp-contract=off", f"-I{ov}", str(ov / "kvf_driver.cu"), str(ov / srcp.name), "-o",
                          str(out)])
                finally:
                    shutil.rmtree(ov, ignore_errors=True)
            built.append(out)
    return built


REF_CLI = HERE / "_ref" / "kvf"


def build_cli(force: bool = False) -> Path | None:
    """The reference's `kvf` compiler CLI, compiled from src/*.cpp with g++
    (its CMake build is not used; the sources need nothing beyond the C++17
    standard library and the reference's own include/)."""
    if REFERENCE is None or not (REFERENCE / "src" / "main.cpp").exists():
        return None
    srcs = sorted((REFERENCE / "src").glob("*.cpp"))
    hdrs = sorted((REFERENCE / "include").rglob("*.h")) + sorted((REFERENCE / "src").glob("*.h"))
    if force or _stale(REF_CLI, srcs + hdrs):
        REF_CLI.parent.mkdir(parents=True, exist_ok=True)
        _run(["g++", "-std=c++17", "-O1", f"-I{REFERENCE / 'include'}", f"-I{REFERENCE / 'src'}",
              *map(str, srcs), "-o", str(REF_CLI)])
    return REF_CLI


def build(force: bool = False) -> None:
    build_oracle(force)
    build_reference(force)
    build_harnesses(force)
    build_refgpu(force)
    build_cli(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(ORACLE_SO)
    print(REF_SO if REF_SO.exists() else "reference tree absent: oracle/_ref not built")
