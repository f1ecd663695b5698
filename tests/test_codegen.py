"""sm_100a source emission, the cost model and its calibration, without a
GPU: the emitted dispatch tables list exactly the ids the library registers,
compile against the drop-in headers and register every id; a plan's launcher
and header compile; the model's fit recovers known constants and its .cal
file round-trips."""
from __future__ import annotations

import math
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import ROOT

from kvforge_b200 import codegen, costmodel
from kvforge_b200._native import lib

INCLUDE = ROOT / "include"
LIBDIR = ROOT / "kvforge_b200" / "_lib"
CUDA_INC = Path("/usr/local/cuda/include")


def _gxx():
    gxx = shutil.which("g++")
    if not gxx or not (CUDA_INC / "cuda_runtime.h").exists():
        pytest.skip("g++ or the CUDA headers are not available")
    return gxx


def test_emitted_ids_are_the_library_registry():
    l = lib()
    c_ids = [l.kvf_b200_variant_name(i).decode() for i in range(l.kvf_b200_variant_count())]
    assert codegen.all_variant_ids() == c_ids


def test_variant_ids_follow_the_reference_format():
    assert codegen.variant_id(1, 1, True, 4, 2, 128) == "int8_tm_p_g4_u2_d128"
    assert codegen.variant_id(1, 0, False, 8, 4, 128, "tc") == "int8_hm_c_g8_u4_d128_tc"
    assert codegen.variant_id(0, 0, False, 1, 2, 64, "mma") == "f16_hm_c_g1_u2_d64_mma"
    with pytest.raises(ValueError):
        codegen.variant_id(0, 0, False, 1, 2, 128, "tc")
    assert codegen.instantiation(1, 128, 4, 2, 1, True) == \
        "kvf::launch<kvf::FMT_INT8, 128, 4, 2, kvf::ORD_TOKEN, true>"
    assert codegen.instantiation(1, 128, 4, 2, 1, True, "tc").endswith(", KVF_PATH_TC>")


def test_emitted_dispatch_compiles_and_registers_every_id(tmp_path):
    gxx = _gxx()
    files = codegen.write_files(codegen.emit_dispatch_sources(), tmp_path)
    assert len(files) == 13  # 12 buckets + kvf_dispatch.cu, as the reference emits
    main = tmp_path / "main.cpp"
    main.write_text(
        '#include "kvf_registry.h"\n#include <cstdio>\n'
        "int main() {\n  kvf::Registry r;\n  kvf_register_all(r);\n  int missing = 0;\n"
        "  for (int i = 0; i < kvf_b200_variant_count(); ++i) if (!r.find(kvf_b200_variant_name(i))) ++missing;\n"
        '  std::printf("%zu %d %d\\n", r.fn.size(), kvf_b200_variant_count(), missing);\n'
        "  return (int)r.fn.size() == kvf_b200_variant_count() && missing == 0 ? 0 : 1;\n}\n")
    exe = tmp_path / "regtest"
    cmd = [gxx, "-std=c++17", "-O0", f"-I{INCLUDE}", f"-I{CUDA_INC}", "-x", "c++",
           *[str(f) for f in files], "-x", "none", str(main), "-o", str(exe), f"-L{LIBDIR}", "-lkvforge_b200",
           "-L/usr/local/cuda/lib64", "-lcudart", f"-Wl,-rpath,{LIBDIR}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    n_reg, n_lib, missing = map(int, r.stdout.split())
    assert n_reg == n_lib == len(codegen.all_variant_ids()) and missing == 0


def test_plan_launcher_and_header_compile(tmp_path):
    gxx = _gxx()
    p = codegen.plan("llama3_8b_gqa", B=1, H=32, Hkv=8, d=128, n=32768, fmt=1, group=64, order=1)
    assert p.splits >= 1 and p.path in ("mma", "tc") and math.isfinite(p.predicted_us)
    big = codegen.plan("llama3_70b", B=64, H=64, Hkv=8, d=128, n=16384, fmt=1, group=64, order=1,
                       paged=True, block_tokens=16)
    assert big.path in ("mma", "tc") and big.block_tokens == 16
    f16 = codegen.plan("mha", B=1, H=32, Hkv=32, d=128, n=4096, fmt=0, group=0, order=0)
    assert f16.path == "mma"  # the tcgen05 kernel takes int8 only
    for q in (p, big, f16):
        src = tmp_path / f"{q.name}.cu"
        src.write_text(codegen.emit_kernel_source(q))
        hdr = codegen.emit_plan_header(q)
        assert f"#define KVF_SPLITS {q.splits}" in hdr and "#define KVF_PATH KVF_PATH_" in hdr
        (tmp_path / f"{q.name}.h").write_text(hdr)
        obj = tmp_path / f"{q.name}.o"
        r = subprocess.run([gxx, "-std=c++17", "-c", "-x", "c++", str(src), f"-I{INCLUDE}", f"-I{CUDA_INC}",
                            "-o", str(obj)], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-2000:]
        syms = subprocess.run(["nm", "-g", str(obj)], capture_output=True, text=True).stdout
        assert f"kvf_launch_{q.name}" in syms and f"kvf_plan_{q.name}" in syms


def _rows_from(coef, shapes, paths=("mma", "tc")):
    rows = []
    for s in shapes:
        for path in paths:
            if path == "tc" and not (s.fmt == 1 and s.d == 128):
                continue
            for sp in costmodel.split_candidates(s.B, s.Hkv, s.n, path):
                f = costmodel.features(s, sp, path)
                us = float(np.dot(f, [coef[path][k] for k in costmodel.KEYS]))
                rows.append(dict(B=s.B, H=s.H, Hkv=s.Hkv, d=s.d, n=s.n, fmt=s.fmt, group=s.group,
                                 paged=int(s.paged), block_tokens=s.block_tokens, tokens="", splits=sp,
                                 path=path, us=us))
    return rows


def test_fit_recovers_known_constants():
    truth = {"mma": dict(c_fixed=7.0, c_byte=0.15, c_stage=1.1, c_split=2.5, c_part=0.8),
             "tc": dict(c_fixed=9.0, c_byte=0.14, c_stage=2.0, c_split=0.7, c_part=0.3)}
    shapes = [costmodel.Shape(1, 32, 8, 128, 32768, 1, 64), costmodel.Shape(16, 32, 8, 128, 8192, 1, 64),
              costmodel.Shape(64, 64, 8, 128, 16384, 1, 64, True, 16), costmodel.Shape(1, 32, 32, 128, 4096, 0, 0),
              costmodel.Shape(4, 32, 8, 128, 16384, 2, 32), costmodel.Shape(64, 32, 8, 128, 4096, 1, 64)]
    rows = _rows_from(truth, shapes)
    m = costmodel.fit(rows)
    for path in truth:
        for k, v in truth[path].items():
            assert m.coef[path][k] == pytest.approx(v, rel=1e-3, abs=1e-4), (path, k)
    assert np.abs(costmodel.relative_errors(m, rows)).max() < 1e-6


def test_calibration_file_round_trips(tmp_path):
    m = costmodel.CostModel({p: {k: i + 0.25 * j for j, k in enumerate(costmodel.KEYS)}
                             for i, p in enumerate(("mma", "tc"))}, "test")
    cal = tmp_path / "x.cal"
    m.save(cal, ["made by a test"])
    text = cal.read_text()
    assert text.startswith("#") and "mma.c_stage = " in text
    back = costmodel.CostModel.load(cal)
    assert back.coef == m.coef
    s = costmodel.Shape(2, 32, 8, 128, 1000, 1, 64)
    assert back.predict_us(s, 3, "tc") == pytest.approx(m.predict_us(s, 3, "tc"))


def test_payload_matches_bench_definition():
    # int8 group 64, d 128: 2 x (128 + 4 * 2) bytes per (token, KV head)
    s = costmodel.Shape(1, 32, 8, 128, 32768, 1, 64)
    assert s.payload_bytes() == 2 * 32768 * 8 * (128 + 8)
    ragged = costmodel.Shape(8, 32, 8, 128, 8192, 0, 0, True, 16, tokens=40000)
    assert ragged.payload_bytes() == 2 * 40000 * 8 * 256
