"""The C-ABI library and the drop-in headers, without a GPU: the library
loads, exports every entry point include/*.h declares, its argument block has
the reference's kvf::Args layout, and the drop-in header compiles the way the
reference's generated sources use it."""
from __future__ import annotations

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import ROOT

import kvforge_b200 as kb
from kvforge_b200._native import SIGNATURES, KvfArgs, lib

INCLUDE = ROOT / "include"


def declared_symbols() -> set[str]:
    names = set()
    for h in INCLUDE.glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"\b(kvf_b200_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    l = lib()
    declared = declared_symbols()
    assert declared, "no entry points found in include/*.h"
    for name in sorted(declared):
        assert hasattr(l, name), f"{name} declared in include/ but not exported"
    bound = {s[0] for s in SIGNATURES}
    assert declared <= bound, declared - bound


def test_version_and_variants():
    l = lib()
    assert b"sm_100a" in l.kvf_b200_version()
    count = l.kvf_b200_variant_count()
    base = 3 * 2 * 2 * 2 * 4 * 2  # the reference's ids (src/codegen.cpp:119-172 over d 64/128, g 1/2/4/8)
    assert count == base + base + 2 * 2 * 4 * 2  # + every id pinned to mma.sync + int8 d128 ids on tcgen05
    names = {l.kvf_b200_variant_name(i).decode() for i in range(count)}
    assert "int8_tm_p_g4_u2_d128" in names and "f16_hm_c_g1_u4_d64" in names
    assert "f16_hm_c_g1_u4_d64_mma" in names and "int8_tm_p_g8_u2_d128_tc" in names
    assert "int8_tm_p_g8_u2_d64_tc" not in names and "f16_hm_c_g1_u2_d128_tc" not in names
    assert l.kvf_b200_variant_name(count) is None
    assert l.kvf_b200_variant_name(-1) is None


def test_unknown_variant_rejected_without_launch():
    a = KvfArgs()
    for bad in [b"f32_hm_c_g1_u2_d128", b"int8_xx_c_g1_u2_d128", b"int8_hm_c_g3_u2_d128",
                b"int8_hm_c_g1_u2_d96", b"int8_hm_c_g1_u2_d128x", b"", b"f16_hm_c_g1_u2_d128_tc",
                b"int8_hm_c_g1_u2_d64_tc", b"int8_hm_c_g1_u2_d128_mmaa", b"int8_hm_c_g1_u2_d128_"]:
        assert lib().kvf_b200_launch_variant(bad, ctypes.byref(a), None) == 98  # InvalidDeviceFunction


def test_args_layout_matches_reference_struct(tmp_path):
    """kvf_args (include/kvforge_b200.h) has kvf::Args' field offsets
    (runtime/kvf_kernels.cuh:29-46) and the ctypes mirror agrees."""
    gcc = shutil.which("gcc") or "/usr/bin/gcc"
    src = tmp_path / "layout.c"
    fields = [f[0] for f in KvfArgs._fields_]
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(kvf_args, {f}));' for f in fields)
    src.write_text(
        "#include <stdio.h>\n#include <stddef.h>\n#include \"kvforge_b200.h\"\n"
        f"int main(void) {{\n  printf(\"size %zu\\n\", sizeof(kvf_args));\n{body}\n  return 0;\n}}\n"
    )
    exe = tmp_path / "layout"
    subprocess.run([gcc, f"-I{INCLUDE}", "-I/usr/local/cuda/include", str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(KvfArgs) == 136
    for f in fields:
        assert int(out[f]) == getattr(KvfArgs, f).offset, f
    # The reference's prefix: 9 pointers, 9 ints, 1 float.
    assert KvfArgs.scale_log2.offset == 9 * 8 + 9 * 4


def test_dropin_header_compiles_generated_launcher(tmp_path):
    """A launcher exactly as src/codegen.cpp:67-93 emits it, and a dispatch
    registration as in gen/kvf_dispatch_*.cu, compile against
    include/kvf_kernels.cuh + include/kvf_registry.h and link to the library."""
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    src = tmp_path / "decode_x.cu"
    src.write_text(
        '#include "kvf_kernels.cuh"\n#include "kvf_registry.h"\n\n'
        'extern "C" cudaError_t kvf_launch_x(const kvf::Args *in, cudaStream_t st) {\n'
        "  kvf::Args a = *in;\n  a.splits = 16;\n  a.warps = 4;\n  a.group_shift = 5;\n"
        "  return kvf::launch<kvf::FMT_INT4, 128, 4, 2, kvf::ORD_HEAD, false>(a, st);\n}\n"
        'extern "C" const char *kvf_plan_x() { return "int4:32 | head_major/contiguous"; }\n'
        "void kvf_register_int8_tm_p(kvf::Registry &r) {\n"
        '  r.add("int8_tm_p_g4_u2_d128", &kvf::launch<kvf::FMT_INT8, 128, 4, 2, kvf::ORD_TOKEN, true>);\n'
        "}\n"
        "int main() {\n  kvf::Registry r;\n  kvf_register_int8_tm_p(r);\n"
        '  return r.find("int8_tm_p_g4_u2_d128") ? 0 : 1;\n}\n'
    )
    exe = tmp_path / "decode_x"
    subprocess.run([nvcc, "-std=c++17", f"-I{INCLUDE}", str(src), "-o", str(exe),
                    f"-L{kb.LIB_PATH.parent}", "-lkvforge_b200", f"-Xlinker=-rpath={kb.LIB_PATH.parent}"],
                   check=True, capture_output=True)
    assert subprocess.run([str(exe)]).returncode == 0


def test_invalid_arguments_are_rejected_before_any_launch():
    l = lib()
    a = KvfArgs()
    a.B, a.H, a.Hkv, a.n, a.splits = 1, 30, 8, 128, 1   # H not a multiple of Hkv
    assert l.kvf_b200_decode(ctypes.byref(a), 0, 128, 1, 0, 0, None) == 1
    a.H = 32
    assert l.kvf_b200_decode(ctypes.byref(a), 0, 96, 1, 0, 0, None) == 1      # d
    assert l.kvf_b200_decode(ctypes.byref(a), 3, 128, 1, 0, 0, None) == 1     # format
    assert l.kvf_b200_decode(ctypes.byref(a), 0, 128, 2, 0, 0, None) == 1     # g neither 1 nor H/Hkv
    a.group_shift = 5                                                          # int8:32 not offered
    assert l.kvf_b200_decode(ctypes.byref(a), 1, 128, 1, 0, 0, None) == 1
    a.H = 128                                                                  # g = 16 > 8
    assert l.kvf_b200_decode(ctypes.byref(a), 0, 128, 1, 0, 0, None) == 1
    a.H = 32
    buf = np.zeros(64, dtype=np.uint8)
    a.q = a.out = buf.ctypes.data
    a.k = buf.ctypes.data + 1                                                  # misaligned payload
    a.v = buf.ctypes.data
    assert l.kvf_b200_decode(ctypes.byref(a), 0, 128, 1, 0, 0, None) == 716
    assert l.kvf_b200_decode(None, 0, 128, 1, 0, 0, None) == 1
    a.B = 0                                                                    # empty batch: no-op
    assert l.kvf_b200_decode(ctypes.byref(a), 0, 128, 1, 0, 0, None) == 0


def test_suggest_splits_without_gpu():
    l = lib()
    # Llama-3-8B shape, one sequence: its 8 KV heads x splits blocks fill every SM.
    s = l.kvf_b200_suggest_splits(1, 32, 8, 32768, 1, 128, 64, 0, 0)
    assert 148 <= 8 * s <= 2048
    # Batch 64 x 8 KV heads already fills the machine several times over.
    s5 = l.kvf_b200_suggest_splits(64, 64, 8, 16384, 1, 128, 64, 1, 16)
    assert 1 <= s5 <= 32
    assert l.kvf_b200_suggest_splits(1, 8, 8, 100, 0, 64, 0, 0, 0) >= 1
    assert l.kvf_b200_suggest_splits(0, 8, 8, 100, 0, 64, 0, 0, 0) == 1


def test_append_argument_checks_need_no_gpu():
    """kvf_b200_append rejects what it cannot place before touching the
    device: a missing cache or new rows, an unknown format, order or head
    dimension, a quantized cache without metadata, a paged cache without a
    block table; nothing to append (t_new = 0 or B = 0) is a no-op."""
    l = lib()
    a = KvfArgs()
    a.B, a.H, a.Hkv, a.n = 2, 8, 8, 64
    fake = 0x1000  # never dereferenced: every case fails or returns before a launch
    assert l.kvf_b200_append(None, 0, 128, 0, 0, fake, fake, 1, fake, None) == 1
    assert l.kvf_b200_append(ctypes.byref(a), 0, 128, 0, 0, fake, fake, 0, fake, None) == 0  # t_new = 0
    assert l.kvf_b200_append(ctypes.byref(a), 0, 96, 0, 0, fake, fake, 1, fake, None) == 1   # head dim
    assert l.kvf_b200_append(ctypes.byref(a), 3, 128, 0, 0, fake, fake, 1, fake, None) == 1  # format
    assert l.kvf_b200_append(ctypes.byref(a), 0, 128, 2, 0, fake, fake, 1, fake, None) == 1  # order
    assert l.kvf_b200_append(ctypes.byref(a), 0, 128, 0, 0, fake, fake, -1, fake, None) == 1  # t_new < 0
    assert l.kvf_b200_append(ctypes.byref(a), 0, 128, 0, 0, None, fake, 1, fake, None) == 1  # no K rows
    assert l.kvf_b200_append(ctypes.byref(a), 0, 128, 0, 0, fake, fake, 1, None, None) == 1  # no positions
    a.k = a.v = fake
    assert l.kvf_b200_append(ctypes.byref(a), 1, 128, 0, 0, fake, fake, 1, fake, None) == 1  # int8, no metadata
    assert l.kvf_b200_append(ctypes.byref(a), 0, 128, 0, 1, fake, fake, 1, fake, None) == 1  # paged, no table
    a.B = 0
    assert l.kvf_b200_append(ctypes.byref(a), 0, 128, 0, 0, fake, fake, 1, fake, None) == 0  # empty batch


def test_kernel_path_errors_need_no_gpu():
    """An explicit path is checked before anything launches: tcgen05 for a
    format it does not take is cudaErrorNotSupported, an unknown path
    cudaErrorInvalidValue (empty batch, so nothing would run either way)."""
    a = KvfArgs()
    a.B, a.H, a.Hkv, a.n, a.splits = 0, 32, 8, 16, 1
    l = lib()
    for path, want in [(0, 0), (1, 0), (2, 801), (3, 1), (-1, 1)]:
        assert l.kvf_b200_decode_path(ctypes.byref(a), 0, 128, 1, 0, 0, path, None) == want, path
    buf = ctypes.create_string_buffer(64)
    assert l.kvf_b200_describe_path(ctypes.byref(a), 0, 128, 0, 0, 2, buf, 64) == 801
