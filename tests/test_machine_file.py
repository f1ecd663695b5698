"""The B200 machine description (kvforge_b200/machines/b200-sxm.gpu and its
resource table) through the reference's own compiler front end.

`kvf machine` runs loadMachine (src/machine.cpp:70-130), including the
resource-table read at :105-128; `kvf plan --machine` plans a decode spec for
the machine and emits plan_info.h (src/main.cpp:112-114, src/emit.cpp). The
CLI is the reference's src/*.cpp compiled by oracle/build.py (build_cli); the
tests skip where the reference tree is absent.
"""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest

from oracle import build as oracle_build

REPO = Path(__file__).resolve().parents[1]

MACHINE = REPO / "kvforge_b200" / "machines" / "b200-sxm.gpu"
RESOURCES = REPO / "kvforge_b200" / "machines" / "resources_sm100.csv"


@pytest.fixture(scope="module")
def kvf() -> Path:
    cli = oracle_build.build_cli()
    if cli is None or not cli.exists():
        pytest.skip("reference tree absent: the reference CLI is not built")
    return cli


def _machine_values() -> dict:
    vals = {}
    for line in MACHINE.read_text().splitlines():
        line = line.split("#", 1)[0]
        if "=" in line:
            k, v = (x.strip().strip('"') for x in line.split("=", 1))
            vals[k] = v
    return vals


def test_machine_file_parses(kvf):
    r = subprocess.run([str(kvf), "machine", str(MACHINE)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    dumped = dict(re.findall(r"^(\w+) = (.+)$", r.stdout, re.M))
    want = _machine_values()
    assert dumped["name"] == want["name"] == "b200-sxm"
    assert int(dumped["sms"]) == int(want["sms"]) == 148
    assert int(dumped["compute_capability"]) == 10
    assert float(dumped["bw_peak_gbs"]) == pytest.approx(float(want["bw_peak_gbs"]))
    assert float(dumped["lat_ns"]) == pytest.approx(float(want["lat_ns"]))
    assert dumped["resources"] == want["resources"] == RESOURCES.name


def test_resource_table_rows_are_readable():
    # loadMachine keys rows by their first seven fields and reads the eighth
    # (registers); rows with fewer than eight fields are skipped silently, so
    # every data row here must have them all.
    rows = RESOURCES.read_text().splitlines()
    assert rows[0].split(",")[:8] == ["fmt", "d", "g", "u", "ord", "paged", "final", "regs"]
    assert len(rows) > 1
    for row in rows[1:]:
        f = row.split(",")
        assert len(f) >= 8, row
        assert all(x.strip().lstrip("-").isdigit() for x in f), row


SPEC = """\
target machine = "{machine}"
target max_rel_err = 0.02

decode llama3_70b(H: 64, H_kv: 8, d: 128, n: 16384, batch: 64) {{
  Q: query<H, d, f32>
  K: kvcache<n, d, ?, ?, ?>
  V: kvcache<n, d, ?, ?, ?>
  O = decode_attn(Q, K, V, scale = auto, splits = ?, gqa_pack = ?)
}}
"""


@pytest.mark.parametrize("how", ["target", "flag"])
def test_plan_on_b200_machine(kvf, tmp_path, how):
    spec = tmp_path / "spec.kv"
    # "flag": the spec names a stand-in machine and --machine overrides it.
    stand_in = tmp_path / "stand_in.gpu"
    stand_in.write_text('name = "stand-in"\nsms = 2\n')
    spec.write_text(SPEC.format(machine=MACHINE if how == "target" else stand_in))
    out = tmp_path / "out"
    cmd = [str(kvf), "plan", str(spec), "--out", str(out), "--quant"]
    if how == "flag":
        cmd += ["--machine", str(MACHINE)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=tmp_path)
    assert r.returncode == 0, r.stderr + r.stdout
    assert re.search(r"^Machine: b200-sxm", r.stdout, re.M), r.stdout
    assert re.search(r"SMs = 148\b", r.stdout), r.stdout
    info = (out / "plan_info.h").read_text()
    assert "#define KVF_PLAN" in info
    assert re.search(r"#define KVF_H 64\b", info) and re.search(r"#define KVF_BATCH 64\b", info)
    # The chosen plan is one the drop-in covers: a format, layout and split
    # count the B200 kernels take.
    fmt = re.search(r"format:\s+(\S+)", r.stdout).group(1)
    assert fmt in ("f16", "int8:32", "int8:64", "int8:128", "int4:32", "int4:64", "int4:128"), fmt
    splits = int(re.search(r"splits=(\d+)", r.stdout).group(1))
    assert splits >= 1
