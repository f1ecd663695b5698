"""The reference's own harnesses, run on this library.

oracle/build.py compiles, unmodified and against include/ (the drop-in
kvf_kernels.cuh, the reference's kvf_registry.h) and libkvforge_b200.so:

* runtime/kvf_driver.cu with each plan the reference's compiler emitted
  (results/plans/<shape>/decode_<shape>.cu + plan_info.h, the launchers of
  src/codegen.cpp:67-117) and with one plan kvforge_b200.codegen emits. The
  driver builds its own data, quantizes and places it with the reference's
  host code (runtime/kvf_host.h), calls KVF_LAUNCH once, and exits 0 only if
  the output is within relative L2 2e-3 of the reference's fp64 attention
  over the dequantised cache (runtime/kvf_driver.cu:43-52, 62);
* bench/sweep.cu over the sm_100a dispatch tables kvforge_b200.codegen emits
  (kvf_register_all), timing a selection of the reference's own candidate
  plans for one shape (every format x order x residency) and verifying each
  the same way (bench/sweep.cu:180-197); it exits 3 if any plan fails.

The binaries are test infrastructure under oracle/_ref/harness/ (never
committed; built where the reference tree exists). Tests skip where they
are absent.
"""
from __future__ import annotations

import csv
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HARNESS = ROOT / "oracle" / "_ref" / "harness"
DRIVERS = sorted(HARNESS.glob("kvf_driver_*")) if HARNESS.exists() else []
SWEEP = HARNESS / "kvf_sweep"
PLANS = sorted(HARNESS.glob("plans_*.csv")) if HARNESS.exists() else []


def _run(cmd, timeout=600):
    return subprocess.run([str(c) for c in cmd], capture_output=True, text=True, timeout=timeout)


def test_sweep_binary_loads_the_library():
    """No GPU needed: the sweep parses its arguments before any CUDA call, so
    a run without --plans proves the binary and libkvforge_b200.so resolve."""
    if not SWEEP.exists():
        pytest.skip("reference harnesses not built (no reference tree at build time)")
    r = _run([SWEEP])
    assert r.returncode == 2 and "usage: sweep" in r.stderr, r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("driver", DRIVERS or [None], ids=[d.name for d in DRIVERS] or ["none"])
def test_reference_driver_passes(cuda, driver):
    if driver is None:
        pytest.skip("reference harnesses not built (no reference tree at build time)")
    r = _run([driver, "--reps", "5"])
    assert r.returncode == 0, f"{driver.name} exit {r.returncode}\n{r.stdout}\n{r.stderr}"
    m = re.search(r"relative error vs dequantised reference (\S+) \((PASS|FAIL)\)", r.stdout)
    assert m and m.group(2) == "PASS" and float(m.group(1)) < 2e-3, r.stdout
    assert re.search(r"rate:\s+\S+ GB/s", r.stdout), r.stdout


@pytest.mark.gpu
def test_reference_sweep_verifies_every_plan(cuda, tmp_path):
    if not SWEEP.exists() or not PLANS:
        pytest.skip("reference harnesses not built (no reference tree at build time)")
    from kvforge_b200._native import lib

    plans = PLANS[0]
    with open(plans, newline="") as f:
        want = list(csv.DictReader(f))
    out = tmp_path / "sweep.csv"
    r = _run([SWEEP, "--plans", plans, "--out", out, "--reps", "3", "--warmup", "1"], timeout=1200)
    assert r.returncode == 0, f"sweep exit {r.returncode}\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    m = re.search(r"registry: (\d+) variants", r.stdout)
    assert m and int(m.group(1)) == lib().kvf_b200_variant_count(), r.stdout
    assert re.search(r"done: (\d+) timed, 0 skipped, 0 failed verification", r.stdout), r.stdout
    with open(out, newline="") as f:
        got = list(csv.DictReader(f))
    assert len(got) == len(want)
    kinds = {(g["fmt"], g["order"], g["residency"]) for g in got}
    assert len(kinds) == 12  # f16/int8/int4 x head/token-major x contiguous/paged
    for g in got:
        assert g["verified"] == "1" and float(g["err_ref"]) < 2e-3, g
        assert float(g["t_us"]) > 0
