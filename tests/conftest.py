"""Shared test setup.

Markers: `gpu` tests need a CUDA device (run with -m gpu on a B200); all
other tests run on the CPU. The oracle's C restatement is (re)built with gcc
on first use; the kernel library must have been built by
`python -m kvforge_b200.build` (or __graft_entry__.build()).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"

# Tolerances of the path: output within max-abs 2e-3 and
# max-rel 1e-2 of the reference's fp64 attention; relative error is taken over
# elements with |ref| > 1e-3. The reference's own verification is rel-L2 < 2e-3
# (runtime/kvf_driver.cu:52, bench/sweep.cu:196).
MAX_ABS = 2e-3
MAX_REL = 1e-2
REL_FLOOR = 1e-3
REL_L2 = 2e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def assert_close(got: np.ndarray, ref: np.ndarray, what: str = "") -> dict:
    got = np.asarray(got, dtype=np.float64).reshape(-1)
    ref = np.asarray(ref, dtype=np.float64).reshape(-1)
    assert got.shape == ref.shape, what
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    err = np.abs(got - ref)
    max_abs = float(err.max(initial=0.0))
    big = np.abs(ref) > REL_FLOOR
    max_rel = float((err[big] / np.abs(ref[big])).max(initial=0.0))
    den = float(np.sqrt((ref * ref).sum()))
    rl2 = float(np.sqrt((err * err).sum()) / den) if den > 0 else 0.0
    stats = {"max_abs": max_abs, "max_rel": max_rel, "rel_l2": rl2}
    assert max_abs <= MAX_ABS, f"{what}: max abs {max_abs:.3g} > {MAX_ABS} {stats}"
    assert max_rel <= MAX_REL, f"{what}: max rel {max_rel:.3g} > {MAX_REL} {stats}"
    assert rl2 < REL_L2, f"{what}: rel L2 {rl2:.3g} >= {REL_L2} {stats}"
    return stats


@pytest.fixture(scope="session")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
