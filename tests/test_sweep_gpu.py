"""The B200 sweep and calibration (kvforge_b200.sweep, the counterpart of the
reference's bench/sweep.cu and `kvf calibrate`, src/calib.cpp and
src/fit.cpp) on a real GPU: a small grid of shapes is timed over split counts
and both kernel paths, the CSV is written and read back, and the cost model's
constants are fitted to it."""
from __future__ import annotations

import math

import pytest

pytestmark = pytest.mark.gpu

TINY_GRID = [
    # (name, base workload, batch, tokens per sequence)
    ("t_int8_tm_b4_n4096", "llama3_8b_gqa_b1_n32768_int8g64_tm", 4, 4096),
    ("t_int4_hm_b2_n8192", "long_gqa_b1_n65536_int4g32_hm", 2, 8192),
    ("t_l70b_p16_b8_n2048", "llama3_70b_b64_n16384_int8g64_tm_p16", 8, 2048),
]


def test_sweep_times_the_grid_and_calibrates(cuda, tmp_path, monkeypatch):
    from kvforge_b200 import api, costmodel, sweep

    monkeypatch.setattr(sweep, "GRID", TINY_GRID)
    out = tmp_path / "sweep.csv"
    rows = sweep.run(out, reps=3, warmup=1, max_splits=3)
    assert api.device_errors() == 0

    # Every shape is swept on the mma.sync path, the int8 ones on tcgen05
    # too, each at the launcher's own split count among the candidates.
    names = {r["name"] for r in rows}
    assert names == {g[0] for g in TINY_GRID}
    for name in names:
        mine = [r for r in rows if r["name"] == name]
        paths = {r["path"] for r in mine}
        assert "mma" in paths
        if mine[0]["fmt"] == 1:
            assert "tc" in paths
        assert any(r["suggested"] for r in mine), name
    for r in rows:
        assert 0 < r["us_min"] <= r["us"] < 1e5, r
        assert math.isfinite(r["predicted_us"]) and r["predicted_us"] > 0, r

    back = sweep.read_csv(out)
    assert len(back) == len(rows)
    assert [int(r["splits"]) for r in back] == [r["splits"] for r in rows]

    cal = tmp_path / "fit.cal"
    model = sweep.calibrate(out, cal)
    assert cal.exists()
    loaded = costmodel.CostModel.load(cal)
    for r in back:
        shape = costmodel._shape(r)
        p = loaded.predict_us(shape, int(r["splits"]), r["path"], costmodel._balanced(r))
        assert math.isfinite(p) and p >= 0
        # the .cal file keeps six significant digits
        assert p == pytest.approx(model.predict_us(shape, int(r["splits"]), r["path"], costmodel._balanced(r)),
                                  rel=1e-4, abs=1e-3)
