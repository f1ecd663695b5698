"""bench.py's reference arm runs on the CPU (the reference's own
kvf::reference_attention from oracle/_ref, or the restatement when the
reference tree is absent) and prints the contract's JSON line."""
from __future__ import annotations

import json
import os
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_prints_the_contract_line():
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1", "--workload", "mha_b1_h32_n4096_f16_hm"],
                         capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["unit"] == "TB/s" and line["higher_is_better"] is True and line["value"] > 0
    assert line["metric"].startswith("decode-attn effective KV TB/s")
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("reference", "port") and cb["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "TB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["workload"] == "mha_b1_h32_n4096_f16_hm"
