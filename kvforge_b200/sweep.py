"""Sweep harness and calibration on B200.

Counterpart of the reference's bench/sweep.cu and ``kvf calibrate``
(src/calib.cpp, src/fit.cpp): times decode steps over a grid of shapes, split
counts and kernel paths on the GPU, writes one CSV row per point (measured
and predicted time), and fits the cost model's constants
(kvforge_b200.costmodel) to the rows.

    python -m kvforge_b200.sweep run --out sweep.csv            # on a B200
    python -m kvforge_b200.sweep calibrate sweep.csv \\
        --cal kvforge_b200/machines/b200-sxm.cal                 # anywhere

Timing is bench.py's: the L2 is flushed (kvforge_b200.l2flush) before every step,
each step is bracketed by CUDA events on the launching stream, and the median
of the repetitions is kept. Inputs are the benchmark workloads' seeded
synthetic data with the swept batch and length.
"""
from __future__ import annotations

import argparse
import csv
import ctypes
import dataclasses
import math
import sys
from pathlib import Path
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import costmodel
from .codegen import variant_id
from .l2flush import L2Flush

FIELDS = ["name", "B", "H", "Hkv", "d", "n", "fmt", "group", "order", "paged", "block_tokens", "tokens",
          "splits", "path", "variant", "payload_bytes", "us", "us_min", "predicted_us", "suggested", "balanced"]

# (name, base workload, batch, tokens per sequence); None keeps the base's.
GRID = [
    ("mha_f16_hm_b1_n4096", "mha_b1_h32_n4096_f16_hm", None, None),
    ("gqa_int8_tm_b1_n32768", "llama3_8b_gqa_b1_n32768_int8g64_tm", None, None),
    ("gqa_int8_tm_b4_n16384", "llama3_8b_gqa_b1_n32768_int8g64_tm", 4, 16384),
    ("gqa_int8_tm_b16_n8192", "llama3_8b_gqa_b1_n32768_int8g64_tm", 16, 8192),
    ("gqa_int8_tm_b64_n4096", "llama3_8b_gqa_b1_n32768_int8g64_tm", 64, 4096),
    ("paged_f16_tm_b8_ragged", "paged_gqa_b8_n2k_8k_f16_tm_p16", None, None),
    ("gqa_int4_hm_b1_n65536", "long_gqa_b1_n65536_int4g32_hm", None, None),
    ("gqa_int4_hm_b4_n16384", "long_gqa_b1_n65536_int4g32_hm", 4, 16384),
    ("l70b_int8_tm_p16_b16_n16384", "llama3_70b_b64_n16384_int8g64_tm_p16", 16, None),
    ("l70b_int8_tm_p16_b64_n16384", "llama3_70b_b64_n16384_int8g64_tm_p16", None, None),
]
QUICK = {"gqa_int8_tm_b1_n32768", "gqa_int8_tm_b16_n8192", "gqa_int4_hm_b1_n65536", "l70b_int8_tm_p16_b16_n16384"}


def _time_steps(step, flush, stream, warmup: int, reps: int) -> List[float]:
    import torch

    for i in range(warmup):
        flush(i)
        step()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for i, (e0, e1) in enumerate(ev):
        flush(i + 7)
        e0.record(stream)
        step()
        e1.record(stream)
    torch.cuda.synchronize()
    return [e0.elapsed_time(e1) * 1000.0 for e0, e1 in ev]


def run(out: Path, quick: bool = False, reps: int = 15, warmup: int = 3, max_splits: int = 6) -> List[dict]:
    """Times the grid on cuda:0 and writes the CSV; returns the rows."""
    import torch

    from . import api, workloads
    from ._native import check, lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = lib()
    stream = torch.cuda.current_stream(dev)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    flush = L2Flush(dev)
    default_model = costmodel.CostModel.load()
    rows: List[dict] = []
    for name, base, B, n in GRID:
        if quick and name not in QUICK:
            continue
        w = workloads.CONFIGS[base]
        repl = {}
        if B is not None:
            repl["B"] = B
        if n is not None:
            repl["n"] = n
        w = dataclasses.replace(w, **repl)
        q, K, V, seq_lens = workloads.generate(w, dev, seed=w.seed)
        cache = api.KVCache.from_logical(K, V, fmt=w.fmt, group=w.group, place=w.place, seq_lens=seq_lens)
        del K, V
        torch.cuda.empty_cache()
        tokens = int(seq_lens.sum()) if seq_lens is not None else None
        shape = costmodel.Shape(w.B, w.H, w.Hkv, w.d, w.n, w.fmt, w.group if w.fmt else 0, w.place.paged,
                                w.place.block_tokens if w.place.paged else 0, tokens)
        suggested = api.suggest_splits(cache, w.H)
        paths = ["mma"] + (["tc"] if w.fmt == 1 and w.d == 128 else [])
        out_t = torch.empty_like(q)
        g = w.H // w.Hkv
        for path in paths:
            cands = costmodel.split_candidates(w.B, w.Hkv, w.n, path)
            if len(cands) > max_splits:  # keep both ends and the wave-filling middle
                idx = np.unique(np.round(np.linspace(0, len(cands) - 1, max_splits)).astype(int))
                cands = [cands[i] for i in idx]
            for s in sorted(set(cands) | {suggested}):
                ws = api.Workspace.allocate(w.B, w.H, w.d, s, dev)
                a = api.make_args(q, cache, out_t, ws)
                code = api.PATHS[path]

                def step():
                    check("kvf_b200_decode_path",
                          L.kvf_b200_decode_path(ctypes.byref(a), w.fmt, w.d, g, w.place.order, int(w.place.paged),
                                                 code, sptr))

                balanced = "chunk=balanced" in api.describe(q, cache, ws, path=path)
                ts = _time_steps(step, flush, stream, warmup, reps if shape.payload_bytes() < 1e9 else max(5, reps // 3))
                errs = api.device_errors()
                if errs:
                    raise RuntimeError(f"{name} splits={s} path={path}: device error bits {errs:#x}")

                rows.append({
                    "name": name, "B": w.B, "H": w.H, "Hkv": w.Hkv, "d": w.d, "n": w.n, "fmt": w.fmt,
                    "group": shape.group, "order": w.place.order, "paged": int(w.place.paged),
                    "block_tokens": shape.block_tokens, "tokens": tokens if tokens is not None else "",
                    "splits": s, "path": path,
                    "variant": variant_id(w.fmt, w.place.order, w.place.paged, g, 2, w.d, path),
                    "payload_bytes": shape.payload_bytes(), "us": round(float(np.median(ts)), 3),
                    "us_min": round(float(np.min(ts)), 3),
                    "predicted_us": round(default_model.predict_us(shape, s, path, balanced), 3),
                    "suggested": int(s == suggested), "balanced": int(balanced),
                })
                print(f"{name:30s} {path:3s} splits={s:4d} {rows[-1]['us']:9.2f} us", flush=True)
                del ws
        del cache, q, out_t
        torch.cuda.empty_cache()
    write_csv(rows, out)
    return rows


def write_csv(rows: Sequence[dict], out: Path) -> None:
    out.parent.mkdir(parents=True, exist_ok=True)
    with open(out, "w", newline="") as f:
        wr = csv.DictWriter(f, fieldnames=FIELDS)
        wr.writeheader()
        for r in rows:
            wr.writerow({k: r.get(k, "") for k in FIELDS})


def read_csv(path: Path) -> List[dict]:
    with open(path, newline="") as f:
        return list(csv.DictReader(f))


def planner_report(model: costmodel.CostModel, rows: Sequence[dict]) -> List[dict]:
    """Per swept shape: the measured time of the plan the model picks among
    the swept (splits, path) points, of the launcher's own default
    (suggested splits, AUTO path), and of the best point."""
    by: Dict[str, List[dict]] = {}
    for r in rows:
        by.setdefault(r["name"], []).append(r)
    rep = []
    for name, rs in by.items():
        best = min(rs, key=lambda r: float(r["us"]))
        pick = min(rs, key=lambda r: model.predict_us(costmodel._shape(r), int(r["splits"]), r["path"],
                                                        costmodel._balanced(r)))
        sugg = [r for r in rs if int(r["suggested"])]
        rep.append({"name": name, "best_us": float(best["us"]), "best": f"{best['path']}/{best['splits']}",
                    "model_us": float(pick["us"]), "model": f"{pick['path']}/{pick['splits']}",
                    "suggested_us": min(float(r["us"]) for r in sugg) if sugg else float("nan")})
    return rep


def calibrate(csv_path: Path, cal_out: Path) -> costmodel.CostModel:
    rows = read_csv(csv_path)
    before = costmodel.CostModel.load()
    model = costmodel.fit(rows)
    e0 = np.abs(costmodel.relative_errors(before, rows))
    e1 = np.abs(costmodel.relative_errors(model, rows))
    header = [f"sweep: {csv_path.name}, {len(rows)} points",
              f"relative error |pred/meas - 1|: mean {e1.mean():.3f}, max {e1.max():.3f} "
              f"(defaults: mean {e0.mean():.3f}, max {e0.max():.3f})"]
    model.save(cal_out, header)
    print("\n".join(header))
    for r in planner_report(model, rows):
        print(f"{r['name']:30s} best {r['best']:>9s} {r['best_us']:9.2f} us | model pick {r['model']:>9s} "
              f"{r['model_us']:9.2f} us | launcher default {r['suggested_us']:9.2f} us")
    return model


def main(argv: Optional[Sequence[str]] = None) -> None:
    ap = argparse.ArgumentParser(prog="python -m kvforge_b200.sweep")
    sub = ap.add_subparsers(dest="cmd", required=True)
    rp = sub.add_parser("run", help="time the grid on cuda:0")
    rp.add_argument("--out", type=Path, required=True)
    rp.add_argument("--quick", action="store_true")
    rp.add_argument("--reps", type=int, default=15)
    cp = sub.add_parser("calibrate", help="fit the cost model to a sweep CSV")
    cp.add_argument("csv", type=Path)
    cp.add_argument("--cal", type=Path, default=costmodel.DEFAULT_CAL)
    a = ap.parse_args(argv)
    if a.cmd == "run":
        run(a.out, a.quick, a.reps)
    else:
        calibrate(a.csv, a.cal)


if __name__ == "__main__":
    sys.exit(main())
