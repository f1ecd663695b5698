"""Generates the golden fixtures in this directory from the REFERENCE's own
functions (runtime/kvf_host.h, compiled unmodified into oracle/_ref by
oracle/build.py) and from the reference's published verification results.

    python tests/golden/make_golden.py        (needs the reference tree)

Fixtures (inputs are either stored or regenerated from numpy's legacy
RandomState, whose streams are fixed across numpy versions):
  quantize.npz      per (format, d, group): input rows X and the reference's
                    quantized bytes, metadata words and dequantised values
  f16.npz           fp32 values and the fp16 bits of the reference's f16
                    cache format (__float2half, round to nearest even)
  attention.npz     per (edge shape, format): fp64 attention output of the
                    reference on its own dequantised K/V, plus the exact
                    (unquantised) output; inputs regenerated from the seed
  edge_plans.csv    the plans of the reference's edge-shape verification run
                    (results/edge_check.csv) with the error each one reported
"""
from __future__ import annotations

import csv
import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import build as obuild  # noqa: E402
from oracle.oracle import F16, INT4, INT8, Ref  # noqa: E402

# Edge shapes of the reference's correctness set (tests/edge/*.kv).
EDGE_SHAPES = {
    "edge_n129": dict(B=1, H=32, Hkv=8, D=128, n=129),
    "edge_short": dict(B=1, H=8, Hkv=8, D=64, n=100),
    "edge_odd_n": dict(B=2, H=12, Hkv=4, D=128, n=1001),
    "edge_g8_n3333": dict(B=3, H=16, Hkv=2, D=64, n=3333),
}
FORMATS = {
    "f16": (F16, 0), "int8:64": (INT8, 64), "int8:128": (INT8, 128),
    "int4:32": (INT4, 32), "int4:64": (INT4, 64), "int4:128": (INT4, 128),
}


def edge_inputs(shape: dict, seed: int):
    """q [B,H,D], K, V [B,Hkv,n,D]: RandomState normal, float32."""
    rs = np.random.RandomState(seed)
    B, H, Hkv, D, n = shape["B"], shape["H"], shape["Hkv"], shape["D"], shape["n"]
    q = rs.standard_normal((B, H, D)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    return q, K, V


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def quant_rows(d: int, seed: int) -> np.ndarray:
    rs = np.random.RandomState(seed)
    X = rs.standard_normal((48, d)).astype(np.float32)
    X *= rs.choice([1e-3, 0.1, 1.0, 8.0, 300.0], size=(48, 1)).astype(np.float32)
    X[0, :] = 1.5                      # constant group: scale 0 -> 1
    X[1, :] = 0.0
    X[2, : d // 2] = -2.0              # constant half
    X[3, :] = np.linspace(-1, 1, d, dtype=np.float32)
    X[4, :] = np.float32(-0.0)
    X[5, ::2] = 1e-6
    X[6, :] = rs.standard_normal(d).astype(np.float32) * 7e4  # beyond fp16 range
    return X


def main() -> None:
    obuild.build_reference()
    if not Ref.available():
        raise SystemExit("reference tree absent: fixtures cannot be regenerated here")

    # ---------------------------------------------------------- quantizer
    q = {}
    for i, (name, (fmt, group)) in enumerate(FORMATS.items()):
        if fmt == F16:
            continue
        for d in (64, 128):
            if group > d:
                continue
            X = quant_rows(d, 100 + 10 * i + d)
            data, meta, deq = Ref.quantize(fmt, d, group, X)
            key = f"{name}_d{d}"
            q[f"{key}/x"] = X
            q[f"{key}/data"] = data
            q[f"{key}/meta"] = meta
            q[f"{key}/deq"] = deq
    np.savez_compressed(HERE / "quantize.npz", **q)

    # ---------------------------------------------------------- fp16 bits
    rs = np.random.RandomState(7)
    special = np.array(
        [0.0, -0.0, 1e-8, 2.98e-8, 2.9802322e-08, 5.96e-8, 6.0e-8, 6.1e-5, 6.103515625e-05, 1e-4,
         0.333333, 1.0, 1.00048828125, 1.0009765625, 1.00146484375, 2047.5, 2048.5, 65504.0,
         65519.99, 65520.0, 1e6, -1e6, np.inf, -np.inf],
        dtype=np.float32,
    )
    vals = np.concatenate([special, rs.standard_normal(4000).astype(np.float32) *
                           rs.choice([1e-6, 1e-3, 1, 1e3, 3e4], size=4000).astype(np.float32)])
    vals = vals[: (vals.size // 64) * 64]
    data, _, deq = Ref.quantize(F16, 64, 0, vals.reshape(-1, 64))
    np.savez_compressed(HERE / "f16.npz", x=vals, bits=data.view(np.uint16).reshape(-1), deq=deq.reshape(-1))

    # ---------------------------------------------------------- attention
    att = {}
    for si, (sname, shape) in enumerate(EDGE_SHAPES.items()):
        seed = 1000 + si
        qv, K, V = edge_inputs(shape, seed)
        D = shape["D"]
        scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
        exact = Ref.attention(qv, K, V, scale)
        att[f"{sname}/digest"] = np.frombuffer(digest(qv, K, V).encode(), dtype=np.uint8)
        att[f"{sname}/seed"] = np.array([seed])
        att[f"{sname}/exact"] = exact
        for fname, (fmt, group) in FORMATS.items():
            if group > D:
                continue
            _, _, kd = Ref.quantize(fmt, D, group, K.reshape(-1, D))
            _, _, vd = Ref.quantize(fmt, D, group, V.reshape(-1, D))
            out = Ref.attention(qv, kd.reshape(K.shape), vd.reshape(V.shape), scale)
            att[f"{sname}/{fname}"] = out
            att[f"{sname}/{fname}/err_exact"] = np.array([Ref.rel_l2(out, exact)])
    np.savez_compressed(HERE / "attention.npz", **att)

    # ---------------------------------------------------------- edge plans
    src = obuild.REFERENCE / "results" / "edge_check.csv"
    cols = ["name", "H", "H_kv", "d", "n", "batch", "fmt", "group", "order", "residency",
            "block_tokens", "splits", "gqa_pack", "err_exact", "err_ref", "verified"]
    seen = set()
    with open(src) as f, open(HERE / "edge_plans.csv", "w", newline="") as g:
        w = csv.writer(g)
        w.writerow(cols)
        for r in csv.DictReader(f):
            key = tuple(r[c] for c in cols[:13])
            if key in seen:
                continue
            seen.add(key)
            w.writerow([r[c] for c in cols])
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".csv")))


if __name__ == "__main__":
    main()
