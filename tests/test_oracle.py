"""The oracle (oracle/kvf_oracle.c) pinned against the reference's own
outputs (tests/golden, generated from runtime/kvf_host.h by make_golden.py)
and against the error magnitudes the reference published for its edge
shapes (results/edge_check.csv). CPU only."""
from __future__ import annotations

import csv
import hashlib

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import oracle as O

FORMATS = {
    "f16": (O.F16, 0), "int8:64": (O.INT8, 64), "int8:128": (O.INT8, 128),
    "int4:32": (O.INT4, 32), "int4:64": (O.INT4, 64), "int4:128": (O.INT4, 128),
}
EDGE_SHAPES = {
    "edge_n129": dict(B=1, H=32, Hkv=8, D=128, n=129),
    "edge_short": dict(B=1, H=8, Hkv=8, D=64, n=100),
    "edge_odd_n": dict(B=2, H=12, Hkv=4, D=128, n=1001),
    "edge_g8_n3333": dict(B=3, H=16, Hkv=2, D=64, n=3333),
}


def edge_inputs(shape, seed):
    rs = np.random.RandomState(seed)
    B, H, Hkv, D, n = shape["B"], shape["H"], shape["Hkv"], shape["D"], shape["n"]
    q = rs.standard_normal((B, H, D)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    return q, K, V


@pytest.fixture(scope="module")
def qfix():
    return np.load(GOLDEN / "quantize.npz")


@pytest.fixture(scope="module")
def afix():
    return np.load(GOLDEN / "attention.npz")


def test_f16_bits_match_reference():
    f = np.load(GOLDEN / "f16.npz")
    bits = O.f2h(f["x"])
    assert np.array_equal(bits, f["bits"])
    assert np.array_equal(O.h2f(bits).view(np.uint32), f["deq"].view(np.uint32))


@pytest.mark.parametrize("name", list(FORMATS))
def test_quantize_matches_reference_on_special_values(name):
    """NaN (any sign and payload, first in a group and inside one), +-inf,
    +-0 and values beyond the fp16 range, against the reference's own
    kvf::quantize built from its sources (oracle/_ref): codes, metadata words
    and dequantised values bit for bit."""
    if not O.Ref.available():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    fmt, group = FORMATS[name]
    rs = np.random.RandomState(7)
    specials = np.array([0x7fc00000, 0xffc00000, 0x7f800001, 0xff800001, 0x7fffffff, 0x7f800000, 0xff800000,
                         0x00000000, 0x80000000, 0x49742400, 0xc9742400, 0x477fe000, 0x477ff000],
                        dtype=np.uint32).view(np.float32)
    for d in (64, 128):
        if group > d:
            continue
        X = rs.standard_normal((256, d)).astype(np.float32)
        m = rs.rand(*X.shape) < 0.05
        X[m] = rs.choice(specials, int(m.sum()))
        X[::7, 0] = np.nan
        X[::5, d // 2 + 1] = -np.nan
        got = O.quantize(fmt, d, group, X)
        want = O.Ref.quantize(fmt, d, group, X)
        for g_, w_ in zip(got, want):
            if g_ is None:
                continue
            assert np.array_equal(np.asarray(g_).view(np.uint8), np.asarray(w_).view(np.uint8)), (name, d)


@pytest.mark.parametrize("key", [f"{n}_d{d}" for n in FORMATS if n != "f16" for d in (64, 128)
                                 if FORMATS[n][1] <= d])
def test_quantize_matches_reference(qfix, key):
    name, d = key.rsplit("_d", 1)
    fmt, group = FORMATS[name]
    X = qfix[f"{key}/x"]
    data, meta, deq = O.quantize(fmt, int(d), group, X)
    assert np.array_equal(data, qfix[f"{key}/data"])
    assert np.array_equal(meta, qfix[f"{key}/meta"])
    assert np.array_equal(deq.view(np.uint32), qfix[f"{key}/deq"].view(np.uint32))


@pytest.mark.parametrize("shape_name", list(EDGE_SHAPES))
def test_attention_matches_reference(afix, shape_name):
    shape = EDGE_SHAPES[shape_name]
    seed = int(afix[f"{shape_name}/seed"][0])
    q, K, V = edge_inputs(shape, seed)
    h = hashlib.sha256()
    for a in (q, K, V):
        h.update(a.tobytes())
    assert h.hexdigest() == bytes(afix[f"{shape_name}/digest"]).decode(), "input generator drifted"
    D = shape["D"]
    scale = O.scale_f32(D)
    exact = O.attention(q, K, V, scale)
    assert np.array_equal(exact.view(np.uint32), afix[f"{shape_name}/exact"].view(np.uint32))
    for fname, (fmt, group) in FORMATS.items():
        if group > D:
            continue
        _, _, kd = O.quantize(fmt, D, group, K.reshape(-1, D))
        _, _, vd = O.quantize(fmt, D, group, V.reshape(-1, D))
        out = O.attention(q, kd.reshape(K.shape), vd.reshape(V.shape), scale)
        assert np.array_equal(out.view(np.uint32), afix[f"{shape_name}/{fname}"].view(np.uint32)), fname


def test_error_magnitudes_match_published(afix):
    """Quantization error vs exact attention on N(0,1) data, as the reference
    measured it for the same shapes (err_exact of results/edge_check.csv; our
    inputs are a different N(0,1) draw, so agreement is statistical)."""
    pub = {}
    with open(GOLDEN / "edge_plans.csv") as f:
        for r in csv.DictReader(f):
            fname = "f16" if r["fmt"] == "f16" else f"{r['fmt']}:{r['group']}"
            pub.setdefault((r["name"], fname), float(r["err_exact"]))
    checked = 0
    for (sname, fname), e_pub in pub.items():
        key = f"{sname}/{fname}/err_exact"
        if key not in afix:
            continue
        ours = float(afix[key][0])
        assert 0.6 * e_pub < ours < 1.6 * e_pub, (sname, fname, ours, e_pub)
        checked += 1
    assert checked >= 15


def test_published_plans_all_verified():
    with open(GOLDEN / "edge_plans.csv") as f:
        rows = list(csv.DictReader(f))
    assert len(rows) > 500
    assert all(r["verified"] == "1" and float(r["err_ref"]) < 2e-3 for r in rows)


def test_ragged_attention_is_per_sequence_reference():
    """seq_lens: sequence b uses its first n_b tokens, exactly as the reference
    function called with Shape{B=1, n=n_b} on that sequence's rows."""
    rs = np.random.RandomState(5)
    B, H, Hkv, D, n = 3, 8, 2, 64, 200
    q = rs.standard_normal((B, H, D)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    lens = np.array([200, 77, 0], dtype=np.int32)
    scale = O.scale_f32(D)
    got = O.attention(q, K, V, scale, seq_lens=lens)
    for b in range(B):
        if lens[b] == 0:
            assert np.all(got[b] == 0)
            continue
        one = O.attention(q[b : b + 1], np.ascontiguousarray(K[b : b + 1, :, : lens[b]]),
                          np.ascontiguousarray(V[b : b + 1, :, : lens[b]]), scale)
        assert np.array_equal(got[b], one[0])
        if O.Ref.available():
            r = O.Ref.attention(q[b : b + 1], np.ascontiguousarray(K[b : b + 1, :, : lens[b]]),
                                np.ascontiguousarray(V[b : b + 1, :, : lens[b]]), scale)
            assert np.array_equal(got[b].view(np.uint32), r[0].view(np.uint32))


def test_threads_do_not_change_results():
    rs = np.random.RandomState(9)
    q = rs.standard_normal((2, 8, 128)).astype(np.float32)
    K = rs.standard_normal((2, 4, 300, 128)).astype(np.float32)
    V = rs.standard_normal((2, 4, 300, 128)).astype(np.float32)
    a = O.attention(q, K, V, 0.088, threads=1)
    b = O.attention(q, K, V, 0.088, threads=4)
    assert np.array_equal(a, b)


@pytest.mark.skipif(not O.Ref.available(), reason="reference functions not built here")
def test_row_of_matches_reference():
    rs = np.random.RandomState(3)
    B, Hkv, n = 3, 4, 70
    for order in (0, 1):
        for bt in (0, 16, 32):
            mb = (n + bt - 1) // bt if bt else 0
            table = rs.permutation(B * max(mb, 1)).astype(np.int32)
            for b in range(B):
                for h in range(Hkv):
                    for t in (0, 1, 15, 16, 17, n - 1):
                        want = O.Ref.row_of(order, int(bt > 0), bt, Hkv, n, table, mb, b, h, t)
                        assert O.row_of(order, bt, Hkv, n, table, mb, b, h, t) == want


@pytest.mark.skipif(not O.Ref.available(), reason="reference functions not built here")
def test_scale_log2_matches_make_args():
    from kvforge_b200.api import scale_log2

    for d in (64, 128):
        assert np.float32(scale_log2(d)) == np.float32(O.Ref.scale_log2(d))
