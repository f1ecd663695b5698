"""Parity of the sm_100a kernels with the reference, through the C ABI.

* quantizer: bit-exact with kvf::quantize (runtime/kvf_host.h:72-120);
* decode: every plan of the reference's own edge-shape verification run
  (results/edge_check.csv -> tests/golden/edge_plans.csv) launched by its
  variant id, checked against the reference's fp64 attention outputs
  (tests/golden/attention.npz) within max-abs 2e-3, max-rel 1e-2 and the
  reference's rel-L2 < 2e-3;
* the five benchmark configurations at full size against the oracle
  (every sequence, config 5 in chunks of 8), ragged and empty sequences, split
  invariance, argument errors.
"""
from __future__ import annotations

import csv
import ctypes

import numpy as np
import pytest

from conftest import GOLDEN, assert_close
from oracle import oracle as O

torch = pytest.importorskip("torch")

from kvforge_b200 import FMT_F16, FMT_INT4, FMT_INT8, ORD_HEAD, ORD_TOKEN  # noqa: E402
from kvforge_b200 import api, workloads  # noqa: E402
from kvforge_b200._native import KvfError, check, lib  # noqa: E402
from kvforge_b200.layout import Placement  # noqa: E402

pytestmark = pytest.mark.gpu

FMTS = {"f16": FMT_F16, "int8": FMT_INT8, "int4": FMT_INT4}
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


def run(q, K, V, fmt, group, place, splits, seq_lens=None, variant=None, device="cuda:0", fused=True,
        path="auto"):
    """One decode through api.decode (variant None) or through the registry by
    variant id; path "tc" / "mma" pins the kernel (the id gets its suffix)."""
    qd = torch.as_tensor(q, device=device)
    Kd = torch.as_tensor(K, device=device)
    Vd = torch.as_tensor(V, device=device)
    cache = api.KVCache.from_logical(Kd, Vd, fmt=fmt, group=group, place=place, seq_lens=seq_lens)
    out = torch.full_like(qd, float("nan"))
    ws = api.Workspace.allocate(q.shape[0], q.shape[1], q.shape[2], splits, qd.device, fused=fused)
    if variant is None:
        api.decode(qd, cache, out=out, workspace=ws, path=path)
    else:
        a = api.make_args(qd, cache, out, ws)
        vid = variant + {"auto": "", "tc": "_tc", "mma": "_mma"}[path]
        check("kvf_b200_launch_variant",
              lib().kvf_b200_launch_variant(vid.encode(), ctypes.byref(a),
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    return out.cpu().numpy()


INT8_128 = {"f16": False, "int8": True, "int4": False}


@pytest.fixture(params=["auto", "tcgen05", "mma.sync"])
def kernel_path(request):
    """Runs a test on the default kernel choice and on each int8 kernel forced
    (see path_for)."""
    return request.param


def path_for(kernel_path, fmt, d):
    """The path argument for a kernel_path variant: "tcgen05" pins the
    tcgen05 kernel wherever it applies (int8 rows of 128 dimensions) and the
    mma.sync kernel elsewhere, "mma.sync" pins the mma.sync kernel."""
    if kernel_path == "auto":
        return "auto"
    return "tc" if kernel_path == "tcgen05" and fmt == FMT_INT8 and d == 128 else "mma"


def skip_if_path_irrelevant(kernel_path, fmt, d):
    """The forced variants only differ from "auto" for int8 rows of 128."""
    if kernel_path != "auto" and not (fmt == FMT_INT8 and d == 128):
        pytest.skip("kernel choice applies to int8, d=128 only")


@pytest.fixture(scope="module")
def afix():
    return np.load(GOLDEN / "attention.npz")


# ------------------------------------------------------------------ quantizer
@pytest.mark.parametrize("fmt,group", [(FMT_INT8, 64), (FMT_INT8, 128), (FMT_INT4, 32), (FMT_INT4, 64),
                                       (FMT_INT4, 128)])
@pytest.mark.parametrize("d", [64, 128])
def test_quantize_bit_exact(cuda, fmt, group, d):
    if group > d:
        pytest.skip("group larger than the row")
    qfix = np.load(GOLDEN / "quantize.npz")
    name = {FMT_INT8: "int8", FMT_INT4: "int4"}[fmt]
    X = qfix[f"{name}:{group}_d{d}/x"]
    rs = np.random.RandomState(d + group)
    X = np.concatenate([X, (rs.standard_normal((4096, d)) * 3).astype(np.float32)])
    data, meta = api.quantize(torch.as_tensor(X, device=cuda), fmt, group)
    rd, rm, _ = O.quantize(fmt, d, group, X)
    assert np.array_equal(data.cpu().numpy(), rd)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), rm)
    # and the reference's own bytes for the fixture rows
    n0 = qfix[f"{name}:{group}_d{d}/x"].shape[0]
    assert np.array_equal(data.cpu().numpy()[:n0], qfix[f"{name}:{group}_d{d}/data"])


@pytest.mark.parametrize("fmt,group", [(FMT_F16, 0), (FMT_INT8, 64), (FMT_INT8, 128), (FMT_INT4, 32),
                                       (FMT_INT4, 128)])
@pytest.mark.parametrize("d", [64, 128])
def test_quantize_special_values_bit_exact(cuda, fmt, group, d):
    """Rows with NaN (any sign and payload, first in a group and inside one),
    +-inf, +-0 and values beyond the fp16 range: the device bytes and
    metadata equal the oracle's, which the CPU tests pin to the reference's
    own quantizer on the same kind of rows."""
    if group > d:
        pytest.skip("group larger than the row")
    rs = np.random.RandomState(d + group + 5)
    specials = np.array([0x7fc00000, 0xffc00000, 0x7f800001, 0xff800001, 0x7fffffff, 0x7f800000, 0xff800000,
                         0x00000000, 0x80000000, 0x49742400, 0xc9742400, 0x477fe000, 0x477ff000],
                        dtype=np.uint32).view(np.float32)
    X = rs.standard_normal((512, d)).astype(np.float32)
    m = rs.rand(*X.shape) < 0.05
    X[m] = rs.choice(specials, int(m.sum()))
    X[::7, 0] = np.nan
    X[::5, d // 2 + 1] = -np.nan
    data, meta = api.quantize(torch.as_tensor(X, device=cuda), fmt, group)
    rd, rm, _ = O.quantize(fmt, d, group, X)
    assert np.array_equal(data.cpu().numpy().view(np.uint8), np.asarray(rd).view(np.uint8).reshape(data.shape))
    if meta is not None:
        assert np.array_equal(meta.cpu().numpy().view(np.uint32), rm)


def test_quantize_f16_bits(cuda):
    f = np.load(GOLDEN / "f16.npz")
    data, meta = api.quantize(torch.as_tensor(f["x"].reshape(-1, 64), device=cuda), FMT_F16)
    assert meta is None
    assert np.array_equal(data.cpu().numpy().view(np.uint16).reshape(-1), f["bits"])


# -------------------------------------------- the reference's own verification
def _edge_plans():
    with open(GOLDEN / "edge_plans.csv") as f:
        return list(csv.DictReader(f))


def _variant_id(r):
    g = int(r["H"]) // int(r["H_kv"])
    pack = g if r["gqa_pack"] == "1" else 1
    return (f"{r['fmt']}_{'hm' if r['order'] == 'head_major' else 'tm'}_"
            f"{'p' if r['residency'] == 'paged' else 'c'}_g{pack}_u2_d{r['d']}")


@pytest.mark.parametrize("shape_name", list(EDGE_SHAPES))
def test_reference_edge_plans(cuda, afix, shape_name, kernel_path):
    """Every plan the reference verified for this edge shape, by variant id."""
    shape = EDGE_SHAPES[shape_name]
    q, K, V = edge_inputs(shape, int(afix[f"{shape_name}/seed"][0]))
    rows = [r for r in _edge_plans() if r["name"] == shape_name]
    assert rows
    worst = {}
    for r in rows:
        fmt = FMTS[r["fmt"]]
        group = int(r["group"])
        fname = "f16" if fmt == FMT_F16 else f"{r['fmt']}:{group}"
        place = Placement(ORD_HEAD if r["order"] == "head_major" else ORD_TOKEN, r["residency"] == "paged",
                          int(r["block_tokens"]))
        got = run(q, K, V, fmt, group, place, int(r["splits"]), variant=_variant_id(r),
                  path=path_for(kernel_path, fmt, int(r["d"])))
        st = assert_close(got, afix[f"{shape_name}/{fname}"], f"{shape_name} {fname} {place.name} s={r['splits']}")
        worst[fname] = max(worst.get(fname, 0.0), st["rel_l2"])
    # the reference's kernels reported rel-L2 ~2e-7 against the same oracle
    assert max(worst.values()) < 1e-5, worst


# ------------------------------------------------------------ configurations
def _oracle_for(w, q, K, V, seq_lens, b_sel=None):
    """Dequantise on the host with the oracle quantizer and run the fp64
    oracle, optionally on a subset of sequences."""
    if b_sel is not None:
        q, K, V = q[b_sel], K[b_sel], V[b_sel]
        seq_lens = None if seq_lens is None else seq_lens[b_sel]
    _, _, kd = O.quantize(w.fmt, w.d, w.group, K.reshape(-1, w.d))
    _, _, vd = O.quantize(w.fmt, w.d, w.group, V.reshape(-1, w.d))
    return O.attention(q, kd.reshape(K.shape), vd.reshape(V.shape), O.scale_f32(w.d), seq_lens=seq_lens)


@pytest.mark.parametrize("name", workloads.CONFIG_ORDER)
def test_config_parity(cuda, name, kernel_path):
    w = workloads.CONFIGS[name]
    skip_if_path_irrelevant(kernel_path, w.fmt, w.d)
    qd, Kd, Vd, seq_lens = workloads.generate(w, cuda)
    cache = api.KVCache.from_logical(Kd, Vd, fmt=w.fmt, group=w.group, place=w.place, seq_lens=seq_lens)
    out = api.decode(qd, cache, splits=api.suggest_splits(cache, w.H), path=path_for(kernel_path, w.fmt, w.d))
    torch.cuda.synchronize()
    # Every sequence, in chunks of 8 (config 5's logical fp32 K and V are
    # 4.3 GB each; a chunk keeps ~2 GB of them on the host at a time).
    for b0 in range(0, w.B, 8):
        sel = slice(b0, min(w.B, b0 + 8))
        q = qd[sel].cpu().numpy()
        K = Kd[sel].cpu().numpy()
        V = Vd[sel].cpu().numpy()
        ref = _oracle_for(w, q, K, V, None if seq_lens is None else seq_lens[sel])
        del K, V
        assert_close(out[sel].cpu().numpy(), ref, f"{name} sequences {b0}..{sel.stop - 1}")
    assert api.device_errors() == 0


@pytest.mark.parametrize("fmt,group", [(FMT_F16, 0), (FMT_INT8, 64), (FMT_INT4, 32)])
@pytest.mark.parametrize("place", [Placement(ORD_HEAD, False, 0), Placement(ORD_TOKEN, False, 0),
                                   Placement(ORD_HEAD, True, 32), Placement(ORD_TOKEN, True, 16)],
                         ids=lambda p: p.name)
def test_ragged_and_empty_sequences(cuda, fmt, group, place, kernel_path):
    skip_if_path_irrelevant(kernel_path, fmt, 128)
    rs = np.random.RandomState(11)
    B, H, Hkv, D, n = 7, 16, 4, 128, 700
    q = rs.standard_normal((B, H, D)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    lens = np.array([700, 0, 1, 15, 17, 64, 333], dtype=np.int32)
    _, _, kd = O.quantize(fmt, D, group, K.reshape(-1, D))
    _, _, vd = O.quantize(fmt, D, group, V.reshape(-1, D))
    ref = O.attention(q, kd.reshape(K.shape), vd.reshape(V.shape), O.scale_f32(D), seq_lens=lens)
    for splits in (1, 3, 8):
        got = run(q, K, V, fmt, group, place, splits, seq_lens=lens, path=path_for(kernel_path, fmt, D))
        assert_close(got, ref, f"{place.name} splits={splits}")
        assert np.all(got[1] == 0.0)


def test_nan_rows_past_sequence_end_are_ignored(cuda):
    """f16 rows after a sequence's last token may hold any bits."""
    rs = np.random.RandomState(12)
    B, H, Hkv, D, n = 2, 8, 2, 128, 96
    q = rs.standard_normal((B, H, D)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    lens = np.array([50, 81], dtype=np.int32)
    place = Placement(ORD_HEAD, False, 0)
    cache = api.KVCache.from_logical(torch.as_tensor(K, device=cuda), torch.as_tensor(V, device=cuda),
                                     fmt=FMT_F16, place=place, seq_lens=lens)
    # Poison every stored row past each sequence's length with NaN bits.
    for b in range(B):
        for h in range(Hkv):
            r0 = (b * Hkv + h) * n
            cache.k.view(torch.int16)[r0 + lens[b]: r0 + n] = 0x7E00
            cache.v.view(torch.int16)[r0 + lens[b]: r0 + n] = 0x7E00
    qd = torch.as_tensor(q, device=cuda)
    ref = O.attention(q, O.h2f(O.f2h(K)), O.h2f(O.f2h(V)), O.scale_f32(D), seq_lens=lens)
    for splits in (1, 2):
        got = api.decode(qd, cache, splits=splits).cpu().numpy()
        assert_close(got, ref, f"splits={splits}")


def test_split_count_does_not_change_the_result(cuda, kernel_path):
    rs = np.random.RandomState(13)
    B, H, Hkv, D, n = 2, 32, 8, 128, 5000
    q = rs.standard_normal((B, H, D)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    place = Placement(ORD_TOKEN, True, 64)
    outs = [run(q, K, V, FMT_INT8, 64, place, s, path=path_for(kernel_path, FMT_INT8, D))
            for s in (1, 2, 5, 16, 64, 313)]
    for o in outs[1:]:
        assert np.abs(o - outs[0]).max() < 1e-5


@pytest.mark.parametrize("fmt,group,place,d,gq,n,splits", [
    (FMT_F16, 0, Placement(ORD_HEAD, False, 0), 128, 1, 4096, 37),      # mha: 8 head groups x 37
    (FMT_INT8, 64, Placement(ORD_TOKEN, False, 0), 128, 4, 9000, 48),   # gqa int8: 2 head groups x 48
    (FMT_INT4, 32, Placement(ORD_HEAD, False, 0), 128, 4, 5000, 48),    # gqa int4, some splits empty
    (FMT_F16, 0, Placement(ORD_TOKEN, False, 0), 64, 2, 3000, 64),      # d=64, the most splits f16 takes
    (FMT_INT8, 64, Placement(ORD_TOKEN, False, 0), 128, 4, 20000, 147),  # int8: a whole wave, late splits empty
    (FMT_INT4, 32, Placement(ORD_HEAD, False, 0), 128, 4, 30000, 147),   # int4: a whole wave
])
def test_tail_merge_matches_the_merge_kernel(cuda, fmt, group, place, d, gq, n, splits):
    """A single sequence on the mma.sync kernel with split counters in one
    wave (at most 160 splits for int8 and int4, 64 for f16): the last
    finishers of each head group merge
    the splits inside the launch. The result equals the separate merge
    kernel's bit for bit (the same merge arithmetic), matches the oracle, and
    the counters are back at zero after every call."""
    rs = np.random.RandomState(21)
    B, Hkv = 1, 8
    H = Hkv * gq
    q = rs.standard_normal((B, H, d)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, d)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, d)).astype(np.float32)
    _, _, kq = O.quantize(fmt, d, group, K.reshape(-1, d))
    _, _, vq = O.quantize(fmt, d, group, V.reshape(-1, d))
    ref = O.attention(q, kq.reshape(K.shape), vq.reshape(V.shape), O.scale_f32(d))
    qd = torch.as_tensor(q, device=cuda)
    cache = api.KVCache.from_logical(torch.as_tensor(K, device=cuda), torch.as_tensor(V, device=cuda),
                                     fmt=fmt, group=group, place=place)
    ws = api.Workspace.allocate(B, H, d, splits, cuda, fused=True)
    assert "merge=in-kernel(tail)" in api.describe(qd, cache, ws, path="mma")
    outs = []
    for _ in range(3):
        outs.append(api.decode(qd, cache, workspace=ws, path="mma").cpu().numpy())
        assert int(ws.split_sem.abs().sum()) == 0
    two = api.decode(qd, cache, workspace=ws, path="mma", flags=api.FLAG_MERGE_KERNEL).cpu().numpy()
    for o in outs:
        assert np.array_equal(o, two)
    assert_close(outs[0], ref, f"tail merge fmt={fmt} d={d} splits={splits}")
    assert api.device_errors() == 0


@pytest.mark.parametrize("fmt,group,place,d,gq", [
    (FMT_INT8, 64, Placement(ORD_TOKEN, True, 16), 128, 4),
    (FMT_INT8, 128, Placement(ORD_HEAD, False, 0), 128, 8),
    (FMT_F16, 0, Placement(ORD_HEAD, False, 0), 128, 1),
])
def test_in_kernel_split_merge_matches_two_launch_merge(cuda, fmt, group, place, d, gq, kernel_path):
    skip_if_path_irrelevant(kernel_path, fmt, d)
    """With split counters the last block of each (sequence, KV head) merges
    the partials itself; checked against the reference's two-launch scheme and
    the oracle on ragged sequences, twice in a row (the counters must be back
    at zero after each call)."""
    rs = np.random.RandomState(16)
    B, Hkv, n = 3, 4, 2500
    H = Hkv * gq
    q = rs.standard_normal((B, H, d)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, d)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, d)).astype(np.float32)
    lens = np.array([2500, 700, 0], dtype=np.int32)
    _, _, kq = O.quantize(fmt, d, group, K.reshape(-1, d))
    _, _, vq = O.quantize(fmt, d, group, V.reshape(-1, d))
    ref = O.attention(q, kq.reshape(K.shape), vq.reshape(V.shape), O.scale_f32(d), seq_lens=lens)
    qd = torch.as_tensor(q, device=cuda)
    cache = api.KVCache.from_logical(torch.as_tensor(K, device=cuda), torch.as_tensor(V, device=cuda),
                                     fmt=fmt, group=group, place=place, seq_lens=lens)
    for splits in (2, 7, 24):
        fused_ws = api.Workspace.allocate(B, H, d, splits, cuda, fused=True)
        path = path_for(kernel_path, fmt, d)
        for _ in range(2):
            got = api.decode(qd, cache, workspace=fused_ws, path=path).cpu().numpy()
            assert_close(got, ref, f"in-kernel merge, splits={splits}")
        assert int(fused_ws.split_sem.abs().sum()) == 0
        two = api.decode(qd, cache, workspace=api.Workspace.allocate(B, H, d, splits, cuda, fused=False), path=path)
        assert np.abs(got - two.cpu().numpy()).max() < 1e-5, f"splits={splits}"
    assert api.device_errors() == 0


def test_auto_path_switches_kernel_at_32_units(cuda):
    """AUTO takes the mma.sync kernel for 8 (sequence, KV head) units and the
    tcgen05 kernel from 32; pinned paths take theirs regardless. No
    environment variable steers the choice."""
    rs = np.random.RandomState(17)
    for B, want in ((1, "mma.sync"), (4, "tcgen05")):
        K = torch.as_tensor(rs.standard_normal((B, 8, 512, 128)).astype(np.float32), device=cuda)
        cache = api.KVCache.from_logical(K, K, fmt=FMT_INT8, group=64, place=Placement(ORD_TOKEN, False, 0))
        q = torch.zeros((B, 32, 128), dtype=torch.float32, device=cuda)
        ws = api.Workspace.allocate(B, 32, 128, 4, cuda)
        assert api.describe(q, cache, ws).startswith(f"kernel={want}")
        assert api.describe(q, cache, ws, path="tc").startswith("kernel=tcgen05")
        assert api.describe(q, cache, ws, path="mma").startswith("kernel=mma.sync")
    with pytest.raises(KvfError):
        api.describe(q, cache, ws, path="mma", flags=api.FLAG_MERGE_KERNEL | api.FLAG_GRID_MERGE)
    with pytest.raises(KvfError):
        api.describe(q, cache, ws, flags=0x800)


@pytest.mark.parametrize("place", [Placement(ORD_TOKEN, False, 0), Placement(ORD_HEAD, True, 16)],
                         ids=lambda p: p.name)
def test_path_pinned_variants_run_their_kernel(cuda, place):
    """The "_tc" / "_mma" variant ids (and api.decode(path=...)) run the named
    kernel whatever the launcher would choose, with the same results."""
    rs = np.random.RandomState(23)
    B, H, Hkv, D, n = 2, 32, 8, 128, 700
    q = rs.standard_normal((B, H, D)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    qd = torch.as_tensor(q, device=cuda)
    cache = api.KVCache.from_logical(torch.as_tensor(K, device=cuda), torch.as_tensor(V, device=cuda),
                                     fmt=FMT_INT8, group=64, place=place)
    ws = api.Workspace.allocate(B, H, D, 3, cuda)
    assert api.describe(qd, cache, ws, path="tc").startswith("kernel=tcgen05")
    assert api.describe(qd, cache, ws, path="mma").startswith("kernel=mma.sync")
    _, _, kd = O.quantize(FMT_INT8, D, 64, K.reshape(-1, D))
    _, _, vd = O.quantize(FMT_INT8, D, 64, V.reshape(-1, D))
    ref = O.attention(q, kd.reshape(K.shape), vd.reshape(V.shape), O.scale_f32(D))
    base = f"int8_{'tm' if place.order == ORD_TOKEN else 'hm'}_{'p' if place.paged else 'c'}_g4_u2_d128"
    outs = {}
    for suffix in ("_tc", "_mma", ""):
        outs[suffix] = run(q, K, V, FMT_INT8, 64, place, 3, variant=base + suffix)
        assert_close(outs[suffix], ref, base + suffix)
    for path in ("tc", "mma"):
        got = api.decode(qd, cache, workspace=ws, path=path)
        torch.cuda.synchronize()
        assert_close(got.cpu().numpy(), ref, path)
    assert api.device_errors() == 0
    with pytest.raises(Exception):
        f16 = api.KVCache.from_logical(torch.as_tensor(K, device=cuda), torch.as_tensor(V, device=cuda),
                                       fmt=FMT_F16, group=0, place=place)
        api.decode(qd, f16, workspace=ws, path="tc")


def test_merge_entry_point_recombines_partials(cuda):
    rs = np.random.RandomState(14)
    B, H, Hkv, D, n = 1, 8, 8, 64, 1000
    q = torch.as_tensor(rs.standard_normal((B, H, D)).astype(np.float32), device=cuda)
    K = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    V = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    cache = api.KVCache.from_logical(K, V, fmt=FMT_F16, place=Placement(ORD_HEAD, False, 0))
    ws = api.Workspace.allocate(B, H, D, 4, cuda)
    out = api.decode(q, cache, workspace=ws).clone()
    again = torch.zeros_like(out)
    a = api.make_args(q, cache, again, ws)
    check("kvf_b200_merge", lib().kvf_b200_merge(ctypes.byref(a), D, None))
    torch.cuda.synchronize()
    assert torch.equal(out, again)


def test_repeated_launches_are_deterministic(cuda):
    w = workloads.CONFIGS[workloads.HEADLINE]
    qd, Kd, Vd, sl = workloads.generate(w, cuda)
    cache = api.KVCache.from_logical(Kd, Vd, fmt=w.fmt, group=w.group, place=w.place, seq_lens=sl)
    ws = api.Workspace.allocate(w.B, w.H, w.d, api.suggest_splits(cache, w.H), cuda)
    first = api.decode(qd, cache, workspace=ws).clone()
    for _ in range(5):
        assert torch.equal(api.decode(qd, cache, workspace=ws), first)


def test_errors_surface_as_codes(cuda):
    rs = np.random.RandomState(15)
    q = torch.as_tensor(rs.standard_normal((1, 8, 128)).astype(np.float32), device=cuda)
    K = torch.as_tensor(rs.standard_normal((1, 8, 64, 128)).astype(np.float32), device=cuda)
    cache = api.KVCache.from_logical(K, K, fmt=FMT_INT8, group=64, place=Placement(ORD_HEAD, False, 0))
    out = torch.empty_like(q)
    ws = api.Workspace.allocate(1, 8, 128, 2, cuda)
    a = api.make_args(q, cache, out, ws)
    a.k_meta = None
    assert lib().kvf_b200_decode(ctypes.byref(a), FMT_INT8, 128, 1, 0, 0, None) == 1
    a = api.make_args(q, cache, out, ws)
    a.part_o = None
    assert lib().kvf_b200_decode(ctypes.byref(a), FMT_INT8, 128, 1, 0, 0, None) == 1
    a = api.make_args(q, cache, out, ws)
    a.v = a.v + 8
    assert lib().kvf_b200_decode(ctypes.byref(a), FMT_INT8, 128, 1, 0, 0, None) == 716
    assert api.device_errors() == 0


@pytest.mark.parametrize("zero_copy", [True, False], ids=["zero_copy", "copies"])
@pytest.mark.parametrize("fmt,group,place", [
    (FMT_INT8, 64, Placement(ORD_TOKEN, False, 0)),
    (FMT_F16, 0, Placement(ORD_HEAD, True, 16)),
    (FMT_INT8, 128, Placement(ORD_TOKEN, True, 16)),
], ids=["int8_tm", "f16_hm_p16", "int8_tm_p16"])
def test_decoder_graph_replays_match_direct_decode(cuda, fmt, group, place, zero_copy):
    """api.Decoder (one CUDA graph per step: queries from and output to pinned
    host memory, with or without copy-engine transfers) gives what api.decode
    gives, step after step, for new queries and a changed cache."""
    rs = np.random.RandomState(31)
    B, H, Hkv, D, n = 2, 16, 4, 128, 900
    K = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    V = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    cache = api.KVCache.from_logical(K, V, fmt=fmt, group=group, place=place)
    dec = api.Decoder(cache, H, splits=5, zero_copy=zero_copy)
    assert dec.graph is not None
    for step in range(3):
        q = torch.as_tensor(rs.standard_normal((B, H, D)).astype(np.float32))
        got = dec.step(q).clone()
        want = api.decode(q.to(cuda), cache, splits=5).cpu()
        assert torch.equal(got, want), step
    # The graph reads the cache in place: new contents show up in the next step.
    if fmt == FMT_F16:
        cache.v.zero_()
        assert torch.count_nonzero(dec.step(q)) == 0
    assert api.device_errors() == 0


@pytest.mark.parametrize("zero_copy", [True, False], ids=["zero_copy", "copies"])
@pytest.mark.parametrize("kernel", ["tc", "mma"])
def test_decoder_graph_on_each_int8_kernel(cuda, zero_copy, kernel):
    """The same with 32 KV-head units (the tcgen05 kernel's range) on each
    int8 kernel: the staged queries and the output in pinned host memory
    equal api.decode on the same path bit for bit, and the oracle."""
    rs = np.random.RandomState(37)
    B, H, Hkv, D, n = 8, 32, 4, 128, 700
    K = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    V = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    lens = np.array([700, 1, 333, 0, 512, 699, 128, 129], dtype=np.int32)
    cache = api.KVCache.from_logical(K, V, fmt=FMT_INT8, group=64, place=Placement(ORD_TOKEN, True, 16),
                                     seq_lens=lens)
    dec = api.Decoder(cache, H, splits=3, zero_copy=zero_copy, path=kernel)
    assert f"kernel={'tcgen05' if kernel == 'tc' else 'mma.sync'}" in api.describe(
        dec.q, cache, dec.workspace, path=kernel)
    Kn, Vn = K.cpu().numpy(), V.cpu().numpy()
    _, _, kq = O.quantize(FMT_INT8, D, 64, Kn.reshape(-1, D))
    _, _, vq = O.quantize(FMT_INT8, D, 64, Vn.reshape(-1, D))
    for step in range(3):
        q = torch.as_tensor(rs.standard_normal((B, H, D)).astype(np.float32))
        got = dec.step(q).clone()
        want = api.decode(q.to(cuda), cache, splits=3, path=kernel).cpu()
        assert torch.equal(got, want), step
        ref = O.attention(q.numpy(), kq.reshape(Kn.shape), vq.reshape(Vn.shape), O.scale_f32(D), seq_lens=lens)
        assert_close(got.numpy(), ref, f"decoder {kernel} step {step}")
    assert api.device_errors() == 0


@pytest.mark.parametrize("fused", [True, False], ids=["in_kernel_merge", "merge_kernel"])
@pytest.mark.parametrize("place", [Placement(ORD_TOKEN, True, 16), Placement(ORD_HEAD, False, 0)],
                         ids=lambda p: p.name)
def test_decode_from_host_on_the_tcgen05_path(cuda, fused, place):
    """kvf_b200_decode_from_host on the tcgen05 path with more blocks than one
    wave: 12 sequences x 8 KV heads x 12 splits, 96 blocks a sequence, so on
    148 SMs x 2 sequences 0-2 are staged and decoded first and sequences 3-11
    (295 KB of queries) staged beside that decode and decoded after it.
    Ragged lengths, output to pinned host memory, lse on the device: equal to
    api.decode bit for bit, directly and in a captured graph, with either
    merge."""
    rs = np.random.RandomState(43)
    B, H, Hkv, D, n, S = 12, 64, 8, 128, 300, 12
    K = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    V = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    lens = rs.randint(0, n + 1, B).astype(np.int32)
    lens[0] = n
    cache = api.KVCache.from_logical(K, V, fmt=FMT_INT8, group=64, place=place, seq_lens=lens)
    q = rs.standard_normal((B, H, D)).astype(np.float32)
    qd = torch.as_tensor(q, device=cuda)
    want_out = torch.empty_like(qd)
    want_lse = torch.empty((B, H), device=cuda)
    api.decode(qd, cache, out=want_out, lse=want_lse, splits=S, path="tc",
               workspace=api.Workspace.allocate(B, H, D, S, cuda, fused=fused))
    q_host = torch.as_tensor(q).pin_memory()
    out_host = torch.full((B, H, D), float("nan")).pin_memory()
    lse = torch.full((B, H), float("nan"), device=cuda)
    ws = api.Workspace.allocate(B, H, D, S, cuda, fused=fused)
    qbuf = torch.zeros_like(qd)
    a = api.make_args(qbuf, cache, want_out, ws)
    a.out = out_host.data_ptr()
    a.lse = lse.data_ptr()
    g = H // Hkv

    def issue():  # on the current stream (the capture stream inside the graph)
        check("kvf_b200_decode_from_host",
              lib().kvf_b200_decode_from_host(ctypes.byref(a), FMT_INT8, D, g, place.order, int(place.paged),
                                              api.PATHS["tc"], ctypes.c_void_p(q_host.data_ptr()),
                                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))

    issue()
    torch.cuda.synchronize()
    assert torch.equal(out_host, want_out.cpu())
    assert torch.equal(lse, want_lse)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        issue()
    out_host.fill_(float("nan"))
    lse.fill_(float("nan"))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out_host, want_out.cpu())
    assert torch.equal(lse, want_lse)
    if fused:
        assert int(ws.split_sem.abs().sum()) == 0
    assert api.device_errors() == 0


def test_decode_from_host_rejects_pageable_buffers(cuda):
    """Host buffers the device cannot address are refused before any launch."""
    rs = np.random.RandomState(32)
    K = torch.as_tensor(rs.standard_normal((1, 2, 64, 128)).astype(np.float32), device=cuda)
    cache = api.KVCache.from_logical(K, K, fmt=FMT_F16, place=Placement(ORD_HEAD, False, 0))
    qd = torch.zeros((1, 8, 128), dtype=torch.float32, device=cuda)
    out = torch.zeros_like(qd)
    ws = api.Workspace.allocate(1, 8, 128, 1, cuda)
    a = api.make_args(qd, cache, out, ws)
    pageable = np.zeros((1, 8, 128), dtype=np.float32)
    pinned = torch.zeros((1, 8, 128), dtype=torch.float32).pin_memory()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    f = lib().kvf_b200_decode_from_host
    assert f(ctypes.byref(a), FMT_F16, 128, 1, ORD_HEAD, 0, 0, ctypes.c_void_p(pageable.ctypes.data), st) == 1
    a.out = pageable.ctypes.data
    assert f(ctypes.byref(a), FMT_F16, 128, 1, ORD_HEAD, 0, 0, ctypes.c_void_p(pinned.data_ptr()), st) == 1
    a.out = out.data_ptr()
    assert f(ctypes.byref(a), FMT_F16, 128, 1, ORD_HEAD, 0, 0, ctypes.c_void_p(pinned.data_ptr()), st) == 0
    torch.cuda.synchronize()
    assert api.device_errors() == 0


@pytest.mark.parametrize("B,H,Hkv,n,fmt,group,place", [
    (1, 32, 8, 3000, FMT_INT8, 64, Placement(ORD_TOKEN, False, 0)),
    (6, 16, 4, 1500, FMT_F16, 0, Placement(ORD_TOKEN, True, 16)),
], ids=["b1_int8_tm", "b6_f16_tm_p16"])
def test_in_launch_grid_merge_equals_merge_kernel(cuda, B, H, Hkv, n, fmt, group, place):
    """The mma.sync kernel's split merge after a grid barrier (cooperative
    launch) gives the merge kernel's result bit for bit, launch after launch
    (its barrier counters return to zero)."""
    rs = np.random.RandomState(41)
    q = torch.as_tensor(rs.standard_normal((B, H, 128)).astype(np.float32), device=cuda)
    K = torch.as_tensor(rs.standard_normal((B, Hkv, n, 128)).astype(np.float32), device=cuda)
    V = torch.as_tensor(rs.standard_normal((B, Hkv, n, 128)).astype(np.float32), device=cuda)
    cache = api.KVCache.from_logical(K, V, fmt=fmt, group=group, place=place)
    ws = api.Workspace.allocate(B, H, 128, 7, cuda)
    outs = {}
    for mode, flags in (("0", api.FLAG_MERGE_KERNEL), ("1", api.FLAG_GRID_MERGE)):
        desc = api.describe(q, cache, ws, path="mma", flags=flags)
        assert ("merge=in-kernel(grid)" in desc) == (mode == "1"), desc
        for _ in range(3):
            outs[mode] = api.decode(q, cache, workspace=ws, path="mma", flags=flags).clone()
        torch.cuda.synchronize()
        assert int(ws.split_sem.abs().sum()) == 0
    assert torch.equal(outs["0"], outs["1"])
    assert api.device_errors() == 0


@pytest.mark.parametrize("fmt,group,place", [
    (FMT_F16, 0, Placement(ORD_TOKEN, True, 16)),
    (FMT_INT8, 64, Placement(ORD_HEAD, False, 0)),
], ids=["f16_tm_p16", "int8_hm"])
def test_balanced_splits_on_ragged_batches(cuda, fmt, group, place):
    """Sequences of unequal length share one chunk of tokens (the mma.sync
    launch balances them over one wave of blocks): the device picks the chunk
    kvf_b200_balanced_chunk computes on the host (each sequence's partials
    fill exactly its first ceil(len / chunk) split slots), the output matches
    the oracle, and the cooperative in-launch merge, the merge kernel and a
    zero-copy Decoder step (merge kernel after a dependent launch) agree bit
    for bit."""
    rs = np.random.RandomState(43)
    B, H, Hkv, D, n = 8, 32, 8, 128, 2048
    lens = np.array([2048, 0, 1, 700, 1999, 64, 1500, 333], dtype=np.int32)
    q = rs.standard_normal((B, H, D)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    _, _, kd = O.quantize(fmt, D, group, K.reshape(-1, D))
    _, _, vd = O.quantize(fmt, D, group, V.reshape(-1, D))
    ref = O.attention(q, kd.reshape(K.shape), vd.reshape(V.shape), O.scale_f32(D), seq_lens=lens)
    qd = torch.as_tensor(q, device=cuda)
    cache = api.KVCache.from_logical(torch.as_tensor(K, device=cuda), torch.as_tensor(V, device=cuda),
                                     fmt=fmt, group=group, place=place, seq_lens=lens)
    # The suggestion follows the AUTO kernel (tcgen05 for the int8 case); the
    # test runs the mma.sync kernel, so it keeps a capacity of at least 8.
    S = max(api.suggest_splits(cache, H), 8)
    bt = place.block_tokens if place.paged else 0
    assert S >= lib().kvf_b200_suggest_splits(B, H, Hkv, n, fmt, D, group, int(place.paged), bt)
    ws = api.Workspace.allocate(B, H, D, S, cuda)
    desc = api.describe(qd, cache, ws, path="mma")
    assert "chunk=balanced" in desc, desc
    f = dict(kv.split("=", 1) for kv in desc.split() if "=" in kv)
    grid, hh = int(f["grid"]), int(f["heads/block"])
    gran = int(f["chunk"].split("gran=")[1].rstrip(")"))
    c = int(lib().kvf_b200_balanced_chunk(lens.ctypes.data_as(ctypes.c_void_p), B, n, S, Hkv // hh, grid, gran))
    assert c > 0
    sb = (lens.astype(np.int64) + c - 1) // c
    outs = {}
    for mode, flags in (("0", api.FLAG_MERGE_KERNEL), ("1", api.FLAG_GRID_MERGE)):
        ws.part_ml.fill_(float("nan"))
        outs[mode] = api.decode(qd, cache, workspace=ws, path="mma", flags=flags).clone()
        torch.cuda.synchronize()
        written = torch.isfinite(ws.part_ml[..., 0]).cpu().numpy()  # [B][H][S]
        want = np.arange(S)[None, None, :] < sb[:, None, None]
        assert np.array_equal(written, np.broadcast_to(want, written.shape)), mode
        assert_close(outs[mode].cpu().numpy(), ref, f"coop={mode}")
        assert int(ws.split_sem.abs().sum()) == 0
    assert torch.equal(outs["0"], outs["1"])
    assert np.all(outs["0"][1].cpu().numpy() == 0.0)
    dec = api.Decoder(cache, H, splits=S, path="mma")
    got = dec.step(torch.as_tensor(q))
    assert torch.equal(got, outs["1"].cpu())
    # FLAG_NO_BALANCE: one split count for all sequences, same results.
    assert "chunk=balanced" not in api.describe(qd, cache, ws, path="mma", flags=api.FLAG_NO_BALANCE)
    uni = api.decode(qd, cache, workspace=ws, path="mma", flags=api.FLAG_NO_BALANCE).cpu().numpy()
    assert_close(uni, ref, "unbalanced")
    assert np.abs(uni - outs["1"].cpu().numpy()).max() < 1e-5
    assert api.device_errors() == 0


def test_balanced_splits_fall_back_when_units_exceed_one_wave(cuda):
    """More (sequence, head group) units than one wave of blocks: the launch
    keeps the uniform split plan, with the same results."""
    rs = np.random.RandomState(44)
    B, H, Hkv, D, n = 320, 4, 4, 64, 40
    lens = rs.randint(0, n + 1, size=B).astype(np.int32)
    q = rs.standard_normal((B, H, D)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    ref = O.attention(q, O.h2f(O.f2h(K)), O.h2f(O.f2h(V)), O.scale_f32(D), seq_lens=lens)
    qd = torch.as_tensor(q, device=cuda)
    cache = api.KVCache.from_logical(torch.as_tensor(K, device=cuda), torch.as_tensor(V, device=cuda),
                                     fmt=FMT_F16, place=Placement(ORD_HEAD, False, 0), seq_lens=lens)
    ws = api.Workspace.allocate(B, H, D, 3, cuda)
    desc = api.describe(qd, cache, ws)
    assert "chunk=balanced" not in desc, desc
    assert_close(api.decode(qd, cache, workspace=ws).cpu().numpy(), ref, "uniform plan")
    assert api.device_errors() == 0
