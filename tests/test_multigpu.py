"""Multi-GPU decode (kvforge_b200.sharding) on the GPU.

* kvf_b200_merge_states: decoding disjoint token ranges separately (with the
  lse output) and combining them equals one decode over all tokens, and the
  oracle, on one GPU;
* with two or more GPUs, two ranks run the split-KV protocol (exchange fused
  into the split merge, separate NVLink push/merge kernels, NCCL all-gather;
  several steps each) and the KV-head protocol end
  to end and must match a single-GPU decode of the same inputs and the fp64
  oracle (skipped on a one-GPU box).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from conftest import assert_close
from oracle import oracle as O

torch = pytest.importorskip("torch")

from kvforge_b200 import FMT_F16, FMT_INT4, FMT_INT8, ORD_HEAD, ORD_TOKEN, api, sharding  # noqa: E402
from kvforge_b200._native import lib  # noqa: E402
from kvforge_b200.layout import Placement  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt,group,place", [
    (FMT_INT4, 32, Placement(ORD_HEAD, False, 0)),
    (FMT_INT8, 64, Placement(ORD_TOKEN, True, 16)),
    (FMT_F16, 0, Placement(ORD_TOKEN, False, 0)),
])
def test_merge_states_over_token_ranges_equals_one_decode(cuda, fmt, group, place):
    rs = np.random.RandomState(41)
    B, H, Hkv, D, n, P = 2, 32, 8, 128, 3000, 3
    q = torch.as_tensor(rs.standard_normal((B, H, D)).astype(np.float32), device=cuda)
    K = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    V = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    lens = np.array([3000, 1100], dtype=np.int32)
    full = api.decode(q, api.KVCache.from_logical(K, V, fmt=fmt, group=group, place=place, seq_lens=lens))
    outs = torch.empty((P, B, H, D), device=cuda)
    lses = torch.empty((P, B, H), device=cuda)
    for r in range(P):
        t0, t1 = sharding.token_range(n, P, r)
        ll = sharding.local_seq_lens(lens, n, t0, t1)
        part = api.KVCache.from_logical(K[:, :, t0:t1].contiguous(), V[:, :, t0:t1].contiguous(), fmt=fmt,
                                        group=group, place=place, seq_lens=ll)
        api.decode(q, part, out=outs[r], lse=lses[r])
    # the second sequence has no tokens in the last range: its lse is -inf there
    assert torch.isinf(lses[P - 1, 1]).all()
    merged = api.merge_states(outs, lses)
    torch.cuda.synchronize()
    assert (merged - full).abs().max().item() < 1e-5
    Kn, Vn = K.cpu().numpy(), V.cpu().numpy()
    _, _, kd = O.quantize(fmt, D, group, Kn.reshape(-1, D))
    _, _, vd = O.quantize(fmt, D, group, Vn.reshape(-1, D))
    ref = O.attention(q.cpu().numpy(), kd.reshape(Kn.shape), vd.reshape(Vn.shape), O.scale_f32(D), seq_lens=lens)
    assert_close(merged.cpu().numpy(), ref, "merged")
    assert api.device_errors() == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(dev, kind):
    g = torch.Generator(device=dev)
    g.manual_seed(51)
    if kind == "splitkv":
        B, H, Hkv, D, n = 1, 32, 8, 128, 5000
    else:
        B, H, Hkv, D, n = 4, 64, 8, 128, 1500
    q = torch.randn((B, H, D), generator=g, device=dev)
    K = torch.randn((B, Hkv, n, D), generator=g, device=dev)
    V = torch.randn((B, Hkv, n, D), generator=g, device=dev)
    return q, K, V


def _rank(rank, world, port, results):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        q, K, V = _inputs(dev, "splitkv")
        lens = np.array([4321], dtype=np.int32)
        a = {}
        for exchange in ("fused", "nvlink", "nccl"):
            sk = sharding.SplitKVDecode(q, K, V, fmt=FMT_INT4, group=32, place=Placement(ORD_HEAD, False, 0),
                                        seq_lens=lens, world=world, rank=rank, exchange=exchange)
            for _ in range(3):  # several steps: epochs and the two gather buffers alternate
                a[exchange] = sk.step().cpu().numpy()
            sk.close()
        q, K, V = _inputs(dev, "kvheads")
        hs = sharding.HeadShardedDecode(q, K, V, fmt=FMT_INT8, group=64, place=Placement(ORD_TOKEN, True, 16),
                                        seq_lens=None, world=world, rank=rank)
        b = hs.step(gather=True).cpu().numpy()
        torch.cuda.synchronize()
        results[rank] = (a, b, api.device_errors() | lib().kvf_b200_exchange_errors())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_nccl_ranks_match_one_gpu():
    import torch.multiprocessing as mp

    world = 2
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_rank, args=(world, _free_port(), results), nprocs=world, join=True)
        res = dict(results)
    dev = torch.device("cuda", 0)
    q, K, V = _inputs(dev, "splitkv")
    ref_a = api.decode(q, api.KVCache.from_logical(K, V, fmt=FMT_INT4, group=32, place=Placement(ORD_HEAD, False, 0),
                                                   seq_lens=np.array([4321], dtype=np.int32))).cpu().numpy()
    q, K, V = _inputs(dev, "kvheads")
    ref_b = api.decode(q, api.KVCache.from_logical(K, V, fmt=FMT_INT8, group=64,
                                                   place=Placement(ORD_TOKEN, True, 16))).cpu().numpy()
    # and the fp64 oracle over the oracle quantizer's dequantised K and V
    orc = {}
    for kind, fmt, group, lens in (("splitkv", FMT_INT4, 32, np.array([4321], dtype=np.int32)),
                                   ("kvheads", FMT_INT8, 64, None)):
        q, K, V = (t.cpu().numpy() for t in _inputs(dev, kind))
        D = q.shape[2]
        _, _, kd = O.quantize(fmt, D, group, K.reshape(-1, D))
        _, _, vd = O.quantize(fmt, D, group, V.reshape(-1, D))
        orc[kind] = O.attention(q, kd.reshape(K.shape), vd.reshape(V.shape), O.scale_f32(D), seq_lens=lens)
    assert_close(ref_a, orc["splitkv"], "one-GPU split-KV inputs")
    assert_close(ref_b, orc["kvheads"], "one-GPU KV-head inputs")
    for r in range(world):
        a, b, errs = res[r]
        assert errs == 0
        for exchange, got in a.items():
            assert np.abs(got - ref_a).max() < 1e-5, (r, exchange)
            assert_close(got, orc["splitkv"], f"rank {r} split-KV, {exchange} exchange")
        assert np.abs(b - ref_b).max() < 1e-6, r
        assert_close(b, orc["kvheads"], f"rank {r} KV heads")


@pytest.mark.gpu
def test_exchange_wait_runs_out_and_reports(cuda):
    """Failure detection without a fault: a two-rank exchange on one GPU
    whose other rank never exists. This rank's part goes into its own cells
    and into a stand-in buffer; the other rank's cells in its own buffer never
    carry the step's epoch, so every bounded wait (5 ms) runs out. The kernel
    returns, the output is zero, bit 1 of kvf_b200_device_errors() is set, and
    the next decode on the same context is correct."""
    import ctypes

    from kvforge_b200.sharding import KvfExchange

    rs = np.random.RandomState(41)
    B, H, Hkv, n, d, splits = 1, 8, 2, 512, 128, 4
    q = rs.standard_normal((B, H, d)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, d)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, d)).astype(np.float32)
    place = Placement(ORD_HEAD, False, 0)
    cache = api.KVCache.from_logical(torch.as_tensor(K, device=cuda), torch.as_tensor(V, device=cuda),
                                     fmt=FMT_INT8, group=64, place=place)
    qd = torch.as_tensor(q, device=cuda)
    out = torch.full((B, H, d), 7.0, device=cuda)
    ws = api.Workspace.allocate(B, H, d, splits, cuda, fused=False)
    a = api.make_args(qd, cache, out, ws)
    cells = 2 * 2 * B * H * (d + 1)
    own = torch.zeros(cells, dtype=torch.int64, device=cuda)
    stand_in = torch.zeros(cells, dtype=torch.int64, device=cuda)
    x = KvfExchange()
    x.P, x.rank, x.epoch, x.timeout_ms = 2, 0, 1, 5
    x.gather = own.data_ptr()
    x.peer_gather[0] = own.data_ptr()
    x.peer_gather[1] = stand_in.data_ptr()
    assert api.device_errors() == 0
    rc = lib().kvf_b200_decode_exchange(ctypes.byref(a), FMT_INT8, d, 1, ORD_HEAD, 0, ctypes.byref(x), None)
    assert rc == 0
    torch.cuda.synchronize()
    assert api.device_errors() & 2
    assert float(out.abs().max()) == 0.0
    # This rank's part reached both buffers, tagged with the epoch.
    assert int((stand_in >> 32).max()) == 1 and int((own >> 32).max()) == 1
    # The context is still usable.
    got = api.decode(qd, cache, splits=splits).cpu().numpy()
    _, _, kq = O.quantize(FMT_INT8, d, 64, K.reshape(-1, d))
    _, _, vq = O.quantize(FMT_INT8, d, 64, V.reshape(-1, d))
    ref = O.attention(q, kq.reshape(K.shape), vq.reshape(V.shape), O.scale_f32(d))
    assert np.abs(got - ref).max() < 2e-3
    assert api.device_errors() == 0
