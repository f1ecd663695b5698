"""Multi-GPU host logic on the CPU: two gloo ranks run the split-KV and the
KV-head-sharded protocols of kvforge_b200.sharding end to end (partition,
packed state, one all-gather, combination / reordering), with the fp64
oracle standing in for each rank's GPU decode, and must reproduce the
single-device result. The GPU kernels of the same protocol are covered in
test_multigpu.py."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from kvforge_b200 import sharding  # noqa: E402
from oracle import oracle as O  # noqa: E402


def test_partitions_cover_exactly():
    for n, P in [(65536, 8), (1000, 3), (129, 2), (0, 4), (100, 8)]:
        ranges = [sharding.token_range(n, P, r) for r in range(P)]
        assert ranges[0][0] == 0 and ranges[-1][1] == n
        for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
            assert a1 == b0 and a0 <= a1
        assert all(t0 % 128 == 0 for t0, _ in ranges if t0 < n)
    assert [sharding.head_range(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        sharding.head_range(8, 3, 0)
    lens = np.array([0, 100, 300, 1000])
    assert sharding.local_seq_lens(lens, 1000, 256, 512).tolist() == [0, 0, 44, 256]
    order = sharding.head_order(2, 8, 2)
    # rank 1's first head of sequence 0 is query head 4
    assert order[0, 4].item() == 1 * 2 * 4 + 0 * 4 + 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rs = np.random.RandomState(31)
    B, H, Hkv, D, n = 2, 8, 4, 64, 700
    q = rs.standard_normal((B, H, D)).astype(np.float32)
    K = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, D)).astype(np.float32)
    lens = np.array([700, 250], dtype=np.int32)
    return q, K, V, lens


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, K, V, lens = _inputs()
        B, H, D = q.shape
        Hkv, n = K.shape[1], K.shape[2]
        scale = O.scale_f32(D)
        # ---- split-KV: this rank's tokens, packed state, one gather, combine
        t0, t1 = sharding.token_range(n, world, rank)
        ll = sharding.local_seq_lens(lens, n, t0, t1)
        out_r, lse_r = O.attention_states(q, K[:, :, t0:t1], V[:, :, t0:t1], scale, seq_lens=ll)
        _, per = sharding.state_layout(B, H, D)
        state = torch.empty(per)
        sharding.pack_state(torch.from_numpy(out_r), torch.from_numpy(lse_r), state)
        gathered = torch.empty(per * world)
        sharding.gather_states(state, gathered)
        outs, lses = sharding.unpack_states(gathered, B, H, D, world)
        split_out = O.merge_states(outs.numpy(), lses.numpy())
        # ---- KV-head sharding: this rank's heads, gather, reorder
        h0, h1 = sharding.head_range(Hkv, world, rank)
        g = H // Hkv
        loc = O.attention(q[:, h0 * g:h1 * g], K[:, h0:h1], V[:, h0:h1], scale, seq_lens=lens)
        parts = [torch.empty_like(torch.from_numpy(loc)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(loc))
        flat = torch.stack(parts).reshape(-1, D)
        head_out = flat[sharding.head_order(B, H, world).reshape(-1)].reshape(B, H, D).numpy()
        results[rank] = (split_out, head_out)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reproduce_the_single_device_result():
    world = 2
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        res = dict(results)
    q, K, V, lens = _inputs()
    full = O.attention(q, K, V, O.scale_f32(q.shape[2]), seq_lens=lens)
    for rank in range(world):
        split_out, head_out = res[rank]
        assert np.abs(split_out - full).max() < 1e-5, rank
        assert np.abs(head_out - full).max() < 1e-6, rank
