"""Token-balanced splits for batches of unequal sequences, without a GPU.

The kernels pick the chunk on the device from seq_lens; kvf_b200_balanced_chunk
is the same search on the host. These tests check the plan's properties over
seeded random batches: the chunk is a multiple of the granularity, no
sequence needs more splits than the workspace holds, the work items fit in
the launched grid, the chunk is the smallest with those properties, and the
items (sequence by sequence, head group fastest, as the kernel numbers its
blocks) cover every token of every head group exactly once.
"""
from __future__ import annotations

import ctypes

import numpy as np

from kvforge_b200._native import lib


def chunk_of(lens: np.ndarray, n: int, splits: int, units: int, grid: int, gran: int) -> int:
    arr = np.ascontiguousarray(lens, dtype=np.int32)
    return int(lib().kvf_b200_balanced_chunk(arr.ctypes.data_as(ctypes.c_void_p), len(arr), n, splits, units,
                                             grid, gran))


def items(lens: np.ndarray, c: int) -> np.ndarray:
    """Splits per sequence under chunk c."""
    return (np.clip(lens, 0, None).astype(np.int64) + c - 1) // c


def test_balanced_chunk_properties():
    rs = np.random.RandomState(5)
    for _ in range(400):
        B = int(rs.randint(1, 40))
        n = int(rs.choice([1, 15, 100, 700, 2048, 8192, 65536]))
        gran = int(rs.choice([16, 32, 64, 128]))
        units = int(rs.choice([1, 2, 4, 8]))
        grid = units * B + int(rs.randint(0, 600))
        splits = int(rs.randint(1, 300))
        lens = rs.randint(0, n + 1, size=B).astype(np.int32)
        if rs.rand() < 0.2:
            lens[rs.randint(B)] = n
        c = chunk_of(lens, n, splits, units, grid, gran)
        sb = items(np.minimum(lens, n), c)
        assert c > 0 and c % gran == 0
        assert sb.max(initial=0) <= splits, (c, splits)
        assert units * sb.sum() <= grid
        # The smallest such chunk: one granule less breaks a constraint.
        cp = c - gran
        if cp >= gran and cp * splits >= n:
            assert units * items(np.minimum(lens, n), cp).sum() > grid

        # Block x: head group x % units, item x // units; items in order of
        # sequence, then split.
        covered = np.zeros((B, units, n), dtype=np.int32)
        starts = np.concatenate([[0], np.cumsum(sb)])
        for x in range(grid):
            u, j = x % units, x // units
            if j >= starts[-1]:
                continue
            b = int(np.searchsorted(starts, j, side="right") - 1)
            s = j - starts[b]
            t0, t1 = s * c, min(int(lens[b]), s * c + c)
            assert t0 < t1
            covered[b, u, t0:t1] += 1
        for b in range(B):
            assert np.all(covered[b, :, : lens[b]] == 1)
            assert np.all(covered[b, :, lens[b]:] == 0)


def test_uniform_batch_gets_the_wave_filling_chunk():
    """All sequences of length n: the balanced chunk is the one that fills one
    wave, i.e. the same split count the uniform plan would use."""
    lens = np.full(8, 8192, dtype=np.int32)
    c = chunk_of(lens, 8192, 148, 2, 296, 16)
    assert c == 464 and 2 * 8 * -(-8192 // c) <= 296
    assert 2 * 8 * -(-8192 // (c - 16)) > 296


def test_balanced_chunk_rejects_bad_arguments():
    lens = np.array([10, 20], dtype=np.int32)
    assert chunk_of(lens, 20, 4, 2, 3, 16) == -1   # 2 units x 2 sequences > 3 blocks
    assert chunk_of(lens, 20, 0, 1, 8, 16) == -1
    assert chunk_of(lens, 20, 4, 1, 8, 0) == -1
    assert lib().kvf_b200_balanced_chunk(None, 2, 20, 4, 1, 8, 16) == -1


def test_ragged_split_suggestion():
    """For a ragged batch on the mma.sync path the suggestion is a capacity at
    least the uniform one; where the tensor-core kernel runs, or the batch
    has more units than one wave, it is the uniform one."""
    l = lib()
    uni = l.kvf_b200_suggest_splits(8, 32, 8, 8192, 0, 128, 0, 1, 16)
    rag = l.kvf_b200_suggest_splits_ragged(8, 32, 8, 8192, 0, 128, 0, 1, 16)
    assert rag >= uni >= 1 and rag <= 8192 // 16
    for args in [(64, 64, 8, 16384, 1, 128, 64, 1, 16), (400, 8, 4, 512, 0, 128, 0, 0, 0)]:
        assert l.kvf_b200_suggest_splits_ragged(*args) == l.kvf_b200_suggest_splits(*args), args


def test_cost_model_follows_balanced_launches():
    """The planner's model of a balanced launch: one wave, blocks of at least
    tokens / (blocks per head group) tokens, partials of the used splits
    only; unchanged for the tensor-core path and for launches that did not
    balance (sweep rows taken before launches balanced)."""
    from kvforge_b200 import costmodel

    s = costmodel.Shape(8, 32, 8, 128, 32768, 0, 0, True, 16, 32768 + 7 * 1024)
    bal = costmodel.features(s, 148, "mma", balanced=True)
    uni = costmodel.features(s, 148, "mma", balanced=False)
    assert bal[2] == 17          # 272-token chunks, 16-token stages, one wave
    assert uni[2] == 8 * 14      # 224-token chunks, 2368 blocks in 8 waves
    assert bal[4] < uni[4]
    assert np.array_equal(costmodel.features(s, 4, "tc", balanced=True), costmodel.features(s, 4, "tc"))
    assert costmodel._balanced({"balanced": "1"}) and not costmodel._balanced({})
