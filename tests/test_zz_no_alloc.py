"""kvf_b200_decode_noalloc: the decode entry point for callers that cannot
allocate device memory (an engine that reserved all of HBM for its KV pool,
a plugin whose framework owns every allocation). Its split partials live in a
static device array inside the library instead of a caller workspace.

Checked through the C ABI against kvf_b200_decode with a caller-provided
workspace (no split counters either, so both calls take the same launches and
only the partials' address differs: the outputs must be bit-identical), on
two calls in a row (different queries and split counts, so the second call
runs on the first call's leftovers in the shared array). At the size limit,
the largest split count whose partials fit is accepted and matches too, and
one more split is rejected with an error code before anything is launched. This
file is collected last so that a failure here stops a -x run only after every
other test has run; it also passes alone in a fresh process, where its first
call performs the per-device set-up.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from kvforge_b200 import FMT_INT8, ORD_TOKEN, api  # noqa: E402
from kvforge_b200._native import lib  # noqa: E402
from kvforge_b200.layout import Placement  # noqa: E402

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 8 << 20  # KVF_B200_NOALLOC_SCRATCH_BYTES


def _noalloc(q, cache, out, splits):
    # The workspace pointers stay null: the entry point must not need them.
    ws = api.Workspace(splits, None, None)
    a = api.make_args(q, cache, out, ws)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib().kvf_b200_decode_noalloc(ctypes.byref(a), cache.fmt, cache.d, 1, cache.place.order,
                                         int(cache.place.paged), stream)


def test_noalloc_matches_workspace_entry_point(cuda):
    rs = np.random.RandomState(21)
    B, H, Hkv, D, n = 3, 32, 8, 128, 3000
    K = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    V = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    cache = api.KVCache.from_logical(K, V, fmt=FMT_INT8, group=64, place=Placement(ORD_TOKEN, True, 16),
                                     seq_lens=np.array([3000, 1234, 17], dtype=np.int32))
    for call, splits in enumerate((24, 5)):
        q = torch.as_tensor(rs.standard_normal((B, H, D)).astype(np.float32), device=cuda)
        want = api.decode(q, cache, workspace=api.Workspace.allocate(B, H, D, splits, cuda, fused=False))
        got = torch.full_like(q, float("nan"))
        assert _noalloc(q, cache, got, splits) == 0, f"call {call}"
        torch.cuda.synchronize()
        assert torch.equal(got, want), (f"no-alloc call {call}, splits={splits}: max difference "
                                        f"{(got - want).abs().max().item():.3g}")
    assert api.device_errors() == 0


def _fits(B, H, D, splits):
    # part_ml (rounded up to 256 bytes) then part_o, as the entry point lays them out.
    heads = B * H * splits
    return (heads * 8 + 255) // 256 * 256 + heads * D * 4 <= SCRATCH_BYTES


def test_noalloc_at_and_beyond_the_scratch_limit(cuda):
    rs = np.random.RandomState(22)
    B, H, Hkv, D, n = 8, 64, 8, 128, 2048
    K = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    V = torch.as_tensor(rs.standard_normal((B, Hkv, n, D)).astype(np.float32), device=cuda)
    cache = api.KVCache.from_logical(K, V, fmt=FMT_INT8, group=64, place=Placement(ORD_TOKEN, False, 0))
    q = torch.as_tensor(rs.standard_normal((B, H, D)).astype(np.float32), device=cuda)
    largest = max(s for s in range(1, 64) if _fits(B, H, D, s))
    assert largest == 31 and not _fits(B, H, D, largest + 1)
    out = torch.full_like(q, float("nan"))
    assert _noalloc(q, cache, out, largest + 1) == 1  # cudaErrorInvalidValue, nothing launched
    assert torch.isnan(out).all()
    assert _noalloc(q, cache, out, largest) == 0
    want = api.decode(q, cache, workspace=api.Workspace.allocate(B, H, D, largest, cuda, fused=False))
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    assert api.device_errors() == 0
