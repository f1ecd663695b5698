"""kvf_b200_decode_noalloc: the decode entry point for callers that cannot
allocate device memory (an engine that reserved all of HBM for its KV pool,
a plugin whose framework owns every allocation). Its split partials live in a
static device array inside the library instead of a caller workspace.

Checked through the C ABI against kvf_b200_decode with a caller-provided
workspace, on two calls in a row (different queries and split counts, so the
second call runs on the first call's leftovers in the shared array), and the
size limit is rejected with an error code before anything is launched. This
file is collected last so that a failure here stops a -x run only after every
other test has run; it also passes alone in a fresh process, where its first
call performs the per-device set-up.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import assert_close

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
        want = api.decode(q, cache, workspace=api.Workspace.allocate(B, H, D, splits, cuda))
        got = torch.full_like(q, float("nan"))
        assert _noalloc(q, cache, got, splits) == 0, f"call {call}"
        torch.cuda.synchronize()
        assert_close(got.cpu().numpy(), want.cpu().numpy(), f"no-alloc call {call}, splits={splits}")
    assert api.device_errors() == 0


def test_noalloc_rejects_partials_beyond_the_scratch(cuda):
    rs = np.random.RandomState(22)
    B, H, Hkv, D, n = 8, 64, 8, 128, 2048
    K = torch.as_tensor(rs.standard_normal((1, Hkv, n, D)).astype(np.float32), device=cuda).expand(B, -1, -1, -1)
    cache = api.KVCache.from_logical(K.contiguous(), K.contiguous(), fmt=FMT_INT8, group=64,
                                     place=Placement(ORD_TOKEN, False, 0))
    q = torch.zeros((B, H, D), dtype=torch.float32, device=cuda)
    out = torch.zeros_like(q)
    splits = SCRATCH_BYTES // (B * H * (D + 2) * 4) + 1
    assert _noalloc(q, cache, out, splits) == 1  # cudaErrorInvalidValue, nothing launched
    ok_splits = splits - 2
    assert _noalloc(q, cache, out, ok_splits) == 0
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
