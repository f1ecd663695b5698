"""kvf_b200_append on the GPU: new K/V tokens quantized (bit-exact with the
quantizer, kvf::quantize at runtime/kvf_host.h:72-120) and written at their
physical rows (runtime/kvf_kernels.cuh:51-64) of every placement; a decode
after the append equals a decode of a cache built with the tokens in place."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close
from oracle import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from kvforge_b200 import FMT_F16, FMT_INT4, FMT_INT8, ORD_HEAD, ORD_TOKEN, api  # noqa: E402
from kvforge_b200.layout import Placement  # noqa: E402

FORMATS = [(FMT_F16, 0), (FMT_INT8, 64), (FMT_INT4, 32), (FMT_INT8, 16)]
PLACES = [Placement(ORD_HEAD, False, 0), Placement(ORD_TOKEN, False, 0), Placement(ORD_HEAD, True, 16),
          Placement(ORD_TOKEN, True, 32)]


def _buffers(cache):
    return [t for t in (cache.k, cache.v, cache.k_meta, cache.v_meta) if t is not None]


@pytest.mark.parametrize("fmt,group", FORMATS)
@pytest.mark.parametrize("place", PLACES, ids=lambda p: p.name)
def test_append_writes_the_rows_a_full_build_holds(cuda, fmt, group, place):
    rs = np.random.RandomState(31)
    B, Hkv, n, d, t_new = 3, 4, 96, 128, 5
    pos = np.array([20, 91, 0], dtype=np.int32)  # the second sequence ends exactly at n
    K = rs.standard_normal((B, Hkv, n, d)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, d)).astype(np.float32)
    K2, V2 = K.copy(), V.copy()
    newk = np.stack([K[b, :, pos[b]:pos[b] + t_new] for b in range(B)])
    newv = np.stack([V[b, :, pos[b]:pos[b] + t_new] for b in range(B)])
    for b in range(B):  # other values where the new tokens go
        K2[b, :, pos[b]:pos[b] + t_new] = rs.standard_normal((Hkv, t_new, d)) * 7
        V2[b, :, pos[b]:pos[b] + t_new] = rs.standard_normal((Hkv, t_new, d)) * 7
    full = api.KVCache.from_logical(torch.as_tensor(K, device=cuda), torch.as_tensor(V, device=cuda), fmt=fmt,
                                    group=group, place=place)
    cache = api.KVCache.from_logical(torch.as_tensor(K2, device=cuda), torch.as_tensor(V2, device=cuda),
                                     fmt=fmt, group=group, place=place)
    api.append(cache, torch.as_tensor(newk, device=cuda), torch.as_tensor(newv, device=cuda),
               pos=torch.as_tensor(pos, device=cuda))
    assert api.device_errors() == 0
    for got, want in zip(_buffers(cache), _buffers(full)):
        assert torch.equal(got, want)


def test_append_skips_and_reports_tokens_past_the_end(cuda):
    rs = np.random.RandomState(32)
    B, Hkv, n, d, t_new = 2, 2, 64, 128, 4
    place = Placement(ORD_TOKEN, True, 16)
    K = rs.standard_normal((B, Hkv, n, d)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, d)).astype(np.float32)
    cache = api.KVCache.from_logical(torch.as_tensor(K, device=cuda), torch.as_tensor(V, device=cuda),
                                     fmt=FMT_INT8, group=64, place=place)
    before = [t.clone() for t in _buffers(cache)]
    newk = rs.standard_normal((B, Hkv, t_new, d)).astype(np.float32)
    pos = np.array([62, 10], dtype=np.int32)  # tokens 64, 65 of sequence 0 do not exist
    api.append(cache, torch.as_tensor(newk, device=cuda), torch.as_tensor(newk, device=cuda),
               pos=torch.as_tensor(pos, device=cuda))
    assert api.device_errors() & 4
    assert api.device_errors() == 0  # read and cleared
    # Exactly the in-range rows changed: tokens 62, 63 of sequence 0 and 10..13 of sequence 1.
    K3 = K.copy()
    K3[0, :, 62:64] = newk[0, :, :2]
    K3[1, :, 10:14] = newk[1]
    want = api.KVCache.from_logical(torch.as_tensor(K3, device=cuda), torch.as_tensor(V, device=cuda),
                                    fmt=FMT_INT8, group=64, place=place)
    assert torch.equal(cache.k, want.k) and torch.equal(cache.k_meta, want.k_meta)
    assert not torch.equal(cache.k, before[0])


@pytest.mark.parametrize("fmt,group", [(FMT_INT8, 64), (FMT_F16, 0)])
def test_decode_after_appending_steps(cuda, fmt, group):
    """Three decode steps, each appending one token per sequence at its
    length (pos defaults to seq_lens, which the append raises), decode after
    each against the oracle over the tokens stored so far."""
    rs = np.random.RandomState(33)
    B, H, Hkv, n, d = 2, 16, 4, 512, 128
    lens = np.array([300, 77], dtype=np.int32)
    K = rs.standard_normal((B, Hkv, n, d)).astype(np.float32)
    V = rs.standard_normal((B, Hkv, n, d)).astype(np.float32)
    place = Placement(ORD_TOKEN, False, 0)
    cache = api.KVCache.from_logical(torch.as_tensor(K, device=cuda), torch.as_tensor(V, device=cuda), fmt=fmt,
                                     group=group, place=place, seq_lens=lens)
    _, _, kq = O.quantize(fmt, d, group, K.reshape(-1, d))
    _, _, vq = O.quantize(fmt, d, group, V.reshape(-1, d))
    kq, vq = kq.reshape(K.shape), vq.reshape(V.shape)
    for step in range(3):
        new = np.stack([K[b, :, lens[b] + step:lens[b] + step + 1] for b in range(B)])
        newv = np.stack([V[b, :, lens[b] + step:lens[b] + step + 1] for b in range(B)])
        api.append(cache, torch.as_tensor(new, device=cuda), torch.as_tensor(newv, device=cuda))
        now = lens + step + 1
        assert np.array_equal(cache.seq_lens.cpu().numpy(), now)
        q = rs.standard_normal((B, H, d)).astype(np.float32)
        got = api.decode(torch.as_tensor(q, device=cuda), cache, splits=4).cpu().numpy()
        ref = O.attention(q, kq, vq, O.scale_f32(d), seq_lens=now)
        assert_close(got, ref, f"append step {step}")
    assert api.device_errors() == 0
