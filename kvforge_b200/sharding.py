"""Decode across GPUs, one process per GPU, for the two configurations that
shard.

split-KV (``Workload.shard == "splitkv"``): rank r of P owns the token range
``token_range(n, P, r)`` of every sequence and KV head, with its own local KV
cache. Each rank decodes its range with kvf_b200_decode, which also writes
the log2 softmax denominator of every query head (``kvf_args::lse``). Output
and lse live in one packed buffer per rank ([B*H*D] floats then [B*H]), so a
single NCCL all-gather moves every rank's state (B*H*(D+1)*4 bytes per rank,
16.5 KB at B=1, H=32) and the kvf_b200_merge_states kernel combines the P
states on every rank:
    out = sum_p 2^(lse_p - LSE) out_p,   LSE = log2 sum_p 2^lse_p.

KV-head sharding (``Workload.shard == "kvheads"``): rank r owns KV heads
``head_range(Hkv, P, r)`` of every sequence and their H/Hkv query heads each,
so attention needs no exchange at all; ``gather=True`` adds an all-gather of
the outputs into the replicated [B][H][D] tensor (rank-major, then reordered
into head order).

The reference decodes on one GPU; this module has no counterpart there. The
partitioning helpers are plain Python so the protocol is testable with gloo
ranks on the CPU.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import numpy as np
import torch

from . import api
from ._native import check, lib
from .layout import Placement


def token_range(n: int, world: int, rank: int, granule: int = 128) -> Tuple[int, int]:
    """Contiguous, granule-aligned slice [t0, t1) of n tokens for `rank`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank out of range")
    per = -(-n // world)
    per = -(-per // granule) * granule
    t0 = min(n, rank * per)
    return t0, min(n, t0 + per)


def head_range(Hkv: int, world: int, rank: int) -> Tuple[int, int]:
    """KV heads [h0, h1) of `rank`; Hkv must divide evenly."""
    if Hkv % world:
        raise ValueError(f"{Hkv} KV heads do not split evenly over {world} ranks")
    per = Hkv // world
    return rank * per, (rank + 1) * per


def local_seq_lens(seq_lens: Optional[np.ndarray], n: int, t0: int, t1: int) -> Optional[np.ndarray]:
    """Tokens of each sequence that fall in [t0, t1), or None when every
    sequence has all n tokens."""
    if seq_lens is None:
        return None
    return np.clip(np.asarray(seq_lens, dtype=np.int64) - t0, 0, t1 - t0).astype(np.int32)


def state_layout(B: int, H: int, d: int) -> Tuple[int, int]:
    """(lse offset, floats per rank) of the packed per-rank state buffer."""
    return B * H * d, B * H * d + B * H


def pack_state(out: torch.Tensor, lse: torch.Tensor, state: torch.Tensor) -> torch.Tensor:
    """Writes out [B][H][D] and lse [B][H] into one packed rank state."""
    n = out.numel()
    state[:n].copy_(out.reshape(-1))
    state[n:n + lse.numel()].copy_(lse.reshape(-1))
    return state


def unpack_states(gathered: torch.Tensor, B: int, H: int, d: int, world: int):
    """Views (outs [P][B][H][D], lses [P][B][H]) of gathered packed states."""
    lse_off, per = state_layout(B, H, d)
    g = gathered.view(world, per)
    return g[:, :lse_off].view(world, B, H, d), g[:, lse_off:].view(world, B, H)


def gather_states(state: torch.Tensor, gathered: torch.Tensor, group=None) -> torch.Tensor:
    """All-gathers every rank's packed state into `gathered` ([P * per],
    rank-major): one collective, NCCL on the GPUs, gloo on the CPU."""
    import torch.distributed as dist

    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, state, group=group)
    else:
        dist.all_gather(list(gathered.view(dist.get_world_size(group), -1).unbind(0)), state, group=group)
    return gathered


def head_order(B: int, H: int, world: int) -> torch.Tensor:
    """Index that turns rank-major gathered outputs [P][B][H/P] into [B][H]
    order (rank r holds query heads r*H/P .. (r+1)*H/P - 1)."""
    hp = H // world
    idx = torch.arange(world * B * hp).view(world, B, hp).permute(1, 0, 2).reshape(B, H)
    return idx


class SplitKVDecode:
    """One rank of a split-KV decode. Holds the local cache slice, the local
    workspace and the packed state buffers; ``step()`` is one decode step."""

    def __init__(self, q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, *, fmt: int, group: int,
                 place: Placement, seq_lens: Optional[np.ndarray], world: int, rank: int, group_pg=None,
                 splits: Optional[int] = None):
        import torch.distributed as dist

        self.dist = dist
        self.pg = group_pg
        self.world, self.rank = world, rank
        B, H, d = q.shape
        n = K.shape[2]
        self.t0, self.t1 = token_range(n, world, rank)
        lens = local_seq_lens(seq_lens, n, self.t0, self.t1)
        Kl = K[:, :, self.t0:self.t1].contiguous()
        Vl = V[:, :, self.t0:self.t1].contiguous()
        self.cache = api.KVCache.from_logical(Kl, Vl, fmt=fmt, group=group, place=place, seq_lens=lens)
        self.q = q
        self.B, self.H, self.d = B, H, d
        s = splits or api.suggest_splits(self.cache, H)
        self.ws = api.Workspace.allocate(B, H, d, s, q.device)
        lse_off, per = state_layout(B, H, d)
        self.lse_off, self.per = lse_off, per
        self.state = torch.empty(per, dtype=torch.float32, device=q.device)
        self.gathered = torch.empty(per * world, dtype=torch.float32, device=q.device)
        self.out = torch.empty((B, H, d), dtype=torch.float32, device=q.device)
        self.args = api.make_args(q, self.cache, self.state[:lse_off].view(B, H, d), self.ws)
        self.args.lse = self.state.data_ptr() + 4 * lse_off
        self.lib = lib()

    def payload_bytes(self) -> int:
        return self.cache.payload_bytes()

    def step(self, stream=None) -> torch.Tensor:
        st = torch.cuda.current_stream(self.q.device) if stream is None else stream
        sp = ctypes.c_void_p(st.cuda_stream)
        c = self.cache
        check("kvf_b200_decode", self.lib.kvf_b200_decode(ctypes.byref(self.args), c.fmt, self.d, 1, c.place.order,
                                                          int(c.place.paged), sp))
        gather_states(self.state, self.gathered, self.pg)
        base = self.gathered.data_ptr()
        check("kvf_b200_merge_states",
              self.lib.kvf_b200_merge_states(ctypes.c_void_p(base), ctypes.c_void_p(base + 4 * self.lse_off),
                                             self.world, self.B * self.H, self.d, self.per, self.per,
                                             ctypes.c_void_p(self.out.data_ptr()), None, sp))
        return self.out


class HeadShardedDecode:
    """One rank of a KV-head-sharded decode: KV heads [h0, h1) and their
    query heads. ``step(gather)`` decodes and optionally all-gathers the
    replicated output."""

    def __init__(self, q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, *, fmt: int, group: int,
                 place: Placement, seq_lens: Optional[np.ndarray], world: int, rank: int, group_pg=None,
                 splits: Optional[int] = None):
        import torch.distributed as dist

        self.dist = dist
        self.pg = group_pg
        self.world, self.rank = world, rank
        B, H, d = q.shape
        Hkv = K.shape[1]
        self.h0, self.h1 = head_range(Hkv, world, rank)
        gq = H // Hkv
        self.q = q[:, self.h0 * gq:self.h1 * gq].contiguous()
        self.cache = api.KVCache.from_logical(K[:, self.h0:self.h1].contiguous(), V[:, self.h0:self.h1].contiguous(),
                                              fmt=fmt, group=group, place=place, seq_lens=seq_lens)
        self.B, self.H, self.d = B, H, d
        Hl = self.q.shape[1]
        s = splits or api.suggest_splits(self.cache, Hl)
        self.ws = api.Workspace.allocate(B, Hl, d, s, q.device)
        self.out_local = torch.empty((B, Hl, d), dtype=torch.float32, device=q.device)
        self.gathered = torch.empty((world, B, Hl, d), dtype=torch.float32, device=q.device)
        self.order = head_order(B, H, world).to(q.device)
        self.args = api.make_args(self.q, self.cache, self.out_local, self.ws)
        self.lib = lib()

    def payload_bytes(self) -> int:
        return self.cache.payload_bytes()

    def step(self, gather: bool = False, stream=None) -> torch.Tensor:
        st = torch.cuda.current_stream(self.q.device) if stream is None else stream
        c = self.cache
        check("kvf_b200_decode", self.lib.kvf_b200_decode(ctypes.byref(self.args), c.fmt, self.d, 1, c.place.order,
                                                          int(c.place.paged), ctypes.c_void_p(st.cuda_stream)))
        if not gather:
            return self.out_local
        self.dist.all_gather_into_tensor(self.gathered, self.out_local, group=self.pg)
        return self.gathered.view(-1, self.d)[self.order.view(-1)].view(self.B, self.H, self.d)


__all__ = ["token_range", "head_range", "local_seq_lens", "state_layout", "pack_state", "unpack_states",
           "gather_states", "head_order", "SplitKVDecode", "HeadShardedDecode"]
