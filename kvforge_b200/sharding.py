"""Decode across GPUs, one process per GPU, for the two configurations that
shard.

split-KV (``Workload.shard == "splitkv"``): rank r of P owns the token range
``token_range(n, P, r)`` of every sequence and KV head, with its own local KV
cache. Each rank decodes its range with kvf_b200_decode, which also writes
the log2 softmax denominator of every query head (``kvf_args::lse``). Output
and lse live in one packed buffer per rank ([B*H*D] floats then [B*H]:
B*H*(D+1)*4 bytes, 16.5 KB at B=1, H=32), and every rank combines the P
states:
    out = sum_p 2^(lse_p - LSE) out_p,   LSE = log2 sum_p 2^lse_p.
By default the exchange is fused into the decode's split merge
(``FusedExchange``, kvf_b200_decode_exchange): the merge kernel stores each
32-column slice of this rank's result straight into every rank's gather
buffer over NVLink (buffers mapped through CUDA IPC), each value in a 64-bit
cell with the step's epoch, waits (bounded) until every part of the slice
carries the epoch and writes the combination, so a step is the same two
launches as on one GPU. Alternatives kept for comparison: a separate push and
wait-and-merge pair of kernels (``PeerExchange``), or one NCCL all-gather
plus kvf_b200_merge_states.

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


class PeerExchange:
    """Gather and flag buffers of one rank, shared with the other ranks of the
    node through CUDA IPC (plain peer mappings). Two gather buffers alternate
    by step parity; step e writes `e` into the flags."""

    def __init__(self, per: int, world: int, rank: int, group=None):
        import torch.distributed as dist

        if world > 8:
            raise ValueError("the peer exchange supports at most 8 ranks")
        L = lib()
        self.L, self.per, self.world, self.rank = L, per, world, rank
        self.gbase, self.fbase = ctypes.c_void_p(), ctypes.c_void_p()
        hg, hf = (ctypes.c_char * 64)(), (ctypes.c_char * 64)()
        check("kvf_b200_ipc_alloc", L.kvf_b200_ipc_alloc(2 * world * per * 4, ctypes.byref(self.gbase), hg))
        check("kvf_b200_ipc_alloc", L.kvf_b200_ipc_alloc(256, ctypes.byref(self.fbase), hf))
        handles = [None] * world
        dist.all_gather_object(handles, (bytes(hg), bytes(hf)), group=group)
        self.opened = []
        gpeer, fpeer = [], []
        for q, (h1, h2) in enumerate(handles):
            if q == rank:
                gpeer.append(self.gbase.value)
                fpeer.append(self.fbase.value)
                continue
            pg, pf = ctypes.c_void_p(), ctypes.c_void_p()
            check("kvf_b200_ipc_open", L.kvf_b200_ipc_open(ctypes.create_string_buffer(h1, 64), ctypes.byref(pg)))
            check("kvf_b200_ipc_open", L.kvf_b200_ipc_open(ctypes.create_string_buffer(h2, 64), ctypes.byref(pf)))
            self.opened += [pg, pf]
            gpeer.append(pg.value)
            fpeer.append(pf.value)
        P = ctypes.c_void_p * world
        self._arrays = [P(*[gpeer[q] + ((par * world + rank) * per) * 4 for q in range(world)]) for par in (0, 1)]
        self._arrays.append(P(*[fpeer[q] + rank * 4 for q in range(world)]))
        self.slots = [ctypes.cast(self._arrays[par], ctypes.c_void_p) for par in (0, 1)]
        self.flags = ctypes.cast(self._arrays[2], ctypes.c_void_p)
        self.epoch = 0
        dist.barrier(group=group)

    def exchange_merge(self, state: torch.Tensor, rows: int, d: int, lse_off: int, out: torch.Tensor,
                       stream, timeout_ms: int = 1000) -> None:
        self.epoch += 1
        e = self.epoch
        sp = ctypes.c_void_p(stream.cuda_stream)
        check("kvf_b200_push_state", self.L.kvf_b200_push_state(ctypes.c_void_p(state.data_ptr()), self.per,
                                                                self.slots[e & 1], self.flags, self.world, e, sp))
        gathered = self.gbase.value + (e & 1) * self.world * self.per * 4
        check("kvf_b200_wait_merge_states",
              self.L.kvf_b200_wait_merge_states(ctypes.c_void_p(gathered), self.fbase, self.world, e, rows, d,
                                                self.per, lse_off, ctypes.c_void_p(out.data_ptr()), None,
                                                timeout_ms, sp))

    def close(self, group=None) -> None:
        """Collective: every rank unmaps its peers' buffers, then frees its own."""
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier(group=group)
        for ptr in self.opened:
            self.L.kvf_b200_ipc_close(ptr)
        self.opened = []
        dist.barrier(group=group)
        for ptr in (self.gbase, self.fbase):
            if ptr.value:
                self.L.kvf_b200_ipc_free(ptr)
        self.gbase, self.fbase = ctypes.c_void_p(), ctypes.c_void_p()


class KvfExchange(ctypes.Structure):
    """Mirror of kvf_exchange (kvforge_b200.h)."""

    _fields_ = [("P", ctypes.c_int), ("rank", ctypes.c_int), ("epoch", ctypes.c_int), ("timeout_ms", ctypes.c_uint),
                ("gather", ctypes.c_void_p), ("peer_gather", ctypes.c_void_p * 8)]


def _share(L, sizes, world: int, rank: int, group):
    """Allocates zeroed IPC-shareable buffers of `sizes` bytes, exchanges the
    handles and maps every peer's buffers: (own pointers, per-rank pointer
    lists, opened mappings to close)."""
    import torch.distributed as dist

    own, handles = [], []
    for n in sizes:
        p, h = ctypes.c_void_p(), (ctypes.c_char * 64)()
        check("kvf_b200_ipc_alloc", L.kvf_b200_ipc_alloc(n, ctypes.byref(p), h))
        own.append(p)
        handles.append(bytes(h))
    everyone = [None] * world
    dist.all_gather_object(everyone, handles, group=group)
    peers = [[None] * world for _ in sizes]
    opened = []
    for q in range(world):
        for k in range(len(sizes)):
            if q == rank:
                peers[k][q] = own[k].value
                continue
            ptr = ctypes.c_void_p()
            check("kvf_b200_ipc_open", L.kvf_b200_ipc_open(ctypes.create_string_buffer(everyone[q][k], 64),
                                                           ctypes.byref(ptr)))
            opened.append(ptr)
            peers[k][q] = ptr.value
    return own, peers, opened


def _unshare(L, own, opened, group):
    import torch.distributed as dist

    torch.cuda.synchronize()
    dist.barrier(group=group)
    for ptr in opened:
        L.kvf_b200_ipc_close(ptr)
    dist.barrier(group=group)
    for ptr in own:
        if ptr.value:
            L.kvf_b200_ipc_free(ptr)


class FusedExchange:
    """Buffer of the exchange fused into the split merge: gather cells
    [2][P][rows][d+1] x 64 bits (value, epoch), on every rank, mapped on every
    other rank through CUDA IPC."""

    def __init__(self, rows: int, d: int, world: int, rank: int, group=None, timeout_ms: int = 1000):
        import torch.distributed as dist

        if world > 8:
            raise ValueError("the fused exchange supports at most 8 ranks")
        self.L, self.group = lib(), group
        self.own, peers, self.opened = _share(self.L, [2 * world * rows * (d + 1) * 8], world, rank, group)
        x = KvfExchange()
        x.P, x.rank, x.epoch, x.timeout_ms = world, rank, 0, timeout_ms
        x.gather = self.own[0].value
        for q in range(world):
            x.peer_gather[q] = peers[0][q]
        self.x = x
        dist.barrier(group=group)

    def next_epoch(self) -> "KvfExchange":
        self.x.epoch += 1
        return self.x

    def close(self) -> None:
        _unshare(self.L, self.own, self.opened, self.group)
        self.own, self.opened = [], []


class SplitKVDecode:
    """One rank of a split-KV decode. Holds the local cache slice, the local
    workspace and the packed state buffers; ``step()`` is one decode step."""

    def __init__(self, q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, *, fmt: int, group: int,
                 place: Placement, seq_lens: Optional[np.ndarray], world: int, rank: int, group_pg=None,
                 splits: Optional[int] = None, exchange: str = "fused"):
        import torch.distributed as dist

        if exchange not in ("fused", "nvlink", "nccl"):
            raise ValueError("exchange must be 'fused', 'nvlink' or 'nccl'")
        self.dist = dist
        self.pg = group_pg
        self.world, self.rank = world, rank
        self.exchange = exchange
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
        if exchange == "fused":
            s = max(2, s)  # the exchange runs in the split merge
        self.ws = api.Workspace.allocate(B, H, d, s, q.device)
        lse_off, per = state_layout(B, H, d)
        self.lse_off, self.per = lse_off, per
        self.state = torch.empty(per, dtype=torch.float32, device=q.device)
        self.gathered = torch.empty(per * world, dtype=torch.float32, device=q.device)
        self.out = torch.empty((B, H, d), dtype=torch.float32, device=q.device)
        self.args = api.make_args(q, self.cache, self.state[:lse_off].view(B, H, d), self.ws)
        self.args.lse = self.state.data_ptr() + 4 * lse_off
        self.lib = lib()
        self.peers = PeerExchange(per, world, rank, group_pg) if exchange == "nvlink" else None
        self.fused = None
        if exchange == "fused":
            self.fused = FusedExchange(B * H, d, world, rank, group_pg)
            self.args = api.make_args(q, self.cache, self.out, self.ws)

    def payload_bytes(self) -> int:
        return self.cache.payload_bytes()

    def close(self) -> None:
        if self.peers is not None:
            self.peers.close(self.pg)
            self.peers = None
        if self.fused is not None:
            self.fused.close()
            self.fused = None

    def step(self, stream=None) -> torch.Tensor:
        st = torch.cuda.current_stream(self.q.device) if stream is None else stream
        sp = ctypes.c_void_p(st.cuda_stream)
        c = self.cache
        if self.fused is not None:
            x = self.fused.next_epoch()
            check("kvf_b200_decode_exchange",
                  self.lib.kvf_b200_decode_exchange(ctypes.byref(self.args), c.fmt, self.d, 1, c.place.order,
                                                    int(c.place.paged), ctypes.byref(x), sp))
            return self.out
        check("kvf_b200_decode", self.lib.kvf_b200_decode(ctypes.byref(self.args), c.fmt, self.d, 1, c.place.order,
                                                          int(c.place.paged), sp))
        if self.peers is not None:
            self.peers.exchange_merge(self.state, self.B * self.H, self.d, self.lse_off, self.out, st)
            return self.out
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
           "gather_states", "head_order", "PeerExchange", "FusedExchange", "SplitKVDecode", "HeadShardedDecode"]
