"""Torch-facing host API over the C ABI.

`KVCache.from_logical` plays the role of the reference's quantize +
upload_cache (runtime/kvf_host.h:72-120, :149-195): quantize logical rows on
the device, then place them in the chosen layout. `decode` is one decode step
through kvf_b200_decode (the counterpart of kvf::launch<>,
runtime/kvf_kernels.cuh:309-320); `make_args` fills the argument block as
make_args does (runtime/kvf_host.h:273-293).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import layout
from ._native import FMT_F16, FMT_INT4, FMT_INT8, KvfArgs, check, lib
from .layout import Placement

LOG2E = 1.4426950408889634


def row_bytes(fmt: int, d: int) -> int:
    return 2 * d if fmt == FMT_F16 else d if fmt == FMT_INT8 else d // 2


def groups_per_row(fmt: int, d: int, group: int) -> int:
    return 0 if fmt == FMT_F16 else d // group


def scale_log2(d: int) -> float:
    """(1/sqrt(D)) * log2(e) in fp32, as make_args computes it (kvf_host.h:292)."""
    s = np.float32(1.0) / np.sqrt(np.float32(d))
    return float(np.float32(s) * np.float32(LOG2E))


def _stream(stream) -> ctypes.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def quantize(x: torch.Tensor, fmt: int, group: int = 0, stream=None):
    """Quantize rows of x (float32 [..., D], CUDA) on the device.

    Returns (data uint8 [rows, row_bytes], meta int32 [rows, D/group] or None).
    Bit-exact with kvf::quantize (runtime/kvf_host.h:72-120)."""
    if not x.is_cuda or x.dtype != torch.float32:
        raise ValueError("quantize expects a float32 CUDA tensor")
    d = x.shape[-1]
    x2 = x.reshape(-1, d).contiguous()
    rows = x2.shape[0]
    data = torch.empty((rows, row_bytes(fmt, d)), dtype=torch.uint8, device=x.device)
    gpr = groups_per_row(fmt, d, group)
    meta = torch.empty((rows, gpr), dtype=torch.int32, device=x.device) if gpr else None
    check(
        "kvf_b200_quantize",
        lib().kvf_b200_quantize(fmt, d, group, x2.data_ptr(), rows, data.data_ptr(),
                                meta.data_ptr() if meta is not None else None, _stream(stream)),
    )
    return data, meta


@dataclass
class KVCache:
    """A KV cache resident on one device, in one format and placement."""

    fmt: int
    d: int
    group: int
    place: Placement
    B: int
    Hkv: int
    n: int
    k: torch.Tensor                      # uint8 [rows_alloc, row_bytes]
    v: torch.Tensor
    k_meta: Optional[torch.Tensor]       # int32 [rows_alloc, D/group]
    v_meta: Optional[torch.Tensor]
    block_table: Optional[torch.Tensor]  # int32 [B, max_blocks]
    max_blocks: int
    seq_lens: Optional[torch.Tensor]     # int32 [B]

    @property
    def gpr(self) -> int:
        return groups_per_row(self.fmt, self.d, self.group)

    def payload_bytes(self) -> int:
        """KV payload of one decode step: 2 * valid rows * (row bytes + 4 * groups),
        the formula of runtime/kvf_driver.cu:51 over the stored tokens."""
        tokens = int(self.seq_lens.sum().item()) if self.seq_lens is not None else self.B * self.n
        rows = tokens * self.Hkv
        return 2 * rows * (row_bytes(self.fmt, self.d) + 4 * self.gpr)

    @classmethod
    def from_logical(cls, K: torch.Tensor, V: torch.Tensor, *, fmt: int, group: int = 0,
                     place: Placement, seq_lens=None, table_seed: int = 18) -> "KVCache":
        """Build a cache from logical float32 K, V [B][Hkv][n][D] on a CUDA device."""
        B, Hkv, n, d = K.shape
        dev = K.device
        kq, km = quantize(K, fmt, group)
        vq, vm = quantize(V, fmt, group)
        table = None
        max_blocks = 0
        pages = 0
        sl = None if seq_lens is None else np.asarray(seq_lens, dtype=np.int32)
        if place.paged:
            table, max_blocks, pages = layout.page_table(B, n, place.block_tokens, table_seed, sl)
        nrows = layout.rows_alloc(B, Hkv, n, place, pages)
        phys = layout.physical_rows(B, Hkv, n, place, table, sl)
        keep = np.nonzero(phys >= 0)[0]
        src = torch.from_numpy(keep).to(dev)
        dst = torch.from_numpy(phys[keep]).to(dev)

        def place_rows(x):
            if x is None:
                return None
            out = torch.zeros((nrows, x.shape[1]), dtype=x.dtype, device=dev)
            out.index_copy_(0, dst, x.index_select(0, src))
            return out

        cache = cls(
            fmt=fmt, d=d, group=group, place=place, B=B, Hkv=Hkv, n=n,
            k=place_rows(kq), v=place_rows(vq), k_meta=place_rows(km), v_meta=place_rows(vm),
            block_table=torch.from_numpy(table).to(dev) if table is not None else None,
            max_blocks=max_blocks,
            seq_lens=torch.from_numpy(sl).to(dev) if sl is not None else None,
        )
        return cache


@dataclass
class Workspace:
    """Split partials: part_o [B][H][splits][D] and part_ml [B][H][splits][2].

    ``split_sem`` (2 * B * H zeroed uint32 counters; the kernel uses two per
    (sequence, KV head), so any Hkv <= H fits) lets the tensor-core kernel merge the splits
    itself: the last block of a (sequence, KV head) merges and resets the
    counters. ``fused=False`` leaves it out: a separate merge kernel, as in
    the reference.
    """

    splits: int
    part_o: Optional[torch.Tensor]
    part_ml: Optional[torch.Tensor]
    split_sem: Optional[torch.Tensor] = None

    @classmethod
    def allocate(cls, B: int, H: int, d: int, splits: int, device, fused: bool = True) -> "Workspace":
        if splits <= 1:
            return cls(1, None, None)
        return cls(
            splits,
            torch.empty((B, H, splits, d), dtype=torch.float32, device=device),
            torch.empty((B, H, splits, 2), dtype=torch.float32, device=device),
            torch.zeros((2 * B * H,), dtype=torch.int32, device=device) if fused else None,
        )


def suggest_splits(cache: KVCache, H: int) -> int:
    """Split count for decoding this cache: the launcher's own choice, or for a
    cache with per-sequence lengths the capacity the balanced launch needs."""
    bt = cache.place.block_tokens if cache.place.paged else 0
    fn = lib().kvf_b200_suggest_splits_ragged if cache.seq_lens is not None else lib().kvf_b200_suggest_splits
    return int(fn(cache.B, H, cache.Hkv, cache.n, cache.fmt, cache.d, cache.group, int(cache.place.paged), bt))


def make_args(q: torch.Tensor, cache: KVCache, out: torch.Tensor, ws: Workspace) -> KvfArgs:
    B, H, d = q.shape
    a = KvfArgs()
    a.q = q.data_ptr()
    a.k = cache.k.data_ptr()
    a.v = cache.v.data_ptr()
    a.k_meta = cache.k_meta.data_ptr() if cache.k_meta is not None else None
    a.v_meta = cache.v_meta.data_ptr() if cache.v_meta is not None else None
    a.block_table = cache.block_table.data_ptr() if cache.block_table is not None else None
    a.out = out.data_ptr()
    a.part_o = ws.part_o.data_ptr() if ws.part_o is not None else None
    a.part_ml = ws.part_ml.data_ptr() if ws.part_ml is not None else None
    a.split_sem = ws.split_sem.data_ptr() if ws.split_sem is not None else None
    a.B, a.H, a.Hkv, a.n = B, H, cache.Hkv, cache.n
    a.splits = ws.splits
    a.warps = 4
    a.group_shift = int(round(math.log2(cache.group))) if cache.fmt != FMT_F16 else 0
    a.block_shift = int(round(math.log2(cache.place.block_tokens))) if cache.place.paged else 0
    a.max_blocks = cache.max_blocks
    a.scale_log2 = scale_log2(d)
    a.seq_lens = cache.seq_lens.data_ptr() if cache.seq_lens is not None else None
    return a


def append(cache: KVCache, k_new: torch.Tensor, v_new: torch.Tensor, pos: Optional[torch.Tensor] = None,
           stream=None) -> None:
    """Appends t_new tokens to every sequence of `cache` on its device
    (kvf_b200_append): k_new, v_new float32 [B][Hkv][t_new][D] are quantized
    exactly as quantize() does and written at the physical rows of tokens
    pos[b] .. pos[b] + t_new - 1. pos (int32 [B], on the cache's device)
    defaults to cache.seq_lens, which is then raised by t_new; a given pos
    leaves seq_lens alone. For a paged cache the block table must already map
    the blocks the new tokens fall in. Tokens at or past cache.n are skipped
    and reported by device_errors() (bit 2)."""
    if k_new.shape != v_new.shape or k_new.dim() != 4:
        raise ValueError("k_new and v_new must both be [B][Hkv][t_new][D]")
    B, Hkv, t_new, d = k_new.shape
    if (B, Hkv, d) != (cache.B, cache.Hkv, cache.d):
        raise ValueError(f"new rows {tuple(k_new.shape)} do not match the cache (B={cache.B}, Hkv={cache.Hkv}, "
                         f"D={cache.d})")
    if k_new.dtype != torch.float32 or v_new.dtype != torch.float32:
        raise ValueError("k_new and v_new must be float32")
    bump = pos is None
    if bump:
        if cache.seq_lens is None:
            raise ValueError("pos is required for a cache without seq_lens")
        pos = cache.seq_lens
    if pos.dtype != torch.int32 or pos.numel() != B or pos.device != cache.k.device:
        raise ValueError("pos must be an int32 tensor of B entries on the cache's device")
    k2, v2, pos = k_new.contiguous(), v_new.contiguous(), pos.contiguous()
    a = KvfArgs()
    a.k = cache.k.data_ptr()
    a.v = cache.v.data_ptr()
    a.k_meta = cache.k_meta.data_ptr() if cache.k_meta is not None else None
    a.v_meta = cache.v_meta.data_ptr() if cache.v_meta is not None else None
    a.block_table = cache.block_table.data_ptr() if cache.block_table is not None else None
    a.B, a.H, a.Hkv, a.n = B, Hkv, Hkv, cache.n
    a.group_shift = int(round(math.log2(cache.group))) if cache.fmt != FMT_F16 else 0
    a.block_shift = int(round(math.log2(cache.place.block_tokens))) if cache.place.paged else 0
    a.max_blocks = cache.max_blocks
    check("kvf_b200_append",
          lib().kvf_b200_append(ctypes.byref(a), cache.fmt, d, cache.place.order, int(cache.place.paged),
                                k2.data_ptr(), v2.data_ptr(), t_new, pos.data_ptr(), _stream(stream)))
    if bump:
        cache.seq_lens.add_(t_new)


PATHS = {"auto": 0, "mma": 1, "tc": 2}  # KVF_PATH_AUTO / KVF_PATH_MMA / KVF_PATH_TC
# Scheduling flags (KVF_FLAG_*), OR'ed into the path value: how the mma.sync
# launch merges its splits and whether it balances ragged batches; the output
# is the same whichever are set.
FLAG_MERGE_KERNEL, FLAG_GRID_MERGE, FLAG_NO_BALANCE = 0x100, 0x200, 0x400


def _path(path: str, flags: int = 0) -> int:
    if path not in PATHS:
        raise ValueError(f"path must be one of {sorted(PATHS)}")
    return PATHS[path] | int(flags)


def decode(q: torch.Tensor, cache: KVCache, *, out: Optional[torch.Tensor] = None,
           splits: Optional[int] = None, workspace: Optional[Workspace] = None, stream=None,
           g: int = 1, lse: Optional[torch.Tensor] = None, path: str = "auto", flags: int = 0) -> torch.Tensor:
    """One decode step: out[b][h] = softmax(q k^T * scale) v over the cache.

    q: float32 [B][H][D] on the cache's device. Returns out (float32 [B][H][D]).
    lse (optional float32 [B][H]) receives log2 of each head's softmax
    denominator, for combining outputs over disjoint token ranges with
    merge_states. path: "auto" (the launcher chooses), "mma" (mma.sync
    kernel) or "tc" (tcgen05 kernel; int8 rows of 128 only); flags: FLAG_*
    scheduling bits."""
    if q.dtype != torch.float32 or not q.is_contiguous():
        raise ValueError("q must be a contiguous float32 tensor [B][H][D]")
    B, H, d = q.shape
    if out is None:
        out = torch.empty_like(q)
    if workspace is None:
        s = splits if splits is not None else suggest_splits(cache, H)
        workspace = Workspace.allocate(B, H, d, s, q.device)
    a = make_args(q, cache, out, workspace)
    if lse is not None:
        if lse.dtype != torch.float32 or not lse.is_contiguous() or lse.numel() != B * H:
            raise ValueError("lse must be a contiguous float32 tensor [B][H]")
        a.lse = lse.data_ptr()
    check(
        "kvf_b200_decode_path",
        lib().kvf_b200_decode_path(ctypes.byref(a), cache.fmt, d, g, cache.place.order,
                                   int(cache.place.paged), _path(path, flags), _stream(stream)),
    )
    return out


class Decoder:
    """Repeated decode steps of a fixed batch over one cache, as a CUDA graph.

    One step takes the queries from a pinned host buffer (q_host), decodes
    (kernel plus split merge) and leaves the output in a pinned host buffer
    (out_host). The work is captured once and each step is a single graph
    replay. With zero_copy (the default) there is no copy-engine transfer at
    all: a small kernel reads the queries over PCIe while the decode kernel
    already streams K/V (kvf_b200_decode_from_host), and the kernels write
    the output straight into out_host; otherwise the step is an H2D copy, the
    decode and a D2H copy.

        dec = Decoder(cache, H)
        out = dec.step(q)          # q: host float32 [B][H][D]; or
        dec.q_host.copy_(q); dec.replay(); torch.cuda.current_stream().synchronize()

    The cache, batch, split count and kernel path are fixed at construction;
    the graph reads the cache in place, so its contents may change between
    steps.
    """

    def __init__(self, cache: KVCache, H: int, *, splits: Optional[int] = None, path: str = "auto",
                 g: int = 1, graph: bool = True, zero_copy: bool = True, flags: int = 0):
        dev = cache.k.device
        B, d = cache.B, cache.d
        self.cache = cache
        self.zero_copy = zero_copy
        self.splits = splits if splits is not None else suggest_splits(cache, H)
        self.q = torch.zeros((B, H, d), dtype=torch.float32, device=dev)
        self.out = torch.zeros((B, H, d), dtype=torch.float32, device=dev)
        self.q_host = torch.zeros((B, H, d), dtype=torch.float32).pin_memory()
        self.out_host = torch.zeros((B, H, d), dtype=torch.float32).pin_memory()
        self.workspace = Workspace.allocate(B, H, d, self.splits, dev)
        self._args = make_args(self.q, cache, self.out, self.workspace)
        if zero_copy:
            self._args.out = self.out_host.data_ptr()
        self._code = (cache.fmt, d, g, cache.place.order, int(cache.place.paged), _path(path, flags))
        self.graph = None
        if graph:
            # Warm up outside the capture (first launches set kernel attributes).
            self._issue(torch.cuda.current_stream(dev))
            torch.cuda.synchronize(dev)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._issue(torch.cuda.current_stream(dev))
            torch.cuda.synchronize(dev)

    def _issue(self, stream) -> None:
        fmt, d, g, order, paged, path = self._code
        sp = ctypes.c_void_p(stream.cuda_stream)
        if self.zero_copy:
            check("kvf_b200_decode_from_host",
                  lib().kvf_b200_decode_from_host(ctypes.byref(self._args), fmt, d, g, order, paged, path,
                                                  ctypes.c_void_p(self.q_host.data_ptr()), sp))
            return
        self.q.copy_(self.q_host, non_blocking=True)
        check("kvf_b200_decode_path",
              lib().kvf_b200_decode_path(ctypes.byref(self._args), fmt, d, g, order, paged, path, sp))
        self.out_host.copy_(self.out, non_blocking=True)

    def replay(self) -> None:
        """One step on the current stream, asynchronously: out_host is valid
        once the stream has reached this point."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._issue(torch.cuda.current_stream(self.q.device))

    def step(self, q: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One step, synchronously: q (host float32 [B][H][D]) if given is
        copied into q_host first; returns out_host."""
        if q is not None:
            self.q_host.copy_(q)
        self.replay()
        torch.cuda.current_stream(self.q.device).synchronize()
        return self.out_host


def merge_states(outs: torch.Tensor, lses: torch.Tensor, out: Optional[torch.Tensor] = None,
                 stream=None) -> torch.Tensor:
    """Combines P outputs of the same heads over disjoint token ranges:
    outs [P][..., D] and lses [P][...] (as from decode(..., lse=...)) ->
    [..., D], on the GPU (kvf_b200_merge_states)."""
    if outs.dtype != torch.float32 or lses.dtype != torch.float32:
        raise ValueError("float32 tensors expected")
    outs = outs.contiguous()
    lses = lses.contiguous()
    P, d = outs.shape[0], outs.shape[-1]
    rows = lses[0].numel()
    if outs[0].numel() != rows * d:
        raise ValueError("outs and lses disagree on the row count")
    if out is None:
        out = torch.empty(outs.shape[1:], dtype=torch.float32, device=outs.device)
    check("kvf_b200_merge_states",
          lib().kvf_b200_merge_states(ctypes.c_void_p(outs.data_ptr()), ctypes.c_void_p(lses.data_ptr()), P, rows,
                                      d, rows * d, rows, ctypes.c_void_p(out.data_ptr()), None, _stream(stream)))
    return out


def describe(q: torch.Tensor, cache: KVCache, workspace: Workspace, path: str = "auto", flags: int = 0) -> str:
    """One line describing the launch decode() would make (kernel, grid,
    stages, shared memory, splits), without launching."""
    B, H, d = q.shape
    a = make_args(q, cache, q, workspace)
    buf = ctypes.create_string_buffer(512)
    check("kvf_b200_describe_path",
          lib().kvf_b200_describe_path(ctypes.byref(a), cache.fmt, d, cache.place.order,
                                       int(cache.place.paged), _path(path, flags), buf, 512))
    return buf.value.decode()


def device_errors() -> int:
    return int(lib().kvf_b200_device_errors())


__all__ = ["KVCache", "Workspace", "Decoder", "decode", "PATHS", "FLAG_MERGE_KERNEL", "FLAG_GRID_MERGE",
           "FLAG_NO_BALANCE", "merge_states", "quantize", "append", "suggest_splits", "make_args", "describe",
           "device_errors", "row_bytes", "groups_per_row", "scale_log2", "FMT_F16", "FMT_INT8", "FMT_INT4"]
