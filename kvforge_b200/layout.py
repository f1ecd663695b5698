"""Cache placement on the host side of the boundary.

Mirrors the reference's placement helpers in runtime/kvf_host.h: `row_of`
follows host_row_of (:124-135) and `page_table` the block-table construction
of upload_cache (:149-165): a seeded permutation of the physical pages, so
pages are not in order. Rows are one token's D channels of one KV head; the
quantization metadata of a row sits at the same physical row index
(:179-182).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from ._native import ORD_HEAD, ORD_TOKEN


@dataclass(frozen=True)
class Placement:
    order: int          # ORD_HEAD or ORD_TOKEN
    paged: bool
    block_tokens: int   # tokens per page when paged, else 0

    @property
    def name(self) -> str:
        o = "head_major" if self.order == ORD_HEAD else "token_major"
        return f"{o}/paged:{self.block_tokens}" if self.paged else f"{o}/contiguous"


def page_table(B: int, n: int, bt: int, seed: int, seq_lens=None) -> tuple[np.ndarray, int, int]:
    """Block table [B][max_blocks] and the number of physical pages.

    Without seq_lens every sequence owns ceil(n/bt) pages (upload_cache,
    kvf_host.h:157-165). With seq_lens a sequence owns ceil(n_b/bt) pages and the
    unused table entries are 0. The pages are a seeded random permutation."""
    max_blocks = (n + bt - 1) // bt
    if seq_lens is None:
        need = np.full(B, max_blocks, dtype=np.int64)
    else:
        need = (np.asarray(seq_lens, dtype=np.int64) + bt - 1) // bt
    pages = int(need.sum())
    perm = np.random.default_rng(seed).permutation(pages).astype(np.int32)
    table = np.zeros((B, max(max_blocks, 1)), dtype=np.int32)
    off = 0
    for b in range(B):
        table[b, : need[b]] = perm[off : off + need[b]]
        off += int(need[b])
    return table, max_blocks, pages


def rows_alloc(B: int, Hkv: int, n: int, place: Placement, pages: int = 0) -> int:
    return pages * Hkv * place.block_tokens if place.paged else B * Hkv * n


def physical_rows(B: int, Hkv: int, n: int, place: Placement, table=None, seq_lens=None) -> np.ndarray:
    """Physical row of every logical row (b*Hkv + h)*n + t, as an int64 array;
    -1 for tokens past a sequence's length (they are not stored)."""
    b = np.arange(B, dtype=np.int64)[:, None, None]
    h = np.arange(Hkv, dtype=np.int64)[None, :, None]
    t = np.arange(n, dtype=np.int64)[None, None, :]
    if not place.paged:
        if place.order == ORD_HEAD:
            rows = (b * Hkv + h) * n + t
        else:
            rows = (b * n + t) * Hkv + h
    else:
        bt = place.block_tokens
        tab = np.asarray(table, dtype=np.int64)
        page = tab[b, t // bt]
        base = page * Hkv * bt
        tl = t % bt
        rows = base + (h * bt + tl if place.order == ORD_HEAD else tl * Hkv + h)
    rows = np.broadcast_to(rows, (B, Hkv, n)).copy()
    if seq_lens is not None:
        valid = t < np.asarray(seq_lens, dtype=np.int64)[:, None, None]
        rows = np.where(np.broadcast_to(valid, rows.shape), rows, -1)
    return rows.reshape(-1)


def row_of(order: int, bt: int, Hkv: int, n: int, table, max_blocks: int, b: int, h: int, t: int) -> int:
    """Physical row of (b, h, t) (kvf_host.h:124-135); bt = 0 means contiguous."""
    if bt == 0:
        return (b * Hkv + h) * n + t if order == ORD_HEAD else (b * n + t) * Hkv + h
    blk, tl = divmod(t, bt)
    page = int(np.asarray(table).reshape(-1)[b * max_blocks + blk])
    base = page * Hkv * bt
    return base + h * bt + tl if order == ORD_HEAD else base + tl * Hkv + h


__all__ = ["Placement", "page_table", "rows_alloc", "physical_rows", "row_of", "ORD_HEAD", "ORD_TOKEN"]
