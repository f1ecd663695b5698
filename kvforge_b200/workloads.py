"""The benchmark workloads and their seeded synthetic inputs.

Shapes are the five configurations the reference's headline metric is quoted
on (decode-attention us/step and effective KV TB/s). Inputs are synthetic:
seeded N(0,1) queries and keys/values generated on the device, with the
per-configuration variations (fp16-representable queries, outlier channels,
ragged sequence lengths, random page tables). There is no dataset.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from ._native import FMT_F16, FMT_INT4, FMT_INT8, ORD_HEAD, ORD_TOKEN
from .layout import Placement


@dataclass(frozen=True)
class Workload:
    name: str
    B: int
    H: int
    Hkv: int
    d: int
    n: int                      # tokens per sequence (the longest, when ragged)
    fmt: int
    group: int
    place: Placement
    ragged: Optional[tuple] = None   # (lo, hi): n_b ~ U[lo, hi], seeded
    lens: Optional[tuple] = None     # explicit tokens per sequence
    outlier_frac: float = 0.0        # fraction of (KV head, channel) pairs scaled x8
    q_fp16: bool = False             # queries rounded to fp16 values
    shard: str = "replicas"          # "replicas", "splitkv" or "kvheads" across GPUs
    seed: int = 1

    @property
    def fmt_name(self) -> str:
        return {FMT_F16: "f16", FMT_INT8: f"int8:{self.group}", FMT_INT4: f"int4:{self.group}"}[self.fmt]

    def seq_lens(self) -> Optional[np.ndarray]:
        if self.lens is not None:
            return np.asarray(self.lens, dtype=np.int32)
        if self.ragged is None:
            return None
        lo, hi = self.ragged
        rng = np.random.default_rng(self.seed + 1000)
        return rng.integers(lo, hi + 1, size=self.B).astype(np.int32)

    def config(self) -> dict:
        return {
            "workload": self.name, "B": self.B, "H": self.H, "Hkv": self.Hkv, "d": self.d,
            "n": (f"U[{self.ragged[0]},{self.ragged[1]}]" if self.ragged is not None
                  else "/".join(map(str, self.lens)) if self.lens is not None else self.n),
            "kv_format": self.fmt_name, "layout": self.place.name,
        }


CONFIGS = {
    w.name: w
    for w in [
        Workload("mha_b1_h32_n4096_f16_hm", 1, 32, 32, 128, 4096, FMT_F16, 0,
                 Placement(ORD_HEAD, False, 0), q_fp16=True),
        Workload("llama3_8b_gqa_b1_n32768_int8g64_tm", 1, 32, 8, 128, 32768, FMT_INT8, 64,
                 Placement(ORD_TOKEN, False, 0), outlier_frac=0.01),
        Workload("paged_gqa_b8_n2k_8k_f16_tm_p16", 8, 32, 8, 128, 8192, FMT_F16, 0,
                 Placement(ORD_TOKEN, True, 16), ragged=(2048, 8192)),
        Workload("long_gqa_b1_n65536_int4g32_hm", 1, 32, 8, 128, 65536, FMT_INT4, 32,
                 Placement(ORD_HEAD, False, 0), shard="splitkv"),
        Workload("llama3_70b_b64_n16384_int8g64_tm_p16", 64, 64, 8, 128, 16384, FMT_INT8, 64,
                 Placement(ORD_TOKEN, True, 16), shard="kvheads"),
    ]
}
CONFIG_ORDER = list(CONFIGS)
# The one-GPU benchmark line: the headline metric names no configuration, so
# it is quoted on the largest configuration that fits one GPU, the
# Llama-3-70B-shape serving batch (2.28 GB of payload per step). It is also
# the KV-head-sharded configuration, so the same line at N GPUs measures one
# problem split over them (strong scaling). The other four run with
# --workload NAME.
HEADLINE = "llama3_70b_b64_n16384_int8g64_tm_p16"

# Further shapes for parity tests and measurements (not benchmark configurations):
# one long sequence among short ones, where one split count for all sequences
# leaves most of the GPU idle.
EXTRA = {
    w.name: w
    for w in [
        Workload("skewed_gqa_b8_n32k_f16_tm_p16", 8, 32, 8, 128, 32768, FMT_F16, 0,
                 Placement(ORD_TOKEN, True, 16), lens=(32768,) + (1024,) * 7),
    ]
}
WORKLOADS = {**CONFIGS, **EXTRA}


def generate(w: Workload, device, seed: Optional[int] = None):
    """Seeded inputs for workload w: q [B,H,D], K and V [B,Hkv,n,D] (float32,
    logical order, on `device`) and seq_lens (np.int32 [B] or None)."""
    seed = w.seed if seed is None else seed
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    q = torch.randn((w.B, w.H, w.d), generator=g, device=device, dtype=torch.float32)
    if w.q_fp16:
        q = q.half().float()
    K = torch.randn((w.B, w.Hkv, w.n, w.d), generator=g, device=device, dtype=torch.float32)
    V = torch.randn((w.B, w.Hkv, w.n, w.d), generator=g, device=device, dtype=torch.float32)
    if w.outlier_frac > 0:
        count = max(1, int(round(w.outlier_frac * w.Hkv * w.d)))
        for X in (K, V):
            idx = torch.randperm(w.Hkv * w.d, generator=g, device=device)[:count]
            hs, cs = idx // w.d, idx % w.d
            X[:, hs, :, cs] *= 8.0
    return q, K, V, w.seq_lens()


__all__ = ["Workload", "CONFIGS", "CONFIG_ORDER", "HEADLINE", "EXTRA", "WORKLOADS", "generate"]
