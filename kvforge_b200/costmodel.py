"""B200 cost model of one decode step, calibrated from sweeps.

Counterpart of the reference's analytic cost model and its calibration
(src/cost.cpp, src/calib.cpp, model/*.cal): predicts the device time of one
decode step (decode kernel plus split merge, as bench.py times it) for a shape,
a split count and a kernel path, so that the planner (codegen.plan) can pick
the fastest plan. The reference models its SIMT kernel from first principles
and fits a handful of efficiency constants; the sm_100a kernels are modelled
by the quantities that set their time on B200, one linear model per kernel
path:

    t_us = c_fixed                       launch, ring fill and drain, event floor
         + c_byte  * payload_MB          streaming the K/V rows and metadata
         + c_stage * waves * stages      the per-block serial stage chain
         + c_split * [splits > 1]        the split merge's launch and tail
         + c_part  * partials_MB         the merge's reads of the partials

where waves = ceil(blocks / (148 SMs x 2 blocks per SM)) and stages is the
number of ring stages one block streams. The coefficients are fitted with
non-negative least squares to a sweep (kvforge_b200.sweep) and stored as
``path.key = value`` lines in machines/b200-sxm.cal, the same key = value format
as the reference's model/constants_*.cal.
"""
from __future__ import annotations

import dataclasses
import math
from pathlib import Path
from typing import Dict, Iterable, List, Optional, Sequence

import numpy as np

SMS = 148
BLOCKS_PER_SM = 2
KEYS = ("c_fixed", "c_byte", "c_stage", "c_split", "c_part")
DEFAULT_CAL = Path(__file__).resolve().parent / "machines" / "b200-sxm.cal"

# Used until a calibration exists: from single measurements of the five
# benchmark workloads (config 2: 71 MB, 147 splits, one wave of 7 stages ->
# ~26 us; config 5: 2.1 GB on the tcgen05 kernel -> ~740 us).
DEFAULTS: Dict[str, Dict[str, float]] = {
    "mma": {"c_fixed": 8.0, "c_byte": 0.16, "c_stage": 1.3, "c_split": 3.0, "c_part": 0.5},
    "tc": {"c_fixed": 10.0, "c_byte": 0.2, "c_stage": 2.9, "c_split": 1.0, "c_part": 0.5},
}


@dataclasses.dataclass(frozen=True)
class Shape:
    B: int
    H: int
    Hkv: int
    d: int
    n: int              # longest sequence
    fmt: int            # 0 f16, 1 int8, 2 int4
    group: int          # quantization group (ignored for f16)
    paged: bool = False
    block_tokens: int = 0
    tokens: Optional[int] = None  # sum of sequence lengths, when ragged (default B * n)

    def row_bytes(self) -> int:
        return {0: 2 * self.d, 1: self.d, 2: self.d // 2}[self.fmt]

    def meta_bytes(self) -> int:
        return 0 if self.fmt == 0 else 4 * (self.d // self.group)

    def payload_bytes(self) -> int:
        """2 (K and V) x valid rows x (row + metadata) bytes: the algorithmic
        bytes of one step (bench.py's payload)."""
        toks = self.tokens if self.tokens is not None else self.B * self.n
        return 2 * toks * self.Hkv * (self.row_bytes() + self.meta_bytes())


def heads_per_block(Hkv: int, path: str) -> int:
    """KV heads one block serves: 1 on tcgen05; 4, 2 or 1 on mma.sync
    (decode.cu heads_per_block)."""
    if path == "tc":
        return 1
    for h in (4, 2):
        if Hkv % h == 0:
            return h
    return 1


def tokens_per_stage(s: Shape, path: str) -> int:
    if path == "tc":
        return 128
    rb = s.row_bytes()
    return 16 * (1 if rb >= 256 else 2 if rb >= 128 else 4)


def features(s: Shape, splits: int, path: str, balanced: bool = False) -> np.ndarray:
    """[1, payload MB, waves x stages per block, splits > 1, partials MB].

    balanced: the launch shared the tokens of unequal sequences out over one
    wave of blocks (mma.sync with seq_lens, decode.cu plan_mma); the chunk is
    then at least tokens / (blocks per head group), the kernels' own rule
    without the per-sequence rounding."""
    hh = heads_per_block(s.Hkv, path)
    units = s.B * (s.Hkv // hh)
    tb = tokens_per_stage(s, path)
    gran = max(tb, s.block_tokens) if s.paged else tb
    up = lambda x: max(gran, math.ceil(x / gran) * gran)  # noqa: E731
    slots = SMS * BLOCKS_PER_SM
    if balanced and path == "mma" and splits > 1 and units <= slots:
        toks = s.tokens if s.tokens is not None else s.B * s.n
        per_group = min(slots, units * splits) // (s.Hkv // hh)
        chunk = up(max(math.ceil(s.n / splits), math.ceil(toks / per_group)))
        stages = math.ceil(min(chunk, s.n) / tb)
        waves = 1
        partial_mb = s.H * math.ceil(toks / chunk + s.B / 2) * (s.d + 2) * 4 / 1e6
    else:
        chunk = up(math.ceil(s.n / max(1, splits)))
        stages = math.ceil(min(chunk, s.n) / tb)
        waves = math.ceil(units * splits / slots)
        partial_mb = s.B * s.H * splits * (s.d + 2) * 4 / 1e6 if splits > 1 else 0.0
    return np.array([1.0, s.payload_bytes() / 1e6, float(waves * stages), 1.0 if splits > 1 else 0.0, partial_mb])


def split_candidates(B: int, Hkv: int, n: int, path: str) -> List[int]:
    """Split counts worth predicting: wave-filling counts and powers of two,
    up to one stage per split."""
    hh = heads_per_block(Hkv, path)
    units = B * (Hkv // hh)
    tb = 128 if path == "tc" else 32
    top = max(1, math.ceil(n / tb))
    cands = {1}
    for k in (1, 2, 3, 4):
        cands.add(max(1, (k * SMS * BLOCKS_PER_SM) // max(1, units)))
    p = 1
    while p <= top:
        cands.add(p)
        p *= 2
    return sorted(c for c in cands if 1 <= c <= top)


@dataclasses.dataclass
class CostModel:
    coef: Dict[str, Dict[str, float]]
    source: str = "defaults"

    @classmethod
    def load(cls, path: Optional[Path] = None) -> "CostModel":
        """Coefficients from a .cal file (machines/b200-sxm.cal by default);
        the built-in defaults for keys it does not set."""
        coef = {p: dict(v) for p, v in DEFAULTS.items()}
        path = Path(path) if path is not None else DEFAULT_CAL
        if not path.exists():
            return cls(coef, "defaults")
        for line in path.read_text().splitlines():
            line = line.split("#", 1)[0].strip()
            if not line or "=" not in line:
                continue
            key, val = (x.strip() for x in line.split("=", 1))
            if "." not in key:
                continue
            p, k = key.split(".", 1)
            if p in coef and k in KEYS:
                coef[p][k] = float(val)
        return cls(coef, str(path))

    def predict_us(self, s: Shape, splits: int, path: str, balanced: bool = False) -> float:
        c = self.coef[path]
        return float(np.dot(features(s, splits, path, balanced), [c[k] for k in KEYS]))

    def save(self, path: Path, header: Sequence[str] = ()) -> None:
        lines = ["# kvforge_b200 cost-model constants (B200, sm_100a), fitted by kvforge_b200.sweep."]
        lines += [f"# {h}" for h in header]
        for p in sorted(self.coef):
            for k in KEYS:
                lines.append(f"{p}.{k} = {self.coef[p][k]:.6g}")
        Path(path).write_text("\n".join(lines) + "\n")


def fit(rows: Iterable[dict]) -> CostModel:
    """Non-negative least squares per kernel path over sweep rows (dicts with
    the Shape fields, 'splits', 'path' and 'us'). Paths without rows keep the
    defaults. Relative residuals are minimised (each row weighted by 1/us) so
    short and long steps count alike."""
    from scipy.optimize import nnls

    by_path: Dict[str, list] = {}
    for r in rows:
        by_path.setdefault(r["path"], []).append(r)
    coef = {p: dict(v) for p, v in DEFAULTS.items()}
    for p, rs in by_path.items():
        A = np.stack([features(_shape(r), int(r["splits"]), p, _balanced(r)) for r in rs])
        y = np.array([float(r["us"]) for r in rs])
        w = 1.0 / y
        x, _ = nnls(A * w[:, None], y * w)
        coef[p] = dict(zip(KEYS, map(float, x)))
    return CostModel(coef, "fit")


def _shape(r: dict) -> Shape:
    return Shape(int(r["B"]), int(r["H"]), int(r["Hkv"]), int(r["d"]), int(r["n"]), int(r["fmt"]),
                 int(r["group"]), bool(int(r["paged"])), int(r["block_tokens"]),
                 int(r["tokens"]) if r.get("tokens") not in (None, "", "None") else None)


def _balanced(r: dict) -> bool:
    """Rows of sweeps taken before launches balanced have no such column."""
    return str(r.get("balanced") or "0") not in ("0", "False", "")


def relative_errors(model: CostModel, rows: Iterable[dict]) -> np.ndarray:
    return np.array([model.predict_us(_shape(r), int(r["splits"]), r["path"], _balanced(r)) / float(r["us"]) - 1.0
                     for r in rows])


__all__ = ["Shape", "CostModel", "features", "fit", "split_candidates", "relative_errors", "DEFAULT_CAL"]
