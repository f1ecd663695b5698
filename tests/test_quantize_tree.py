"""The device quantizer combines a group's min and max across lanes
(quantize.cu, quantize_rows); the host quantizer folds them in one loop from
the first element (runtime/kvf_host.h:91-95: std::min / std::max, i.e.
lo = v < lo ? v : lo and hi = hi < v ? v : hi). This restates the lane
scheme in numpy float32 (4 channels per lane, +inf/-inf start on lanes
without the first element, an xor tree that combines the earlier range
first) and checks that it gives the loop's bits for groups of 4..128
channels with NaN, +-inf and +-0 mixed in. The GPU tests check the kernel's
bytes against the reference quantizer."""
from __future__ import annotations

import numpy as np

f32 = np.float32


def loop_minmax(g):
    lo = hi = g[0]
    for v in g[1:]:
        lo = v if v < lo else lo
        hi = v if hi < v else hi
    return lo, hi


def lane_minmax(g):
    lpg = len(g) // 4
    lo, hi = [], []
    for li in range(lpg):
        e = g[4 * li: 4 * li + 4]
        first = li == 0
        l_ = e[0] if first else f32(np.inf)
        h_ = e[0] if first else f32(-np.inf)
        for k in range(1 if first else 0, 4):
            l_ = e[k] if e[k] < l_ else l_
            h_ = e[k] if h_ < e[k] else h_
        lo.append(l_)
        hi.append(h_)
    off = 1
    while off < lpg:
        nlo, nhi = list(lo), list(hi)
        for li in range(lpg):
            p = li ^ off
            a, b = (li, p) if (li & off) == 0 else (p, li)   # a: the earlier range
            nlo[li] = lo[b] if lo[b] < lo[a] else lo[a]
            nhi[li] = hi[b] if hi[a] < hi[b] else hi[a]
        lo, hi = nlo, nhi
        off <<= 1
    return lo[0], hi[0]


def test_lane_tree_matches_the_host_loop_bit_for_bit():
    rs = np.random.RandomState(0)
    specials = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1.0, -1.0, 65504, -65504, 1e6], dtype=f32)
    for _ in range(4000):
        G = int(rs.choice([4, 8, 16, 32, 64, 128]))
        g = rs.standard_normal(G).astype(f32)
        m = rs.rand(G) < rs.choice([0.0, 0.1, 0.5, 1.0])
        g[m] = rs.choice(specials, int(m.sum()))
        want = np.array(loop_minmax(g), dtype=f32).view(np.uint32)
        got = np.array(lane_minmax(g), dtype=f32).view(np.uint32)
        assert np.array_equal(want, got), g
