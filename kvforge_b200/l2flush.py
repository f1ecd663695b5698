"""Cold-L2 preparation before a timed decode step (bench.py, the sweep).

A write of a buffer larger than L2 evicts the step's inputs, but leaves the
L2 full of dirty lines; the step that follows then pays for writing them
back to HBM while it streams its own inputs (measured on B200: +2 us on the
22 us step of mha_b1_h32_n4096_f16_hm, +4 us on the 52 us step of
paged_gqa_b8_n2k_8k_f16_tm_p16). A read of a second buffer larger
than L2 after the write replaces the dirty lines with clean ones, so the
timed step starts from a cold L2 that owes HBM nothing, as a decode step
after the model's other kernels (weights read, small activations written)
does.
"""
from __future__ import annotations

import torch

DESCRIPTION = ("flushed before every step: a write of 3 x L2, then a read of 3 x L2 from a second buffer "
               "(cold L2 without dirty lines)")


class L2Flush:
    def __init__(self, device):
        l2 = torch.cuda.get_device_properties(device).L2_cache_size
        size = max(96 << 20, 3 * l2)
        self.dirty = torch.empty(size, dtype=torch.uint8, device=device)
        rows = max(1, (size // 4) >> 16)
        self.clean = torch.ones((rows, 1 << 16), dtype=torch.float32, device=device)
        self.sink = torch.empty(rows, dtype=torch.float32, device=device)

    def __call__(self, i: int, clean: bool = True) -> None:
        """clean=False: the write alone, as the reference flushes."""
        self.dirty.fill_(i & 0xFF)
        if clean:
            torch.sum(self.clean, dim=1, out=self.sink)


__all__ = ["L2Flush", "DESCRIPTION"]
