"""Writes the per-variant resource table of the sm_100a kernels in the
format of the reference's machines/resources_*.csv (fmt,d,g,u,ord,paged,final,
regs,smem), which src/machine.cpp loads through the machine file's
`resources =` key. Registers come from the compiled kernels
(cudaFuncGetAttributes), shared memory from the launch plan; run on the GPU
box:

    python -m kvforge_b200.machines.make_resources > kvforge_b200/machines/resources_sm100.csv
"""
from __future__ import annotations

import ctypes
import re
import sys

from kvforge_b200._native import KvfArgs, lib

FMTS = {"f16": 0, "int8": 1, "int4": 2}


def main() -> int:
    L = lib()
    print("fmt,d,g,u,ord,paged,final,regs,smem")
    buf = ctypes.create_string_buffer(512)
    for i in range(L.kvf_b200_variant_count()):
        name = L.kvf_b200_variant_name(i).decode()
        m = re.fullmatch(r"(f16|int8|int4)_(hm|tm)_(c|p)_g(\d)_u(\d)_d(\d+)", name)
        if not m:
            continue
        fmt, ordn, res, g, u, d = FMTS[m[1]], int(m[2] == "tm"), int(m[3] == "p"), int(m[4]), int(m[5]), int(m[6])
        for final in (0, 1):
            a = KvfArgs()
            a.q = a.k = a.v = a.out = a.part_o = a.part_ml = 1 << 20  # never dereferenced: describe only plans
            a.k_meta = a.v_meta = 1 << 20
            a.block_table = 1 << 20
            a.B, a.Hkv, a.n = 1, 8, 4096
            a.H = a.Hkv * g
            a.splits = 1 if final else 8
            a.group_shift = 6 if fmt == 1 else 5
            a.block_shift = 4
            a.max_blocks = 256
            rc = L.kvf_b200_describe(ctypes.byref(a), fmt, d, ordn, res, buf, 512)
            if rc != 0:
                continue
            desc = buf.value.decode()
            regs = re.search(r"regs=(\d+)", desc)[1]
            smem = re.search(r"smem=(\d+)", desc)[1]
            print(f"{fmt},{d},{g},{u},{ordn},{res},{final},{regs},{smem}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
