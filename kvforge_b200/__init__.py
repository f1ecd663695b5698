"""kvforge_b200: B200-native (sm_100a) decode-attention kernels for KVForge.

The product is the C-ABI library built from kvforge_b200/csrc (declared in
include/kvforge_b200.h, with a C++ drop-in for the reference's kvf::launch<>
in include/kvf_kernels.cuh). This package is its host side: the ctypes
binding, cache placement, the device quantizer binding, and the benchmark
workloads. There is no CPU path: without the built library every call raises.
"""
from ._native import (FMT_F16, FMT_INT4, FMT_INT8, FMT_NAMES, ORD_HEAD, ORD_TOKEN, KvfArgs, KvfError,
                      LIB_PATH, lib)
from .layout import Placement

__version__ = "0.1.0"


def __getattr__(name):
    # torch-facing helpers are imported lazily so that `import kvforge_b200`
    # stays cheap for tools that only need the ABI.
    if name in ("api", "workloads"):
        import importlib

        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(name)


__all__ = ["FMT_F16", "FMT_INT8", "FMT_INT4", "FMT_NAMES", "ORD_HEAD", "ORD_TOKEN", "KvfArgs", "KvfError",
           "LIB_PATH", "lib", "Placement"]
