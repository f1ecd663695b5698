"""ctypes binding of the C ABI in include/kvforge_b200.h.

The library is built in-tree (kvforge_b200/_lib/libkvforge_b200.so, see
kvforge_b200/build.py). There is no fallback: if the library is missing or
fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_char_p, c_float, c_int, c_longlong, c_uint, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libkvforge_b200.so"

FMT_F16, FMT_INT8, FMT_INT4 = 0, 1, 2
ORD_HEAD, ORD_TOKEN = 0, 1
FMT_NAMES = {"f16": FMT_F16, "int8": FMT_INT8, "int4": FMT_INT4}


class KvfArgs(ctypes.Structure):
    """Mirror of kvf_args / kvf::Args (runtime/kvf_kernels.cuh:29-46) plus the
    appended seq_lens, split_sem and lse fields."""

    _fields_ = [
        ("q", c_void_p),
        ("k", c_void_p),
        ("v", c_void_p),
        ("k_meta", c_void_p),
        ("v_meta", c_void_p),
        ("block_table", c_void_p),
        ("out", c_void_p),
        ("part_o", c_void_p),
        ("part_ml", c_void_p),
        ("B", c_int),
        ("H", c_int),
        ("Hkv", c_int),
        ("n", c_int),
        ("splits", c_int),
        ("warps", c_int),
        ("group_shift", c_int),
        ("block_shift", c_int),
        ("max_blocks", c_int),
        ("scale_log2", c_float),
        ("seq_lens", c_void_p),
        ("split_sem", c_void_p),
        ("lse", c_void_p),
    ]


class KvfError(RuntimeError):
    """A kvforge_b200 entry point returned a CUDA error code."""

    def __init__(self, fn: str, code: int):
        self.code = code
        super().__init__(f"{fn} failed with cudaError {code} ({CUDA_ERRORS.get(code, 'unknown')})")


CUDA_ERRORS = {
    0: "cudaSuccess",
    1: "cudaErrorInvalidValue",
    2: "cudaErrorMemoryAllocation",
    98: "cudaErrorInvalidDeviceFunction",
    209: "cudaErrorNoKernelImageForDevice",
    716: "cudaErrorMisalignedAddress",
    801: "cudaErrorNotSupported",
}

_lib = None

# (name, restype, argtypes) of every exported entry point.
SIGNATURES = [
    ("kvf_b200_decode", c_int, [ctypes.POINTER(KvfArgs), c_int, c_int, c_int, c_int, c_int, c_void_p]),
    ("kvf_b200_decode_path", c_int, [ctypes.POINTER(KvfArgs), c_int, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    ("kvf_b200_decode_from_host", c_int,
     [ctypes.POINTER(KvfArgs), c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    ("kvf_b200_merge", c_int, [ctypes.POINTER(KvfArgs), c_int, c_void_p]),
    ("kvf_b200_merge_states", c_int, [c_void_p, c_void_p, c_int, c_int, c_int, ctypes.c_longlong,
                                       ctypes.c_longlong, c_void_p, c_void_p, c_void_p]),
    ("kvf_b200_decode_exchange", c_int, [ctypes.POINTER(KvfArgs), c_int, c_int, c_int, c_int, c_int, c_void_p,
                                         c_void_p]),
    ("kvf_b200_push_state", c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    ("kvf_b200_wait_merge_states", c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, ctypes.c_longlong,
                                            ctypes.c_longlong, c_void_p, c_void_p, c_uint, c_void_p]),
    ("kvf_b200_exchange_errors", c_uint, []),
    ("kvf_b200_ipc_alloc", c_int, [ctypes.c_size_t, ctypes.POINTER(c_void_p), c_void_p]),
    ("kvf_b200_ipc_open", c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    ("kvf_b200_ipc_close", c_int, [c_void_p]),
    ("kvf_b200_ipc_free", c_int, [c_void_p]),
    ("kvf_b200_decode_noalloc", c_int, [ctypes.POINTER(KvfArgs), c_int, c_int, c_int, c_int, c_int, c_void_p]),
    ("kvf_b200_launch_variant", c_int, [c_char_p, ctypes.POINTER(KvfArgs), c_void_p]),
    ("kvf_b200_variant_count", c_int, []),
    ("kvf_b200_variant_name", c_char_p, [c_int]),
    ("kvf_b200_suggest_splits", c_int, [c_int] * 9),
    ("kvf_b200_suggest_splits_ragged", c_int, [c_int] * 9),
    ("kvf_b200_balanced_chunk", c_int, [c_void_p] + [c_int] * 6),
    ("kvf_b200_describe", c_int, [ctypes.POINTER(KvfArgs), c_int, c_int, c_int, c_int, c_char_p, c_int]),
    ("kvf_b200_describe_path", c_int, [ctypes.POINTER(KvfArgs), c_int, c_int, c_int, c_int, c_int, c_char_p, c_int]),
    ("kvf_b200_device_errors", c_uint, []),
    ("kvf_b200_quantize", c_int, [c_int, c_int, c_int, c_void_p, c_longlong, c_void_p, c_void_p, c_void_p]),
    ("kvf_b200_append", c_int, [ctypes.POINTER(KvfArgs), c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int,
                                 c_void_p, c_void_p]),
    ("kvf_b200_version", c_char_p, []),
]


def lib() -> ctypes.CDLL:
    """The loaded C-ABI library. Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m kvforge_b200.build` "
                "(the sm_100a kernels have no fallback)"
            )
        l = ctypes.CDLL(os.fspath(LIB_PATH))
        for name, res, args in SIGNATURES:
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def check(fn: str, code: int) -> None:
    if code != 0:
        raise KvfError(fn, code)
