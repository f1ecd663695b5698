"""ctypes wrappers over the test oracle. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; the product (kvforge_b200/) never does.

  C restatement  (oracle/kvf_oracle.c -> oracle/_build/libkvf_oracle.so):
      quantize, attention, row_of, rel_l2, f2h/h2f
  Reference's own functions (oracle/ref_shim.cu -> oracle/_ref/libkvf_ref.so,
  built only where the reference tree exists): Ref.quantize, Ref.attention, ...
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_double, c_float, c_int, c_int64, c_longlong, c_uint, c_ulonglong, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libkvf_oracle.so"
REF_SO = HERE / "_ref" / "libkvf_ref.so"

F16, INT8, INT4 = 0, 1, 2

_o = None
_r = None


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(c_void_p)


def lib():
    global _o
    if _o is None:
        if not ORACLE_SO.exists():
            from .build import build_oracle

            build_oracle()
        _o = ctypes.CDLL(os.fspath(ORACLE_SO))
        _o.kvfo_quantize.restype = c_int
        _o.kvfo_quantize.argtypes = [c_int, c_int, c_int, c_void_p, c_int64, c_void_p, c_void_p, c_void_p]
        _o.kvfo_attention.restype = c_int
        _o.kvfo_attention.argtypes = [c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                      c_void_p, c_float, c_void_p, c_int]
        _o.kvfo_row_of.restype = c_int64
        _o.kvfo_row_of.argtypes = [c_int, c_int, c_int, c_int, c_void_p, c_int, c_int, c_int, c_int]
        _o.kvfo_rel_l2.restype = c_double
        _o.kvfo_rel_l2.argtypes = [c_void_p, c_void_p, c_int64]
        _o.kvfo_f2h_array.argtypes = [c_void_p, c_void_p, c_int64]
        _o.kvfo_h2f_array.argtypes = [c_void_p, c_void_p, c_int64]
        _o.kvfo_max_threads.restype = c_int
    return _o


def row_bytes(fmt: int, d: int) -> int:
    return 2 * d if fmt == F16 else d if fmt == INT8 else d // 2


def f2h(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().kvfo_f2h_array(_ptr(x), _ptr(out), x.size)
    return out


def h2f(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().kvfo_h2f_array(_ptr(h), _ptr(out), h.size)
    return out


def quantize(fmt: int, d: int, group: int, X: np.ndarray):
    """(data uint8 [rows, row_bytes], meta uint32 [rows, d/group] or None, deq f32 [rows, d])."""
    X = np.ascontiguousarray(X, dtype=np.float32).reshape(-1, d)
    rows = X.shape[0]
    data = np.zeros((rows, row_bytes(fmt, d)), dtype=np.uint8)
    meta = np.zeros((rows, d // group), dtype=np.uint32) if fmt != F16 else None
    deq = np.empty_like(X)
    rc = lib().kvfo_quantize(fmt, d, group, _ptr(X), rows, _ptr(data),
                             _ptr(meta) if meta is not None else None, _ptr(deq))
    if rc != 0:
        raise ValueError("kvfo_quantize rejected its arguments")
    return data, meta, deq


def attention(q: np.ndarray, K: np.ndarray, V: np.ndarray, scale: float, seq_lens=None,
              threads: int = 0) -> np.ndarray:
    """fp64 attention (runtime/kvf_host.h:202-234). q [B,H,D]; K, V [B,Hkv,n,D]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    K = np.ascontiguousarray(K, dtype=np.float32)
    V = np.ascontiguousarray(V, dtype=np.float32)
    B, H, d = q.shape
    _, Hkv, n, _ = K.shape
    out = np.empty_like(q)
    sl = None if seq_lens is None else np.ascontiguousarray(seq_lens, dtype=np.int32)
    if threads <= 0:
        threads = max(1, min(os.cpu_count() or 1, lib().kvfo_max_threads()))
    rc = lib().kvfo_attention(B, H, Hkv, d, n, _ptr(sl) if sl is not None else None, _ptr(q), _ptr(K),
                              _ptr(V), c_float(scale), _ptr(out), threads)
    if rc != 0:
        raise ValueError("kvfo_attention rejected its arguments")
    return out


def row_of(order: int, bt: int, Hkv: int, n: int, table, max_blocks: int, b: int, h: int, t: int) -> int:
    tab = None if table is None else np.ascontiguousarray(table, dtype=np.int32)
    return int(lib().kvfo_row_of(order, bt, Hkv, n, _ptr(tab) if tab is not None else None,
                                 max_blocks, b, h, t))


def rel_l2(a: np.ndarray, ref: np.ndarray) -> float:
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    ref = np.ascontiguousarray(ref, dtype=np.float32).reshape(-1)
    return float(lib().kvfo_rel_l2(_ptr(a), _ptr(ref), a.size))


def attention_states(q: np.ndarray, K: np.ndarray, V: np.ndarray, scale: float, seq_lens=None):
    """(out, lse) in fp64 numpy for small cases: out as `attention`, lse[b][h]
    = log2 sum_t 2^(q.k_t * scale * log2 e) over the valid tokens (-inf when a
    sequence has none). The reference has no lse (it decodes on one GPU);
    this is the quantity kvf_args::lse carries so partial outputs over
    disjoint token ranges can be combined (see merge_states)."""
    q = np.asarray(q, dtype=np.float64)
    K = np.asarray(K, dtype=np.float64)
    V = np.asarray(V, dtype=np.float64)
    B, H, d = q.shape
    Hkv, n = K.shape[1], K.shape[2]
    g = H // Hkv
    out = np.zeros((B, H, d))
    lse = np.full((B, H), -np.inf)
    c = scale * np.log2(np.e)
    for b in range(B):
        nb = n if seq_lens is None else int(seq_lens[b])
        for h in range(H):
            if nb <= 0:
                continue
            s = K[b, h // g, :nb] @ q[b, h] * c
            m = s.max()
            w = np.exp2(s - m)
            out[b, h] = w @ V[b, h // g, :nb] / w.sum()
            lse[b, h] = m + np.log2(w.sum())
    return out.astype(np.float32), lse.astype(np.float32)


def merge_states(outs, lses):
    """Combination of per-part (out, lse) over disjoint token ranges, fp64:
    out = sum_p 2^(lse_p - LSE) out_p with LSE = log2 sum_p 2^lse_p; rows
    whose parts are all empty get zeros."""
    outs = np.asarray(outs, dtype=np.float64)
    lses = np.asarray(lses, dtype=np.float64)
    M = lses.max(axis=0)
    finite = np.isfinite(M)
    w = np.where(np.isfinite(lses), np.exp2(lses - np.where(finite, M, 0.0)), 0.0)
    W = w.sum(axis=0)
    out = (w[..., None] * outs).sum(axis=0) / np.where(W > 0, W, 1.0)[..., None]
    out[~(W > 0)] = 0.0
    return out.astype(np.float32)


def scale_f32(d: int) -> float:
    """1/sqrt(D) in fp32 (runtime/kvf_driver.cu:33)."""
    return float(np.float32(1.0) / np.sqrt(np.float32(d)))


class Ref:
    """The reference's own host functions (oracle/_ref/libkvf_ref.so)."""

    _lib = None

    @classmethod
    def available(cls) -> bool:
        return REF_SO.exists()

    @classmethod
    def lib(cls):
        if cls._lib is None:
            l = ctypes.CDLL(os.fspath(REF_SO))
            l.kvfr_quantize.restype = c_int
            l.kvfr_quantize.argtypes = [c_int, c_int, c_int, c_void_p, c_longlong, c_void_p, c_void_p, c_void_p]
            l.kvfr_attention.restype = c_int
            l.kvfr_attention.argtypes = [c_int] * 5 + [c_void_p, c_void_p, c_void_p, c_float, c_void_p]
            l.kvfr_row_of.restype = c_longlong
            l.kvfr_row_of.argtypes = [c_int, c_int, c_int, c_int, c_int, c_void_p, c_int, c_int, c_int, c_int]
            l.kvfr_rel_l2.restype = c_double
            l.kvfr_rel_l2.argtypes = [c_void_p, c_void_p, c_longlong]
            l.kvfr_scale_log2.restype = c_float
            l.kvfr_scale_log2.argtypes = [c_int]
            l.kvfr_make_data.argtypes = [c_int] * 5 + [c_ulonglong, c_void_p, c_void_p, c_void_p]
            cls._lib = l
        return cls._lib

    @classmethod
    def quantize(cls, fmt: int, d: int, group: int, X: np.ndarray):
        X = np.ascontiguousarray(X, dtype=np.float32).reshape(-1, d)
        rows = X.shape[0]
        data = np.zeros((rows, row_bytes(fmt, d)), dtype=np.uint8)
        meta = np.zeros((rows, d // group), dtype=np.uint32) if fmt != F16 else None
        deq = np.empty_like(X)
        cls.lib().kvfr_quantize(fmt, d, group, _ptr(X), rows, _ptr(data),
                                _ptr(meta) if meta is not None else None, _ptr(deq))
        return data, meta, deq

    @classmethod
    def attention(cls, q: np.ndarray, K: np.ndarray, V: np.ndarray, scale: float) -> np.ndarray:
        q = np.ascontiguousarray(q, dtype=np.float32)
        K = np.ascontiguousarray(K, dtype=np.float32)
        V = np.ascontiguousarray(V, dtype=np.float32)
        B, H, d = q.shape
        _, Hkv, n, _ = K.shape
        out = np.empty_like(q)
        cls.lib().kvfr_attention(B, H, Hkv, d, n, _ptr(q), _ptr(K), _ptr(V), c_float(scale), _ptr(out))
        return out

    @classmethod
    def row_of(cls, order, paged, bt, Hkv, n, table, max_blocks, b, h, t) -> int:
        tab = None if table is None else np.ascontiguousarray(table, dtype=np.int32)
        return int(cls.lib().kvfr_row_of(order, paged, bt, Hkv, n, _ptr(tab) if tab is not None else None,
                                         max_blocks, b, h, t))

    @classmethod
    def rel_l2(cls, a: np.ndarray, ref: np.ndarray) -> float:
        a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
        ref = np.ascontiguousarray(ref, dtype=np.float32).reshape(-1)
        return float(cls.lib().kvfr_rel_l2(_ptr(a), _ptr(ref), a.size))

    @classmethod
    def scale_log2(cls, d: int) -> float:
        return float(cls.lib().kvfr_scale_log2(d))
