"""ctypes wrapper of oracle/libattn_oracle.so -- TEST INFRASTRUCTURE ONLY.

The C file (oracle/attn_oracle.c) restates the reference's host attention
(tuning/utils.cuh:139-198) in the same floating-point order; its outputs are
pinned bit for bit to the reference's own verify_attn output in tests/golden.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.  The CUDA engine never calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "libattn_oracle.so"
_lib = None

F16 = 0
BF16 = 1


def build() -> None:
    """Compile libattn_oracle.so (and oracle/_ref when the reference is present)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(_LIB_PATH))
        u16p = ctypes.POINTER(ctypes.c_uint16)
        L.oracle_attn.argtypes = [u16p, u16p, u16p, u16p, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_long, ctypes.c_long,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.oracle_attn.restype = ctypes.c_int
        L.oracle_attn_alt.argtypes = L.oracle_attn.argtypes
        L.oracle_attn_alt.restype = ctypes.c_int
        L.oracle_attn_rows.argtypes = [u16p, u16p, u16p, u16p, ctypes.POINTER(ctypes.c_int64),
                                       ctypes.c_long, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_long, ctypes.c_long, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int]
        L.oracle_attn_rows.restype = ctypes.c_int
        L.oracle_max_threads.restype = ctypes.c_int
        for n, a, r in (("oracle_f32_to_f16", ctypes.c_float, ctypes.c_uint16),
                        ("oracle_f32_to_bf16", ctypes.c_float, ctypes.c_uint16),
                        ("oracle_f16_to_f32", ctypes.c_uint16, ctypes.c_float),
                        ("oracle_bf16_to_f32", ctypes.c_uint16, ctypes.c_float)):
            getattr(L, n).argtypes = [a]
            getattr(L, n).restype = r
        _lib = L
    return _lib


def _u16(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype not in (np.uint16, np.float16):
        raise TypeError(f"expected 16-bit storage, got {a.dtype}")
    return a.view(np.uint16)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16))


def attention(Q, K, V, *, S: int | None = None, bn_tile: int = 128, dtype: int = F16,
              nthreads: int = 0) -> np.ndarray:
    """Full attention over [B, H, rows, D] 16-bit arrays (uint16 bit patterns or
    float16).  Q has rows >= S, K and V rows >= S; returns O shaped like Q with
    rows >= S zero."""
    q, k, v = _u16(Q), _u16(K), _u16(V)
    B, H, sqo, D = q.shape
    skv = k.shape[2]
    S = sqo if S is None else S
    out = np.zeros_like(q)
    rc = lib().oracle_attn(_ptr(q), _ptr(k), _ptr(v), _ptr(out), B, H, S, D, sqo, skv, bn_tile,
                           dtype, nthreads)
    if rc != 0:
        raise ValueError(f"oracle_attn failed: {rc}")
    return out


def attention_alt(Q, K, V, *, S: int | None = None, bn_tile: int = 128, dtype: int = F16,
                  nthreads: int = 0) -> np.ndarray:
    """attention() in the floating-point order of the reference's second CPU
    oracle (verify_attn.cu:4619-4674): the same function, other roundings."""
    q, k, v = _u16(Q), _u16(K), _u16(V)
    B, H, sqo, D = q.shape
    skv = k.shape[2]
    S = sqo if S is None else S
    out = np.zeros_like(q)
    rc = lib().oracle_attn_alt(_ptr(q), _ptr(k), _ptr(v), _ptr(out), B, H, S, D, sqo, skv,
                               bn_tile, dtype, nthreads)
    if rc != 0:
        raise ValueError(f"oracle_attn_alt failed: {rc}")
    return out


def pattern_inputs(B: int, H: int, S: int, D: int, dtype: int = F16):
    """The deterministic inputs of the reference's root test driver
    (verify_attn.cu:4575-4591): with i the flat [B, H, S, D] index,
    q = ((13 i + 7) mod 31 - 15) / 128, k = ((17 i + 5) mod 29 - 14) / 128,
    v = ((19 i + 3) mod 23 - 11) / 128, all exact in f16 and bf16."""
    i = np.arange(B * H * S * D, dtype=np.int64)
    q = ((i * 13 + 7) % 31 - 15).astype(np.float32) / 128.0
    k = ((i * 17 + 5) % 29 - 14).astype(np.float32) / 128.0
    v = ((i * 19 + 3) % 23 - 11).astype(np.float32) / 128.0
    shape = (B, H, S, D)
    return tuple(from_f32(a, dtype).reshape(shape) for a in (q, k, v))


def attention_rows(Q, K, V, rows, *, S: int | None = None, bn_tile: int = 128,
                   dtype: int = F16, nthreads: int = 0) -> np.ndarray:
    """Selected query rows (rows[i] = (b*H + h)*S + s); returns [n, D] uint16."""
    q, k, v = _u16(Q), _u16(K), _u16(V)
    B, H, sqo, D = q.shape
    skv = k.shape[2]
    S = sqo if S is None else S
    r = np.ascontiguousarray(np.asarray(rows, dtype=np.int64))
    out = np.zeros((r.size, D), dtype=np.uint16)
    rc = lib().oracle_attn_rows(_ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                r.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), r.size, B, H, S,
                                D, sqo, skv, bn_tile, dtype, nthreads)
    if rc != 0:
        raise ValueError(f"oracle_attn_rows failed: {rc}")
    return out


def to_f32(a: np.ndarray, dtype: int) -> np.ndarray:
    """Decode 16-bit storage to float32 (f16 or bf16)."""
    a = _u16(a)
    if dtype == F16:
        return a.view(np.float16).astype(np.float32)
    return (a.astype(np.uint32) << 16).view(np.float32)


def from_f32(a: np.ndarray, dtype: int) -> np.ndarray:
    """Encode float32 to 16-bit storage with round-to-nearest-even."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    if dtype == F16:
        return a.astype(np.float16).view(np.uint16)
    x = a.view(np.uint32).astype(np.uint64)
    nan = (x & 0x7FFFFFFF) > 0x7F800000
    r = ((x + 0x7FFF + ((x >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((x[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def ref_binary() -> Path:
    return _HERE / "_ref" / "ref_attn"


def max_threads() -> int:
    return int(lib().oracle_max_threads())
