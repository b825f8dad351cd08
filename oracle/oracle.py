"""ctypes view of the CPU oracle (oracle/libtcb_oracle.so).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / --impl reference leg use it as the checker.  The shipped
library (tcb_b200) never imports this module.

The oracle restates TR's arithmetic for the quantized matvec path; see
oracle/tcb_oracle.h for the per-function citations of sekerahmet/TCB.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtcb_oracle.so")

Q4_0, Q8_0, Q4_K, Q6_K = 2, 8, 12, 14
FORMATS = (Q8_0, Q4_0, Q4_K, Q6_K)
NAMES = {Q8_0: "q8", Q4_0: "q4", Q4_K: "q4_k", Q6_K: "q6_k"}
BLOCK = {Q8_0: (32, 34), Q4_0: (32, 18), Q4_K: (256, 144), Q6_K: (256, 210)}

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc); returns the .so path."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    L = ctypes.CDLL(LIB_PATH)
    P = ctypes.c_void_p
    I = ctypes.c_int
    Z = ctypes.c_size_t
    L.tcbo_f16_to_f32.argtypes = [ctypes.c_uint16]
    L.tcbo_f16_to_f32.restype = ctypes.c_float
    L.tcbo_dequant.argtypes = [I, P, Z, P]
    L.tcbo_dot_f32.argtypes = [P, P, Z]
    L.tcbo_dot_f32.restype = ctypes.c_float
    L.tcbo_quant_dot.argtypes = [I, P, P, I]
    L.tcbo_quant_dot.restype = ctypes.c_float
    L.tcbo_quant_dot_scalar.argtypes = [I, P, P, I]
    L.tcbo_quant_dot_scalar.restype = ctypes.c_float
    L.tcbo_qgemm_float.argtypes = [I, I, I, I, P, P, P, I]
    L.tcbo_quantize_q8.argtypes = [P, I, I, P, P, P]
    L.tcbo_dot_act8.argtypes = [I, I, P, P, P, P]
    L.tcbo_dot_act8.restype = ctypes.c_float
    L.tcbo_qgemm_act8.argtypes = [I, I, I, I, P, P, P, I]
    L.tcbo_set_pinning.argtypes = [I]
    L.tcbo_embedding.argtypes = [I, P, I, P, I, P]
    L.tcbo_check_scales.argtypes = [I, P, Z]
    L.tcbo_check_scales.restype = ctypes.c_long
    L.tcbo_zero_raw.argtypes = [I, P, Z]
    L.tcbo_random_quant.argtypes = [I, ctypes.c_uint32, Z, P]
    L.tcbo_fnv1a_f32.argtypes = [P, Z]
    L.tcbo_fnv1a_f32.restype = ctypes.c_uint64
    _lib = L
    return L


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def row_bytes(fmt: int, K: int) -> int:
    e, b = BLOCK[fmt]
    return K // e * b


def dequant(fmt: int, raw: np.ndarray) -> np.ndarray:
    e, b = BLOCK[fmt]
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    nb = raw.size // b
    y = np.empty(nb * e, dtype=np.float32)
    lib().tcbo_dequant(fmt, _p(raw), nb, _p(y))
    return y


def dot_f32(x: np.ndarray, y: np.ndarray) -> float:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.ascontiguousarray(y, dtype=np.float32)
    return float(lib().tcbo_dot_f32(_p(x), _p(y), x.size))


def quant_dot(fmt: int, x: np.ndarray, wrow: np.ndarray, scalar: bool = False) -> np.float32:
    x = np.ascontiguousarray(x, dtype=np.float32)
    wrow = np.ascontiguousarray(wrow, dtype=np.uint8)
    f = lib().tcbo_quant_dot_scalar if scalar else lib().tcbo_quant_dot
    return np.float32(f(fmt, _p(x), _p(wrow), x.size))


def qgemm_float(fmt: int, a: np.ndarray, w: np.ndarray, N: int, c: np.ndarray | None = None,
                nthreads: int = 0) -> np.ndarray:
    """c[M,N] (+)= a[M,K] . dequant(w[N,K])^T on TR's float path."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    M, K = a.shape
    w = np.ascontiguousarray(w, dtype=np.uint8)
    out = np.zeros((M, N), np.float32) if c is None else np.array(c, dtype=np.float32, copy=True)
    lib().tcbo_qgemm_float(fmt, M, N, K, _p(a), _p(w), _p(out), nthreads or os.cpu_count() or 1)
    return out


def qgemm_act8(fmt: int, a: np.ndarray, w: np.ndarray, N: int, c: np.ndarray | None = None,
               nthreads: int = 0) -> np.ndarray:
    """c[M,N] (+)= TR's int8-activation product (non-finite rows on the float path)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    M, K = a.shape
    w = np.ascontiguousarray(w, dtype=np.uint8)
    out = np.zeros((M, N), np.float32) if c is None else np.array(c, dtype=np.float32, copy=True)
    lib().tcbo_qgemm_act8(fmt, M, N, K, _p(a), _p(w), _p(out), nthreads or os.cpu_count() or 1)
    return out


def set_pinning(on: bool) -> None:
    """Pin the row-parallel workers of the products, worker t to the t-th
    CPU the process may run on (the timed CPU baseline)."""
    lib().tcbo_set_pinning(1 if on else 0)


def quantize_q8(x: np.ndarray, blk: int):
    x = np.ascontiguousarray(x, dtype=np.float32)
    K = x.size
    q = np.empty(K, np.int8)
    d = np.empty(K // blk, np.float32)
    bs = np.empty(K // 16, np.int16)
    lib().tcbo_quantize_q8(_p(x), K, blk, _p(q), _p(d), _p(bs))
    return q, d, bs


def dot_act8(fmt: int, wrow: np.ndarray, q: np.ndarray, d: np.ndarray, bs: np.ndarray) -> np.float32:
    wrow = np.ascontiguousarray(wrow, dtype=np.uint8)
    return np.float32(lib().tcbo_dot_act8(fmt, q.size, _p(wrow), _p(q), _p(d), _p(bs)))


def embedding(fmt: int, raw: np.ndarray, D: int, idx) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    ix = np.ascontiguousarray(idx, dtype=np.int64)
    out = np.empty((ix.size, D), np.float32)
    lib().tcbo_embedding(fmt, _p(raw), D, _p(ix), ix.size, _p(out))
    return out


def check_scales(fmt: int, raw: np.ndarray) -> int:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    return int(lib().tcbo_check_scales(fmt, _p(raw), raw.size))


def zero_raw(fmt: int, nblocks: int) -> np.ndarray:
    raw = np.empty(nblocks * BLOCK[fmt][1], np.uint8)
    lib().tcbo_zero_raw(fmt, _p(raw), nblocks)
    return raw


def random_quant(fmt: int, seed: int, nblocks: int) -> np.ndarray:
    """TR's randomQuant (tensor/quant_test.go:20-45): LCG bytes, finite scales."""
    raw = np.empty(nblocks * BLOCK[fmt][1], np.uint8)
    lib().tcbo_random_quant(fmt, seed & 0xFFFFFFFF, nblocks, _p(raw))
    return raw


def fnv1a_f32(y: np.ndarray) -> int:
    y = np.ascontiguousarray(y, dtype=np.float32)
    return int(lib().tcbo_fnv1a_f32(_p(y), y.size))
