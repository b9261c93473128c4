"""ctypes front end of the CPU oracle (oracle/oracle.c) and of the reference
build in oracle/_ref/.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py, as the checker and the CPU
baseline. The product (vkcuda_b200/) never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libfa_ref.so")

_lib: Optional[ctypes.CDLL] = None
_ref: Optional[ctypes.CDLL] = None

_P = ctypes.c_void_p


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.oracle_max_threads.restype = ctypes.c_int
        L.oracle_fa_runif.restype = ctypes.c_double
        L.oracle_fa_runif.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
        L.oracle_fa_gaussian.restype = ctypes.c_float
        L.oracle_fa_gaussian.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
        L.oracle_fa_inputs.argtypes = [ctypes.c_uint32, ctypes.c_int64, _P, _P, _P]
        L.oracle_attention.argtypes = [_P, _P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.oracle_gemm.argtypes = [_P, _P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.oracle_vadd.argtypes = [_P, _P, _P, ctypes.c_int64, ctypes.c_int]
        L.oracle_sum_f64.restype = ctypes.c_double
        L.oracle_sum_f64.argtypes = [_P, ctypes.c_int64, ctypes.c_int]
        L.oracle_block_reduce.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        _lib = L
    return _lib


def ref_lib() -> Optional[ctypes.CDLL]:
    """The reference's own flash_attn.vc host code, when oracle/_ref was built."""
    global _ref
    if _ref is None and os.path.exists(REF_LIB_PATH):
        R = ctypes.CDLL(REF_LIB_PATH)
        R.ref_fa_runif.restype = ctypes.c_double
        R.ref_fa_runif.argtypes = [ctypes.POINTER(ctypes.c_uint)]
        R.ref_fa_gaussian.restype = ctypes.c_float
        R.ref_fa_gaussian.argtypes = [ctypes.POINTER(ctypes.c_uint)]
        R.ref_fa_inputs.argtypes = [ctypes.c_uint, _P, _P, _P]
        R.ref_fa_attention.argtypes = [_P, _P, _P, _P, ctypes.c_float, ctypes.c_int]
        R.ref_fa_shape.restype = ctypes.c_int
        R.ref_fa_shape.argtypes = [ctypes.c_int]
        _ref = R
    return _ref


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def max_threads() -> int:
    return lib().oracle_max_threads()


# ------------------------------------------------------------------ attention
DEMO_SHAPE = (2, 64, 16)  # NHEAD, SEQ, HDIM of examples/flash_attn.vc:50-54


def demo_scale(d: int) -> np.float32:
    """float(log2(e) / sqrt(d)) as the demo computes it (flash_attn.vc:211)."""
    return np.float32(1.4426950408889634 / np.sqrt(np.float64(d)))


def fa_inputs(seed: int, elems: int):
    Q = np.empty(elems, np.float32)
    K = np.empty(elems, np.float32)
    V = np.empty(elems, np.float32)
    lib().oracle_fa_inputs(seed, elems, _p(Q), _p(K), _p(V))
    return Q, K, V


def attention(Q, K, V, BH: int, N: int, d: int, scale_log2: float, causal: bool,
              bh_range=None, row_range=None, threads: int = 0, out: Optional[np.ndarray] = None):
    """fp64 referenceAttn over [BH][N][d] fp32 arrays (fp16/bf16 values
    widened to fp32 by the caller). Returns O (rows outside the ranges are
    zero unless `out` is given)."""
    assert d <= 1024
    Q = np.ascontiguousarray(Q, np.float32).reshape(-1)
    K = np.ascontiguousarray(K, np.float32).reshape(-1)
    V = np.ascontiguousarray(V, np.float32).reshape(-1)
    O = out if out is not None else np.zeros(BH * N * d, np.float32)
    b0, b1 = bh_range or (0, BH)
    r0, r1 = row_range or (0, N)
    lib().oracle_attention(_p(Q), _p(K), _p(V), _p(O), BH, N, d, float(scale_log2),
                           1 if causal else 0, b0, b1, r0, r1, threads)
    return O


# ------------------------------------------------------------------ GEMM
def gemm(A, B, M: int, N: int, K: int, lda: int, ldb: int, b_kn: bool = True, Cin=None,
         ldc: int = 0, rows=None, threads: int = 0) -> np.ndarray:
    """fp64 D[M][N] = A * B (+ Cin) over fp32 arrays holding the (fp16 / bf16)
    input values; rows outside `rows` stay zero."""
    A = np.ascontiguousarray(A, np.float32).reshape(-1)
    B = np.ascontiguousarray(B, np.float32).reshape(-1)
    D = np.zeros(M * N, np.float64)
    c = None
    if Cin is not None:
        c = np.ascontiguousarray(Cin, np.float32).reshape(-1)
    r0, r1 = rows or (0, M)
    lib().oracle_gemm(_p(A), _p(B), _p(D), _p(c) if c is not None else None, M, N, K, lda, ldb,
                      N, ldc, 1 if b_kn else 0, r0, r1, threads)
    return D.reshape(M, N)


# ------------------------------------------------------------------ streaming
def vadd(a, b, threads: int = 0) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    c = np.empty_like(a)
    lib().oracle_vadd(_p(a), _p(b), _p(c), a.size, threads)
    return c


def sum_f64(x, threads: int = 0) -> float:
    x = np.ascontiguousarray(x, np.float32)
    return lib().oracle_sum_f64(_p(x), x.size, threads)


def block_reduce(x, block: int, groups: Optional[int] = None) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    n = x.size
    g = groups if groups is not None else (n + block - 1) // block
    out = np.empty(g, np.float32)
    lib().oracle_block_reduce(_p(x), _p(out), n, block, g)
    return out


# ------------------------------------------------------------------ reference build
def ref_fa_inputs(seed: int):
    R = ref_lib()
    if R is None:
        return None
    nh, seq, hd = (R.ref_fa_shape(i) for i in range(3))
    e = nh * seq * hd
    Q, K, V = (np.empty(e, np.float32) for _ in range(3))
    R.ref_fa_inputs(seed, _p(Q), _p(K), _p(V))
    return Q, K, V


def ref_fa_attention(Q, K, V, scale: float, causal: bool):
    R = ref_lib()
    if R is None:
        return None
    O = np.empty_like(np.ascontiguousarray(Q, np.float32))
    R.ref_fa_attention(_p(np.ascontiguousarray(Q, np.float32)),
                       _p(np.ascontiguousarray(K, np.float32)),
                       _p(np.ascontiguousarray(V, np.float32)), _p(O), float(scale),
                       1 if causal else 0)
    return O
