"""CPU oracle — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg / reference
arm may import this package, and only as the checker or the timed CPU
baseline; nothing in sion_b200/ imports it.

Wraps oracle/liboracle.so (plain C, fp64; see oracle.c for the reference
file:line each function restates). numpy in, numpy (float64) out.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_DIR = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_DIR, "liboracle.so")
_lib = None


def build() -> str:
    src = os.path.join(_DIR, "oracle.c")
    if not os.path.exists(_SO) or os.path.getmtime(src) > os.path.getmtime(_SO):
        subprocess.run(["make", "-s", "-C", _DIR, "CC=gcc"], check=True)
    return _SO


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(_SO)
        P = C.c_void_p
        L.oracle_sgemm.argtypes = [C.c_int64] * 3 + [C.c_double, P, P, C.c_double, P, P]
        L.oracle_hgemm.argtypes = [C.c_int64] * 3 + [C.c_double, P, P, C.c_int, C.c_double, P, P]
        L.oracle_attention_rows.argtypes = [C.c_int64] * 4 + [P, P, P, C.c_double, P, C.c_int64,
                                                              P, P, C.c_int]
        L.oracle_half_to_double.restype = C.c_double
        L.oracle_half_to_double.argtypes = [C.c_uint16]
        L.oracle_double_to_half.restype = C.c_uint16
        L.oracle_double_to_half.argtypes = [C.c_double]
        L.oracle_half_to_double_array.argtypes = [P, P, C.c_int64]
        L.oracle_double_to_half_array.argtypes = [P, P, C.c_int64]
        L.oracle_attention_bwd.argtypes = [C.c_int64] * 4 + [P, P, P, P, C.c_double, C.c_int,
                                                             P, P, P]
        L.oracle_topk.argtypes = [P, P, C.c_int64, C.c_int64, C.c_int64, C.c_int]
        L.oracle_set_threads.argtypes = [C.c_int]
        L.oracle_get_threads.restype = C.c_int
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _half_bits(a) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return a.view(np.uint16)
    assert a.dtype == np.uint16, a.dtype
    return a


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def threads() -> int:
    return lib().oracle_get_threads()


def sgemm(A: np.ndarray, B: np.ndarray, alpha=1.0, beta=0.0, C0=None) -> np.ndarray:
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M, K = A.shape
    N = B.shape[1]
    assert B.shape[0] == K
    c0 = None if C0 is None else np.ascontiguousarray(C0, dtype=np.float32)
    out = np.empty((M, N), np.float64)
    lib().oracle_sgemm(M, N, K, alpha, _p(A), _p(B), beta, _p(c0), _p(out))
    return out


def hgemm(A, B, nt: bool, alpha=1.0, beta=0.0, C0=None) -> np.ndarray:
    """nt=True: B is [N, K]; nt=False: B is [K, N]. fp16 arrays (or uint16 bits)."""
    A = _half_bits(A)
    B = _half_bits(B)
    M, K = A.shape
    N = B.shape[0] if nt else B.shape[1]
    c0 = None if C0 is None else _half_bits(C0)
    out = np.empty((M, N), np.float64)
    lib().oracle_hgemm(M, N, K, alpha, _p(A), _p(B), 1 if nt else 0, beta, _p(c0), _p(out))
    return out


def attention(Q, K, V, scale=0.0, rows=None, causal=False):
    """Q, K, V fp16 [B, H, S, D]. Returns (O [B,H,R,D] f64, LSE [B,H,R] f64) for the
    query rows `rows` (all rows when None); causal: query i sees keys 0..i."""
    Q, K, V = _half_bits(Q), _half_bits(K), _half_bits(V)
    Bn, H, S, D = Q.shape
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    R = S if r is None else len(r)
    O = np.empty((Bn, H, R, D), np.float64)
    L = np.empty((Bn, H, R), np.float64)
    lib().oracle_attention_rows(Bn, H, S, D, _p(Q), _p(K), _p(V), float(scale), _p(r),
                                0 if r is None else len(r), _p(O), _p(L), 1 if causal else 0)
    return O, L


def attention_bwd(Q, K, V, dO, scale=0.0, causal=False):
    """fp16 [B, H, S, D] inputs -> (dQ, dK, dV) float64 of softmax(Q K^T scale) V."""
    Q, K, V, dO = _half_bits(Q), _half_bits(K), _half_bits(V), _half_bits(dO)
    Bn, H, S, D = Q.shape
    dQ, dK, dV = (np.empty((Bn, H, S, D), np.float64) for _ in range(3))
    lib().oracle_attention_bwd(Bn, H, S, D, _p(Q), _p(K), _p(V), _p(dO), float(scale),
                               1 if causal else 0, _p(dQ), _p(dK), _p(dV))
    return dQ, dK, dV


def topk(data: np.ndarray, k: int, largest: bool = True) -> np.ndarray:
    """data [num_slices, slice_size] float32 -> [num_slices] float32: the k-th
    largest / smallest value of each slice, bit-exact."""
    d = np.ascontiguousarray(data, dtype=np.float32)
    ns, n = d.shape
    out = np.empty(ns, np.uint32)
    lib().oracle_topk(_p(d.view(np.uint32)), _p(out), ns, n, int(k), 1 if largest else 0)
    return out.view(np.float32)


def half_to_double(bits: np.ndarray) -> np.ndarray:
    bits = _half_bits(bits)
    out = np.empty(bits.shape, np.float64)
    lib().oracle_half_to_double_array(_p(bits), _p(out), bits.size)
    return out


def double_to_half(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float64)
    out = np.empty(x.shape, np.uint16)
    lib().oracle_double_to_half_array(_p(x), _p(out), x.size)
    return out
