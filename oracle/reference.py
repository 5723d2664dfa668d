"""The reference's own kernels (oracle/_ref/libsion_ref.so, built from the
unmodified reference sources by oracle/build_ref.sh) — TEST INFRASTRUCTURE
ONLY: a comparator for tests/ and bench.py's reference arm.

Shapes must satisfy the reference's own limits: SGEMM M, N, K multiples of 64
(cute_sgemm_64x64_nn has no bounds checks), HGEMM M, N multiples of 128 and K of
64, attention seqlen multiple of 64, head_dim 64 or 128.
"""
from __future__ import annotations

import ctypes as C
import os

LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libsion_ref.so")
_lib = None


def available() -> bool:
    return os.path.exists(LIB)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        L = C.CDLL(LIB)
        P = C.c_void_p
        L.ref_sgemm.argtypes = [C.c_uint32] * 3 + [C.c_float, P, P, C.c_float, P, P]
        L.ref_hgemm.argtypes = [C.c_uint32] * 3 + [C.c_float, P, P, C.c_float, P, C.c_int, P]
        L.ref_flash_attn.argtypes = [P] * 4 + [C.c_uint32] * 4 + [P]
        _lib = L
    return _lib


def _stream(stream):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"reference {what} failed (status {rc})")


def sgemm(A, B, C_out, alpha=1.0, beta=0.0, stream=None):
    M, K = A.shape
    N = B.shape[1]
    assert M % 64 == 0 and N % 64 == 0 and K % 64 == 0, "reference SGEMM needs 64-multiples"
    _check(lib().ref_sgemm(M, N, K, alpha, A.data_ptr(), B.data_ptr(), beta, C_out.data_ptr(),
                           _stream(stream)), "sgemm")
    return C_out


def hgemm(A, B, C_out, nt=True, alpha=1.0, beta=0.0, stream=None):
    M, K = A.shape
    N = B.shape[0] if nt else B.shape[1]
    assert M % 128 == 0 and N % 128 == 0 and K % 64 == 0, "reference HGEMM needs 128/128/64"
    _check(lib().ref_hgemm(M, N, K, alpha, A.data_ptr(), B.data_ptr(), beta, C_out.data_ptr(),
                           1 if nt else 0, _stream(stream)), "hgemm")
    return C_out


def flash_attn(Q, K, V, O, stream=None):
    B, H, S, D = Q.shape
    assert S % 64 == 0 and D in (64, 128), "reference attention needs S % 64 == 0, D in {64,128}"
    _check(lib().ref_flash_attn(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), H, B, S,
                                D, _stream(stream)), "flash_attn")
    return O
