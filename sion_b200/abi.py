"""ctypes binding of the C ABI in include/felix_c.h (libfelix_b200.so).

This is the binding a Python caller of the drop-in boundary would write; tests
and bench.py call the kernels through it so that what they check and time is
the C ABI itself. Helpers accept torch tensors (device pointers are taken with
``data_ptr()``) and use torch's current CUDA stream unless one is given.
"""
from __future__ import annotations

import ctypes as C
import os
import re

from . import LIB_PATH

SUCCESS, KERNEL_LAUNCH_FAILED, KERNEL_RUNTIME_ERROR, API_ERROR = 0, 1, 2, 3
B_KN, B_NK = 0, 1

_HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                       "include", "felix_c.h")

_SIGS = {
    "felix_last_cuda_error": (C.c_int, []),
    "felix_last_error_message": (C.c_char_p, []),
    "felix_version": (C.c_char_p, []),
    "felix_sgemm": (C.c_int, [C.c_uint32] * 3 + [C.c_float, C.c_void_p, C.c_void_p, C.c_float,
                                                  C.c_void_p, C.c_void_p]),
    "felix_sgemm_ex": (C.c_int, [C.c_uint32] * 3 + [C.c_float, C.c_void_p, C.c_void_p,
                                                     C.c_float, C.c_void_p, C.c_int, C.c_void_p,
                                                     C.c_size_t, C.c_void_p]),
    "felix_sgemm_noalloc": (C.c_int, [C.c_uint32] * 3 + [C.c_float, C.c_void_p, C.c_void_p,
                                                          C.c_float, C.c_void_p, C.c_int,
                                                          C.c_void_p]),
    "felix_sgemm_workspace_size": (C.c_int, [C.c_uint32] * 3 + [C.c_int,
                                                                 C.POINTER(C.c_size_t)]),
    "felix_hgemm": (C.c_int, [C.c_uint32] * 3 + [C.c_float, C.c_void_p, C.c_void_p, C.c_float,
                                                  C.c_void_p, C.c_int, C.c_void_p]),
    "felix_hgemm_ex": (C.c_int, [C.c_uint32] * 3 + [C.c_float, C.c_void_p, C.c_void_p,
                                                     C.c_float, C.c_void_p, C.c_int, C.c_int,
                                                     C.c_int, C.c_int, C.c_void_p, C.c_size_t,
                                                     C.c_void_p]),
    "felix_hgemm_workspace_size": (C.c_int, [C.c_uint32] * 3 + [C.c_int, C.c_int, C.c_int,
                                                                 C.POINTER(C.c_size_t)]),
    "felix_hgemm_ex2": (C.c_int, [C.c_uint32] * 3 + [C.c_float, C.c_void_p, C.c_void_p,
                                                      C.c_float, C.c_void_p, C.c_int, C.c_int,
                                                      C.c_int, C.c_int, C.c_int, C.c_void_p,
                                                      C.c_size_t, C.c_void_p]),
    "felix_hgemm_workspace_size2": (C.c_int, [C.c_uint32] * 3 + [C.c_int] * 4 +
                                    [C.POINTER(C.c_size_t)]),
    "felix_flash_attn_fwd": (C.c_int, [C.c_void_p] * 5 + [C.c_uint32] * 4 + [C.c_float,
                                                                            C.c_void_p]),
    "felix_flash_attn_bwd": (C.c_int, [C.c_void_p] * 9 + [C.c_uint32] * 4 +
                             [C.c_float, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]),
    "felix_flash_attn_bwd_workspace_size": (C.c_int, [C.c_uint32] * 4 + [C.POINTER(C.c_size_t)]),
    "felix_topk_select": (C.c_int, [C.c_void_p, C.c_void_p] + [C.c_uint32] * 3 +
                          [C.c_int, C.c_void_p]),
    "felix_flash_attn_fwd_ex": (C.c_int, [C.c_void_p] * 5 + [C.c_uint32] * 4 +
                                [C.c_float, C.c_int, C.c_void_p]),
    "felix_watchdog_status": (C.c_int, [C.POINTER(C.c_uint), C.c_int]),
    "felix_watchdog_probe": (C.c_int, [C.c_uint32, C.c_void_p]),
    "felix_num_sms": (C.c_int, [C.POINTER(C.c_int)]),
}

_lib = None


class FelixError(RuntimeError):
    def __init__(self, code: int, cuda: int, msg: str):
        names = {1: "KERNEL_LAUNCH_FAILED", 2: "KERNEL_RUNTIME_ERROR", 3: "API_ERROR"}
        super().__init__(f"{names.get(code, code)} | cudaError {cuda} | {msg}")
        self.code, self.cuda = code, cuda


def header_symbols() -> list[str]:
    """Function names declared in include/felix_c.h."""
    txt = open(_HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(felix_[a-z0-9_]+)\s*\(", txt)))


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} missing; run `python -m sion_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(code: int) -> None:
    if code != SUCCESS:
        L = lib()
        raise FelixError(code, L.felix_last_cuda_error(),
                         (L.felix_last_error_message() or b"").decode())


def _stream(stream):
    if stream is None:
        import torch
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return C.c_void_p(stream)
    return C.c_void_p(stream.cuda_stream)


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def sgemm(A, B, C_out, alpha=1.0, beta=0.0, split_k=None, workspace=None, stream=None):
    M, K = A.shape
    N = B.shape[1]
    L = lib()
    if split_k is None and workspace is None:
        check(L.felix_sgemm(M, N, K, alpha, _ptr(A), _ptr(B), beta, _ptr(C_out),
                            _stream(stream)))
    else:
        ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        check(L.felix_sgemm_ex(M, N, K, alpha, _ptr(A), _ptr(B), beta, _ptr(C_out),
                               int(split_k or 0), _ptr(workspace), ws_bytes, _stream(stream)))
    return C_out


def sgemm_noalloc(A, B, C_out, alpha=1.0, beta=0.0, split_k=0, stream=None):
    """SGEMM through felix_sgemm_noalloc (split-K scratch in the library's
    static device array; nothing is allocated)."""
    M, K = A.shape
    N = B.shape[1]
    check(lib().felix_sgemm_noalloc(M, N, K, alpha, _ptr(A), _ptr(B), beta, _ptr(C_out),
                                    int(split_k), _stream(stream)))
    return C_out


def hgemm(A, B, C_out, alpha=1.0, beta=0.0, b_layout=B_NK, block_n=None, stream_k=None,
          max_ctas=None, workspace=None, stream=None, cta_pair=None):
    M, K = A.shape
    N = B.shape[0] if b_layout == B_NK else B.shape[1]
    L = lib()
    if cta_pair is not None:
        ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        check(L.felix_hgemm_ex2(M, N, K, alpha, _ptr(A), _ptr(B), beta, _ptr(C_out), b_layout,
                                int(block_n or 0), int(stream_k or 0), int(max_ctas or 0),
                                int(cta_pair), _ptr(workspace), ws_bytes, _stream(stream)))
        return C_out
    if block_n is None and stream_k is None and max_ctas is None and workspace is None:
        check(L.felix_hgemm(M, N, K, alpha, _ptr(A), _ptr(B), beta, _ptr(C_out), b_layout,
                            _stream(stream)))
    else:
        ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        check(L.felix_hgemm_ex(M, N, K, alpha, _ptr(A), _ptr(B), beta, _ptr(C_out), b_layout,
                               int(block_n or 0), int(stream_k or 0), int(max_ctas or 0),
                               _ptr(workspace), ws_bytes, _stream(stream)))
    return C_out


def hgemm_workspace_size(M, N, K, block_n=0, stream_k=0, max_ctas=0) -> int:
    n = C.c_size_t(0)
    check(lib().felix_hgemm_workspace_size(M, N, K, block_n, stream_k, max_ctas, C.byref(n)))
    return n.value


def hgemm_workspace_size2(M, N, K, block_n=0, stream_k=0, max_ctas=0, cta_pair=0) -> int:
    n = C.c_size_t(0)
    check(lib().felix_hgemm_workspace_size2(M, N, K, block_n, stream_k, max_ctas, cta_pair,
                                            C.byref(n)))
    return n.value


def sgemm_workspace_size(M, N, K, split_k=0) -> int:
    n = C.c_size_t(0)
    check(lib().felix_sgemm_workspace_size(M, N, K, split_k, C.byref(n)))
    return n.value


def flash_attn_fwd(Q, K, V, O, lse=None, scale=0.0, causal=False, stream=None):
    B, H, S, D = Q.shape
    if causal:
        check(lib().felix_flash_attn_fwd_ex(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(lse), H, B,
                                            S, D, float(scale), 1, _stream(stream)))
    else:
        check(lib().felix_flash_attn_fwd(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(lse), H, B, S,
                                         D, float(scale), _stream(stream)))
    return O


def flash_attn_bwd(Q, K, V, O, dO, lse, dQ, dK, dV, scale=0.0, causal=False, workspace=None,
                   stream=None):
    B, H, S, D = Q.shape
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib().felix_flash_attn_bwd(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(dO), _ptr(lse),
                                     _ptr(dQ), _ptr(dK), _ptr(dV), H, B, S, D, float(scale),
                                     1 if causal else 0, _ptr(workspace), ws_bytes,
                                     _stream(stream)))
    return dQ, dK, dV


def flash_attn_bwd_workspace_size(heads, batch, seqlen, head_dim) -> int:
    n = C.c_size_t(0)
    check(lib().felix_flash_attn_bwd_workspace_size(heads, batch, seqlen, head_dim, C.byref(n)))
    return n.value


def topk_select(data, out, k, largest=True, stream=None):
    """data [num_slices, slice_size] fp32 -> out [num_slices]: k-th largest/smallest."""
    num_slices, slice_size = data.shape
    check(lib().felix_topk_select(_ptr(data), _ptr(out), num_slices, slice_size, k,
                                  1 if largest else 0, _stream(stream)))
    return out


def watchdog_status(clear=True) -> int:
    code = C.c_uint(0)
    rc = lib().felix_watchdog_status(C.byref(code), 1 if clear else 0)
    if rc not in (SUCCESS, KERNEL_RUNTIME_ERROR):
        check(rc)
    return code.value


def watchdog_probe(limit_us: int, stream=None) -> None:
    check(lib().felix_watchdog_probe(limit_us, _stream(stream)))


def num_sms() -> int:
    n = C.c_int(0)
    check(lib().felix_num_sms(C.byref(n)))
    return n.value
