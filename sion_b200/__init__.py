"""sion_b200 — Sion's operator hot path (SGEMM, HGEMM, flash-attention forward)
as sm_100a kernels behind the reference's felix:: / sion:: interfaces.

Python surface (mirrors the reference module ``sion``, python/binding.cpp:6-11):

    sgemm(A, B, alpha=1, beta=0)        fp32, A [M,K] @ B [K,N]
    hgemm(A, B, alpha=1, beta=0)        fp16, B stored [K,N]   ("nn")
    hgemm_nt(A, B, alpha=1, beta=0)     fp16, B stored [N,K]   ("nt")
    gemm(A, B, alpha=1, beta=0)         dispatch on dtype
    flash_attention(Q, K, V)            fp16 [B,H,S,D], D in {64,128}
    flash_attention_lse(Q, K, V)        -> (O, fp32 LSE [B,H,S])
    flash_attention_backward(Q, K, V, O, LSE, dO) -> (dQ, dK, dV)
    flash_attention_autograd(Q, K, V)   differentiable forward (torch.autograd)

These come from the native module ``_sion`` (LibTorch C++), which calls the
felix:: C++ API in ``libfelix_b200.so``. The C ABI of that library
(include/felix_c.h) is reachable through :mod:`sion_b200.abi`. There is no
fallback: if the native libraries are missing, every call raises.
"""
from __future__ import annotations

import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libfelix_b200.so")

_ext = None


def _load_ext():
    global _ext
    if _ext is None:
        import importlib

        import torch  # noqa: F401  (loads libc10/libtorch for the extension)

        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m sion_b200.build`")
        try:
            _ext = importlib.import_module("sion_b200._sion")
        except ImportError as e:
            raise ImportError(
                "sion_b200._sion native module is missing or failed to load "
                f"({e}); build it with `python -m sion_b200.build`") from e
    return _ext


def sgemm(A, B, alpha: float = 1.0, beta: float = 0.0):
    return _load_ext().sgemm(A, B, alpha, beta)


def hgemm(A, B, alpha: float = 1.0, beta: float = 0.0):
    return _load_ext().hgemm(A, B, alpha, beta)


def hgemm_nt(A, B, alpha: float = 1.0, beta: float = 0.0):
    return _load_ext().hgemm_nt(A, B, alpha, beta)


def gemm(A, B, alpha: float = 1.0, beta: float = 0.0):
    return _load_ext().gemm(A, B, alpha, beta)


def flash_attention(query, key, value, causal: bool = False):
    return _load_ext().flash_attention(query, key, value, causal)


def flash_attention_lse(query, key, value, causal: bool = False):
    return _load_ext().flash_attention_lse(query, key, value, causal)


def flash_attention_backward(query, key, value, out, lse, grad_out, causal: bool = False):
    """(dQ, dK, dV) of flash_attention given the forward's O and LSE."""
    return _load_ext().flash_attention_backward(query, key, value, out, lse, grad_out, causal)


def _autograd_function():
    import torch

    class FlashAttentionFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx, query, key, value, causal):
            out, lse = flash_attention_lse(query, key, value, causal)
            ctx.save_for_backward(query, key, value, out, lse)
            ctx.causal = causal
            return out

        @staticmethod
        def backward(ctx, grad_out):
            q, k, v, out, lse = ctx.saved_tensors
            dq, dk, dv = flash_attention_backward(q, k, v, out, lse, grad_out.contiguous(),
                                                  ctx.causal)
            return dq, dk, dv, None

    return FlashAttentionFunction


_FA_FN = None


def flash_attention_autograd(query, key, value, causal: bool = False):
    """flash_attention that torch.autograd can differentiate (the backward runs
    the sm_100a backward kernel)."""
    global _FA_FN
    if _FA_FN is None:
        _FA_FN = _autograd_function()
    return _FA_FN.apply(query, key, value, causal)


__all__ = ["sgemm", "hgemm", "hgemm_nt", "gemm", "flash_attention", "flash_attention_lse",
           "flash_attention_backward", "flash_attention_autograd", "LIB_PATH"]
