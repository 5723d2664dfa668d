"""``import sion`` for existing callers of the reference's Python module.

The reference builds its operators as a module named ``sion``
(python/binding.cpp:6-11: ``sgemm``, ``flash_attention``), imported by its
python/sgemm_test.py and python/flash_attn_test.py. This package re-exports
the sm_100a implementation in :mod:`sion_b200` under that name, so those
callers run unchanged; the extra operators (hgemm, hgemm_nt, gemm,
flash_attention_lse, the backward) come along.
"""
from sion_b200 import (  # noqa: F401
    LIB_PATH,
    flash_attention,
    flash_attention_autograd,
    flash_attention_backward,
    flash_attention_lse,
    gemm,
    hgemm,
    hgemm_nt,
    sgemm,
)

__all__ = ["sgemm", "hgemm", "hgemm_nt", "gemm", "flash_attention", "flash_attention_lse",
           "flash_attention_backward", "flash_attention_autograd", "LIB_PATH"]
