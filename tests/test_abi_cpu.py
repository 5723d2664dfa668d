"""C ABI boundary checks that need no GPU: the library loads and exports
every function include/felix_c.h declares, and argument validation that runs
before any device work."""
import ctypes
import os

import pytest

from sion_b200 import LIB_PATH, abi


def test_library_exists():
    assert os.path.exists(LIB_PATH), "run python -m sion_b200.build"


def test_exports_every_header_symbol():
    L = ctypes.CDLL(LIB_PATH)
    syms = abi.header_symbols()
    assert len(syms) >= 13
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing


def test_abi_table_covers_header():
    assert sorted(abi._SIGS) == abi.header_symbols()


def test_version_and_codes():
    L = abi.lib()
    assert b"sm_100a" in L.felix_version()
    assert (abi.SUCCESS, abi.KERNEL_LAUNCH_FAILED, abi.KERNEL_RUNTIME_ERROR, abi.API_ERROR) == \
        (0, 1, 2, 3)


def test_invalid_layout_is_api_error_without_device():
    L = abi.lib()
    rc = L.felix_hgemm(128, 128, 64, 1.0, None, None, 0.0, None, 7, None)
    assert rc == abi.API_ERROR
    assert b"b_layout" in L.felix_last_error_message()
    rc = L.felix_hgemm_ex(128, 128, 64, 1.0, None, None, 0.0, None, abi.B_NK, 0, 5, 0, None, 0,
                          None)
    assert rc == abi.API_ERROR
    rc = L.felix_sgemm_ex(8, 8, 8, 1.0, None, None, 0.0, None, -1, None, 0, None)
    assert rc == abi.API_ERROR


def test_no_device_is_reported_not_crashed():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    n = ctypes.c_int(0)
    rc = abi.lib().felix_num_sms(ctypes.byref(n))
    assert rc == abi.KERNEL_LAUNCH_FAILED
