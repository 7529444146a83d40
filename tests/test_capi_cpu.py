"""C-ABI library checks that need no GPU: it loads, exports every declared
entry point, validates arguments, and refuses to run without a device (the
product has no CPU fallback)."""
import ctypes

import numpy as np
import pytest

from helpers import HEADER, LIB, capi, header_functions


def test_library_exports_every_header_symbol():
    L = ctypes.CDLL(LIB)
    fns = header_functions()
    assert len(fns) >= 12
    missing = [f for f in fns if not hasattr(L, f)]
    assert not missing, f"not exported: {missing}"


def test_version_and_error_string():
    L = capi()
    assert b"sm_100a" in L.mdh_version()
    assert isinstance(L.mdh_last_error(), bytes)


def test_argument_validation_before_device_use():
    L = capi()
    out = ctypes.c_void_p()
    C = np.zeros((4, 8), np.uint8)
    # dim out of range
    assert L.mdh_index_create_u8(ctypes.c_void_p(C.ctypes.data), 4, 0, 1, None, 0, 0, ctypes.byref(out)) == 1
    assert b"dim" in L.mdh_last_error()
    # metric out of range
    assert L.mdh_index_create_u8(ctypes.c_void_p(C.ctypes.data), 4, 8, 5, None, 0, 0, ctypes.byref(out)) == 1
    # null output
    assert L.mdh_index_create_u8(ctypes.c_void_p(C.ctypes.data), 4, 8, 1, None, 0, 0, None) == 1
    # id range
    assert L.mdh_index_create_u8(ctypes.c_void_p(C.ctypes.data), 4, 8, 1, None, 0, 2**31 - 2, ctypes.byref(out)) == 1
    assert L.mdh_set_scan_path(7) == 1
    assert L.mdh_set_candidate_cap_limit(100) == 1
    assert L.mdh_set_candidate_cap_limit(0) == 0
    assert L.mdh_search_f32(None, None, 1, 10, 0, None, None, None) == 1


def test_no_cpu_fallback_without_gpu():
    L = capi()
    if L.mdh_device_count() > 0:
        pytest.skip("a GPU is present")
    out = ctypes.c_void_p()
    C = np.zeros((4, 8), np.uint8)
    st = L.mdh_index_create_u8(ctypes.c_void_p(C.ctypes.data), 4, 8, 1, None, 0, 0, ctypes.byref(out))
    assert st == 2  # MDH_ERR_CUDA
    assert b"no CUDA device" in L.mdh_last_error()
    assert not out.value


def test_header_is_plain_c():
    src = open(HEADER).read()
    assert 'extern "C"' in src
    for banned in ("torch", "std::", "class ", "template"):
        assert banned not in src
