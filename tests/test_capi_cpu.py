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
    assert L.mdh_audit_u8(None, None, 1, 10, 5, None, None, None, None, None, None) == 1
    assert L.mdh_audit_f32(None, None, 1, 0, 5, None, None, None, None, None, None) == 1
    assert L.mdh_ivf_create_f32(None, 10, 8, None, 2, None, -1, None) == 1
    h = ctypes.c_void_p()
    assert L.mdh_ivf_create_f32(None, 10, 8, None, 2, None, -1, ctypes.byref(h)) == 1 and not h.value
    assert L.mdh_ivf_search_f32(None, None, 1, 10, 2, None, None, None) == 1


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


@pytest.mark.parametrize("struct", ["mdh_stats", "mdh_audit"])
def test_structs_match_header(tmp_path, struct):
    """The ctypes mirrors of mdh_stats and mdh_audit (tests, bench.py) have the
    header's sizes and field offsets."""
    import shutil
    import subprocess

    from helpers import Audit, Stats

    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    mirror = {"mdh_stats": Stats, "mdh_audit": Audit}[struct]
    src = tmp_path / "s.c"
    names = [f[0] for f in mirror._fields_]
    body = "".join(f'printf("%zu ", offsetof({struct}, {n}));' for n in names)
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "winnex_madhava_b200.h"\n'
                   f'int main(void) {{ {body} printf("%zu\\n", sizeof({struct})); return 0; }}\n')
    exe = tmp_path / "s"
    subprocess.run(["gcc", "-I", HEADER.rsplit("/", 1)[0], str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    want = [getattr(mirror, n).offset for n in names] + [ctypes.sizeof(mirror)]
    assert got == want


def test_sample_plan_follows_the_cost_model():
    """Sample ladders of 1024 * 4^j rows up to shard / 8 (plus a 16,384-row
    level when the ladder stops short of it); a search scans the cheapest
    chain of them under the cost model (largest sample near sqrt(4,500 k n)):
    longer chains for larger shards and larger k, a single dense level for a
    tiny shard, and shorter chains when ranks share their sample thresholds."""
    L = capi()
    assert L.mdh_plan_level_count(100_000_000, 10) == 6
    assert L.mdh_plan_level_count(100_000_000, 100) == 8
    assert L.mdh_plan_level_count(12_500_000, 10) == 6
    assert L.mdh_plan_level_count(1_000_000, 10) == 5
    assert L.mdh_plan_level_count(100_000, 10) == 4         # 1,024 -> 4,096 -> 16,384 -> 100,000
    assert L.mdh_plan_level_count(20_000, 3_020) == 2       # a first level of >= k rows exists
    assert L.mdh_plan_level_count(5_000, 10) == 1          # dense scan of the shard
    assert L.mdh_plan_level_count(0, 10) == 0
    assert L.mdh_set_threshold_sharing(8) == 0
    try:
        assert L.mdh_plan_level_count(12_500_000, 100) == 6  # one fewer than alone
        assert L.mdh_plan_level_count(1_000_000, 10) == 4
    finally:
        assert L.mdh_set_threshold_sharing(1) == 0
    assert L.mdh_set_sample_ratio(64) == 0
    try:
        assert L.mdh_plan_level_count(12_500_000, 10) == 5  # a shorter ladder (top <= n / 64)
    finally:
        assert L.mdh_set_sample_ratio(0) == 0
    assert L.mdh_set_sample_ratio(1) == 1
    assert L.mdh_set_threshold_sharing(0) == 1
