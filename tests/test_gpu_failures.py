"""Failure handling on the GPU, exercised without a device fault.

* The scans' bounded mbarrier wait, run on a barrier that nothing arrives
  on with a short budget (mdh_check_wait_timeout): it must give up and the
  call must report MDH_ERR_TIMEOUT; the device stays usable.
* Host-side injected faults (mdh_set_fault): an out-of-memory workspace
  growth and a failing shard search thread come back as status codes, and
  the next search on the same index is exact again.
"""
import ctypes

import numpy as np
import pytest

import cases
import oracle
from helpers import capi, ptr

pytestmark = pytest.mark.gpu

MDH_ERR_OOM = 4
MDH_ERR_TIMEOUT = 5
MDH_ERR_INTERNAL = 8


def _index(L, C, devices=None):
    h = ctypes.c_void_p()
    dev = np.asarray(devices, np.int32) if devices else None
    st = L.mdh_index_create_u8(ptr(C), C.shape[0], C.shape[1], 1, ptr(dev), len(devices or []), 0, ctypes.byref(h))
    assert st == 0, L.mdh_last_error()
    return h


def _search(L, h, Q, k):
    ids = np.empty((len(Q), k), np.int32)
    dist = np.empty((len(Q), k), np.int32)
    st = L.mdh_search_u8(h, ptr(Q), len(Q), k, ptr(ids), ptr(dist), None)
    return st, ids, dist


@pytest.fixture(scope="module")
def data():
    C = cases.gmm_u8(60_000, 128, 64, seed=91)
    Q = cases.gmm_u8_queries(200, 128, 64, seed_means=91, seed_q=92)
    return C, Q, oracle.l2_exact_u8_int(C, Q, 10)


def test_bounded_wait_gives_up_and_reports_timeout(data):
    L = capi()
    for budget in (2_000_000, 50_000_000):  # ~1 ms and ~25 ms at B200 clocks
        st = L.mdh_check_wait_timeout(-1, budget)
        assert st == MDH_ERR_TIMEOUT, (st, L.mdh_last_error())
        assert b"gave up" in L.mdh_last_error()
    assert L.mdh_check_wait_timeout(-1, 10) != 0 and b"budget" in L.mdh_last_error()
    # The context is intact: a search right after is exact.
    C, Q, (want_i, want_d) = data
    h = _index(L, C)
    st, ids, dist = _search(L, h, Q, 10)
    assert st == 0, L.mdh_last_error()
    np.testing.assert_array_equal(ids, want_i)
    np.testing.assert_array_equal(dist, want_d)
    assert L.mdh_index_destroy(h) == 0


def test_injected_out_of_memory_then_recovery(data):
    L = capi()
    C, Q, (want_i, want_d) = data
    h = _index(L, C)  # fresh: its first search grows the workspace
    assert L.mdh_set_fault(1) == 0
    st, _, _ = _search(L, h, Q, 10)
    assert st == MDH_ERR_OOM and b"injected" in L.mdh_last_error()
    st, ids, dist = _search(L, h, Q, 10)  # the fault fired once
    assert st == 0, L.mdh_last_error()
    np.testing.assert_array_equal(ids, want_i)
    np.testing.assert_array_equal(dist, want_d)
    assert L.mdh_index_destroy(h) == 0
    assert L.mdh_set_fault(4) != 0 and b"site" in L.mdh_last_error()
    assert L.mdh_set_fault(0) == 0


@pytest.mark.parametrize("devices", [None, [0, 0]])
def test_injected_shard_failure_then_recovery(data, devices):
    """A shard thread that fails before its scan (one shard, or one of two
    shards sharing the GPU) fails the call with its message; the next search
    on the same index is exact."""
    L = capi()
    C, Q, (want_i, want_d) = data
    h = _index(L, C, devices)
    st, ids, _ = _search(L, h, Q, 10)
    assert st == 0, L.mdh_last_error()
    assert L.mdh_set_fault(2) == 0
    st, _, _ = _search(L, h, Q, 10)
    assert st == MDH_ERR_INTERNAL and b"injected fault" in L.mdh_last_error()
    st, ids, dist = _search(L, h, Q, 10)
    assert st == 0, L.mdh_last_error()
    np.testing.assert_array_equal(ids, want_i)
    np.testing.assert_array_equal(dist, want_d)
    assert L.mdh_index_destroy(h) == 0
