"""The allocation-free device search (mdh_search_u8_device_noalloc), through
the C ABI, against the oracle and against the allocating device search
(mdh_search_u8_device).

Collected last (file name) so it also runs after every other GPU test in the
same process; it passes alone as well.  Distances are exact integers, so the
comparison tolerance is zero.
"""
import ctypes

import numpy as np
import pytest

import cases
import oracle
from helpers import Stats, capi, ptr

pytestmark = pytest.mark.gpu

MDH_ERR_UNSUPPORTED = 7


def _index(L, C):
    h = ctypes.c_void_p()
    st = L.mdh_index_create_u8(ptr(np.ascontiguousarray(C)), C.shape[0], C.shape[1], 1, None, 0, 0, ctypes.byref(h))
    assert st == 0, L.mdh_last_error()
    return h


def _call(L, fn, h, dq, nq, ids, dist):
    s = Stats()
    st = fn(h, ctypes.c_void_p(dq.data_ptr()), nq, ids.shape[1], ctypes.c_void_p(ids.data_ptr()),
            ctypes.c_void_p(dist.data_ptr()), None, ctypes.byref(s))
    assert st == 0, L.mdh_last_error()
    return s


def _workspace_bytes(L, h):
    ws = ctypes.c_int64(-1)
    assert L.mdh_index_memory(h, None, ctypes.byref(ws)) == 0, L.mdh_last_error()
    return ws.value


@pytest.mark.parametrize("nq,k", [(256, 10), (40, 100)])
def test_noalloc_on_a_fresh_index_matches_oracle_and_device_search(nq, k):
    torch = pytest.importorskip("torch")
    L = capi()
    C = cases.gmm_u8(200_000, 128, 64, seed=51)
    Q = cases.gmm_u8_queries(nq, 128, 64, seed_means=51, seed_q=52)
    want_i, want_d = oracle.l2_exact_u8_int(C, Q, k)
    h = _index(L, C)
    dq = torch.from_numpy(Q).cuda()
    # No allocating search has run on this index: its search workspace is empty
    # and must stay so through the no-alloc calls.
    assert _workspace_bytes(L, h) == 0
    got = [(torch.full((nq, k), -7, dtype=torch.int32, device="cuda"),
            torch.full((nq, k), -7, dtype=torch.int32, device="cuda")) for _ in range(3)]
    _call(L, L.mdh_search_u8_device_noalloc, h, dq, nq, *got[0])  # first call on the device: set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    stats = [_call(L, L.mdh_search_u8_device_noalloc, h, dq, nq, *got[i]) for i in (1, 2)]
    free1, _ = torch.cuda.mem_get_info()
    assert _workspace_bytes(L, h) == 0
    for i_, d_ in got:
        np.testing.assert_array_equal(i_.cpu().numpy(), want_i)
        np.testing.assert_array_equal(d_.cpu().numpy(), want_d)
    for s in stats:
        assert s.kernel_launches > 0 and s.bound_violations == 0
    # Two calls in a row took no device memory (a candidate scratch for these
    # shapes alone would be megabytes).
    assert free1 >= free0 - (1 << 20), (free0, free1)
    # The allocating search agrees (and does grow the workspace).
    ai = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    ad = torch.empty_like(ai)
    _call(L, L.mdh_search_u8_device, h, dq, nq, ai, ad)
    np.testing.assert_array_equal(ai.cpu().numpy(), want_i)
    np.testing.assert_array_equal(ad.cpu().numpy(), want_d)
    assert _workspace_bytes(L, h) > 0
    assert L.mdh_index_destroy(h) == 0


def test_noalloc_candidate_overflow_reruns_exactly():
    """30,000 copies of one row among 150,000: at k = 256 the queries equal to
    that row tie at distance 0 with every copy, so the no-alloc path's
    4,096-entry candidate lists overflow and rerun with tighter thresholds
    (ids break the ties) until they fit; the result is still the oracle's."""
    torch = pytest.importorskip("torch")
    L = capi()
    rng = np.random.default_rng(57)
    C = cases.gmm_u8(150_000, 128, 64, seed=57)
    dup = rng.choice(len(C), size=30_000, replace=False)
    C[dup] = C[dup[0]]
    Q = np.concatenate([np.repeat(C[dup[:1]], 6, axis=0), cases.gmm_u8_queries(26, 128, 64, 57, 58)])
    nq, k = len(Q), 256
    want_i, want_d = oracle.l2_exact_u8_int(C, Q, k)
    h = _index(L, C)
    dq = torch.from_numpy(Q).cuda()
    for _ in range(2):
        ids = torch.full((nq, k), -7, dtype=torch.int32, device="cuda")
        dd = torch.full_like(ids, -7)
        s = _call(L, L.mdh_search_u8_device_noalloc, h, dq, nq, ids, dd)
        np.testing.assert_array_equal(ids.cpu().numpy(), want_i)
        np.testing.assert_array_equal(dd.cpu().numpy(), want_d)
        # A rerun scans the full level again: more than one full pass of pairs.
        assert s.pairs_scored >= 2 * len(C) * nq, s.pairs_scored
    assert L.mdh_index_destroy(h) == 0


def test_noalloc_rejects_beyond_limits():
    torch = pytest.importorskip("torch")
    L = capi()
    C = cases.gmm_u8(5_000, 128, 16, seed=53)
    h = _index(L, C)
    dq = torch.zeros((257, 128), dtype=torch.uint8, device="cuda")
    ids = torch.empty((257, 10), dtype=torch.int32, device="cuda")
    st = L.mdh_search_u8_device_noalloc(h, ctypes.c_void_p(dq.data_ptr()), 257, 10, ctypes.c_void_p(ids.data_ptr()),
                                        None, None, None)
    assert st == MDH_ERR_UNSUPPORTED and b"at most 256 queries" in L.mdh_last_error()
    big = torch.empty((4, 300), dtype=torch.int32, device="cuda")
    st = L.mdh_search_u8_device_noalloc(h, ctypes.c_void_p(dq.data_ptr()), 4, 300, ctypes.c_void_p(big.data_ptr()),
                                        None, None, None)
    assert st == MDH_ERR_UNSUPPORTED and b"k <= 256" in L.mdh_last_error()
    assert L.mdh_index_destroy(h) == 0
