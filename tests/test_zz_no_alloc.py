"""The allocation-free device search (mdh_search_u8_device_noalloc) against
the allocating one (mdh_search_u8_device), both through the C ABI.

Collected last (file name) so it also runs after every other GPU test in the
same process; it passes alone as well.  Distances are exact integers, so the
comparison tolerance is zero.
"""
import ctypes

import numpy as np
import pytest

import cases
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


@pytest.mark.parametrize("nq,k", [(256, 10), (40, 100)])
def test_noalloc_matches_device_search_twice(nq, k):
    torch = pytest.importorskip("torch")
    L = capi()
    C = cases.gmm_u8(200_000, 128, 64, seed=51)
    Q = cases.gmm_u8_queries(nq, 128, 64, seed_means=51, seed_q=52)
    h = _index(L, C)
    dq = torch.from_numpy(Q).cuda()
    want_i = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    want_d = torch.empty_like(want_i)
    _call(L, L.mdh_search_u8_device, h, dq, nq, want_i, want_d)
    got = [(torch.full_like(want_i, -7), torch.full_like(want_i, -7)) for _ in range(3)]
    _call(L, L.mdh_search_u8_device_noalloc, h, dq, nq, *got[0])  # first call on the device: set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    stats = [_call(L, L.mdh_search_u8_device_noalloc, h, dq, nq, *got[i]) for i in (1, 2)]
    free1, _ = torch.cuda.mem_get_info()
    for i_, d_ in got:
        np.testing.assert_array_equal(i_.cpu().numpy(), want_i.cpu().numpy())
        np.testing.assert_array_equal(d_.cpu().numpy(), want_d.cpu().numpy())
    for s in stats:
        assert s.kernel_launches > 0 and s.bound_violations == 0
    # Two calls in a row took no device memory (a candidate scratch for these
    # shapes alone would be megabytes).
    assert free1 >= free0 - (1 << 20), (free0, free1)
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
