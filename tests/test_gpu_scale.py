"""Parity at the sizes the throughput numbers are quoted on (GPU, C ABI).

The headline search (100M x 128 u8, 10,000 queries, top-10) runs a sample
plan with more levels than the small parity cases reach: the nested samples
grow with the corpus, so only a corpus of several million rows exercises the
largest sample -> full-shard step and its candidate capacity.  These cases
compare ids and exact integer distances with the oracle's int64 ranking
(MadhavaL2::search_exact, src/winnex_madhava.cpp:1224-1246: ascending
(distance, index)):

* 10,000,000 x 128 u8 from the 4,096-component clipped mixture of the
  headline corpus, 128 queries, k = 10 and k = 100: with the default plan
  (a chain of 6-7 levels, as at 100M rows), and with the plan a rank of an
  8-way shared-threshold split uses (mdh_set_threshold_sharing(8)), searched
  alone: its smaller last sample leaves many more candidates, which must not
  change the result;
* the batched configuration at its stated shape: 1,000,000 x 128 u8
  (256 components), 1,000 of its 10,000 queries, k = 10 and k = 100.
"""
import ctypes

import numpy as np
import pytest

import cases
import oracle
from helpers import Stats, capi, ptr

pytestmark = pytest.mark.gpu


def _build(L, C):
    h = ctypes.c_void_p()
    st = L.mdh_index_create_u8(ptr(np.ascontiguousarray(C)), C.shape[0], C.shape[1], 1, None, 0, 0, ctypes.byref(h))
    assert st == 0, L.mdh_last_error()
    return h


def _search(L, h, Q, k):
    ids = np.empty((len(Q), k), np.int32)
    dist = np.empty((len(Q), k), np.int32)
    s = Stats()
    st = L.mdh_search_u8(h, ptr(np.ascontiguousarray(Q)), len(Q), k, ptr(ids), ptr(dist), ctypes.byref(s))
    assert st == 0, L.mdh_last_error()
    return ids, dist, s


@pytest.fixture(scope="module")
def big():
    L = capi()
    C = cases.gmm_u8(10_000_000, 128, 4096, seed=61)
    Q = cases.gmm_u8_queries(128, 128, 4096, seed_means=61, seed_q=62)
    h = _build(L, C)
    want = {k: oracle.l2_topk_u8(C, Q, k) for k in (10, 100)}
    yield L, h, Q, want
    assert L.mdh_index_destroy(h) == 0


@pytest.mark.parametrize("sharing", [1, 8])
@pytest.mark.parametrize("k", [10, 100])
def test_headline_plan_10m_rows(big, sharing, k):
    L, h, Q, want = big
    assert L.mdh_set_threshold_sharing(sharing) == 0
    try:
        ids, dist, s = _search(L, h, Q, k)
    finally:
        assert L.mdh_set_threshold_sharing(1) == 0
    np.testing.assert_array_equal(ids, want[k][0])
    np.testing.assert_array_equal(dist, want[k][1])
    assert s.levels >= 5
    assert s.tensor_core_path == 1 and s.bound_violations == 0
    assert s.full_scan_pairs == 10_000_000 * len(Q)
    # Every scanned pair is either settled by the block bound or formed.
    assert 0 < s.pairs_pruned_by_bound < s.pairs_scored
    assert 0 < s.blocks_passed < s.blocks_tested


@pytest.fixture(scope="module")
def config2():
    L = capi()
    C = cases.gmm_u8(1_000_000, 128, 256, seed=63)
    Q = np.ascontiguousarray(cases.gmm_u8_queries(10_000, 128, 256, seed_means=63, seed_q=64)[::10])
    h = _build(L, C)
    yield L, h, C, Q
    assert L.mdh_index_destroy(h) == 0


@pytest.mark.parametrize("k", [10, 100])
def test_batched_1m_rows_1000_queries(config2, k):
    L, h, C, Q = config2
    ids, dist, s = _search(L, h, Q, k)
    want_ids, want_d = oracle.l2_topk_u8(C, Q, k)
    np.testing.assert_array_equal(ids, want_ids)
    np.testing.assert_array_equal(dist, want_d)
    assert s.tensor_core_path == 1 and s.bound_violations == 0
