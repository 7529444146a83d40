"""Float cosine scores (SpeedEngine over a float32 corpus) through the bf16
tensor-core pass: every kept pair is rescored with the reference's fp32
arithmetic, so the ranked lists equal the oracle's exactly (ties by the
lower id) and equal the exact CUDA-core scan's."""
import ctypes

import numpy as np
import pytest

import cases
import oracle
from helpers import Stats, capi, ptr

pytestmark = pytest.mark.gpu

MDH_SCORE_SPEED, MDH_SCORE_SPEED_BATCH = 1, 2


def _search(L, h, Q, k, mode):
    ids = np.empty((len(Q), k), np.int32)
    score = np.empty((len(Q), k), np.float32)
    s = Stats()
    st = L.mdh_search_f32(h, ptr(np.ascontiguousarray(Q)), len(Q), k, mode, ptr(ids), ptr(score), ctypes.byref(s))
    assert st == 0, L.mdh_last_error()
    return ids, score, s


@pytest.mark.parametrize("d,n,k", [(768, 60_000, 10), (96, 30_000, 32), (200, 20_000, 10)])
def test_bf16_cosine_pass_is_exact(d, n, k):
    L = capi()
    X = cases.cos_gmm_f32(n, d, 32, seed=81)
    Q = cases.cos_gmm_f32(150, d, 32, seed=81, stream=1)
    h = ctypes.c_void_p()
    assert L.mdh_index_create_f32(ptr(X), n, d, 0, None, 0, 0, ctypes.byref(h)) == 0, L.mdh_last_error()
    try:
        want_ids, want_sc = oracle.speed_exact(X, Q, k, True)
        for mode in (MDH_SCORE_SPEED_BATCH, MDH_SCORE_SPEED):
            ids, sc, s = _search(L, h, Q, k, mode)
            np.testing.assert_array_equal(ids, want_ids)
            np.testing.assert_array_equal(sc, want_sc)  # the reference's own fp32 scores
            assert s.tensor_core_path == 3
        L.mdh_set_scan_path(1)
        ids1, sc1, s1 = _search(L, h, Q, k, MDH_SCORE_SPEED_BATCH)
        assert s1.tensor_core_path == 0
        np.testing.assert_array_equal(ids1, want_ids)
    finally:
        L.mdh_set_scan_path(0)
        L.mdh_index_destroy(h)


def test_bf16_cosine_pass_overflow_reruns():
    """A tiny candidate cap forces overflow reruns (exact CUDA-core filter)."""
    L = capi()
    X = cases.cos_gmm_f32(40_000, 128, 4, seed=83)
    Q = cases.cos_gmm_f32(64, 128, 4, seed=83, stream=1)
    h = ctypes.c_void_p()
    assert L.mdh_index_create_f32(ptr(X), len(X), 128, 0, None, 0, 0, ctypes.byref(h)) == 0
    try:
        assert L.mdh_set_candidate_cap_limit(64) == 0
        ids, sc, _ = _search(L, h, Q, 10, MDH_SCORE_SPEED_BATCH)
        want_ids, want_sc = oracle.speed_exact(X, Q, 10, True)
        np.testing.assert_array_equal(ids, want_ids)
        np.testing.assert_array_equal(sc, want_sc)
    finally:
        L.mdh_set_candidate_cap_limit(0)
        L.mdh_index_destroy(h)
