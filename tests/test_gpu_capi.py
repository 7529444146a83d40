"""GPU tests through the C ABI: distances, device-resident search, shard merge."""
import ctypes

import numpy as np
import pytest

import cases
import oracle
from helpers import Stats, capi, ptr

pytestmark = pytest.mark.gpu


def _create_u8(L, C, metric=1, id_offset=0, devices=None):
    h = ctypes.c_void_p()
    dev = None
    nd = 0
    if devices:
        dev = np.asarray(devices, np.int32)
        nd = len(devices)
    st = L.mdh_index_create_u8(ptr(np.ascontiguousarray(C)), C.shape[0], C.shape[1], metric, ptr(dev), nd, id_offset,
                               ctypes.byref(h))
    assert st == 0, L.mdh_last_error()
    return h


def _search_u8(L, h, Q, k):
    nq = len(Q)
    ids = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.int32)
    s = Stats()
    st = L.mdh_search_u8(h, ptr(np.ascontiguousarray(Q)), nq, k, ptr(ids), ptr(dist), ctypes.byref(s))
    assert st == 0, L.mdh_last_error()
    return ids, dist, s


@pytest.mark.parametrize("path", [1, 2, 3, 0])
def test_search_u8_distances_exact(path):
    L = capi()
    L.mdh_set_scan_path(path)
    try:
        C = cases.gmm_u8(300_000, 128, 256, seed=21)
        Q = cases.gmm_u8_queries(1300, 128, 256, seed_means=21, seed_q=22)
        h = _create_u8(L, C)
        ids, dist, s = _search_u8(L, h, Q, 10)
        want_ids, want_d = oracle.l2_exact_u8_int(C, Q, 10)
        np.testing.assert_array_equal(ids, want_ids)
        np.testing.assert_array_equal(dist, want_d)
        assert s.bound_violations == 0 and s.pairs_scored >= C.shape[0] * len(Q)
        assert s.tensor_core_path == {1: 0, 2: 1, 3: 2, 0: 1}[path]
        assert L.mdh_index_destroy(h) == 0
    finally:
        L.mdh_set_scan_path(0)


@pytest.mark.parametrize("nq", [1, 5, 64, 100, 255, 256, 300, 513])
def test_tensor_scan_batch_shapes(nq):
    """Both tensor tile shapes (128 and 256 queries per CTA) and partial query groups."""
    L = capi()
    L.mdh_set_scan_path(2)
    try:
        C = cases.gmm_u8(70_001, 128, 128, seed=23)
        Q = cases.gmm_u8_queries(nq, 128, 128, seed_means=23, seed_q=24)
        h = _create_u8(L, C)
        ids, dist, s = _search_u8(L, h, Q, 16)
        want_ids, want_d = oracle.l2_exact_u8_int(C, Q, 16)
        np.testing.assert_array_equal(ids, want_ids)
        np.testing.assert_array_equal(dist, want_d)
        assert s.tensor_core_path == 1
        assert L.mdh_index_destroy(h) == 0
    finally:
        L.mdh_set_scan_path(0)


@pytest.mark.parametrize("nq", [1, 3, 8, 9, 40])
@pytest.mark.parametrize("metric", [1, 0])
def test_stream_scan_batch_shapes(nq, metric):
    """The streaming CUDA-core scan (query groups of 1/2/4/8, partial last group), L2 and cosine."""
    L = capi()
    L.mdh_set_scan_path(1)
    try:
        C = cases.gmm_u8(50_001, 128, 128, seed=25)
        Q = cases.gmm_u8_queries(nq, 128, 128, seed_means=25, seed_q=26)
        h = _create_u8(L, C, metric=metric)
        ids, dist, s = _search_u8(L, h, Q, 12)
        if metric == 1:
            want_ids, want_d = oracle.l2_exact_u8_int(C, Q, 12)
            np.testing.assert_array_equal(dist, want_d)
        else:
            want_ids = oracle.cosine_exact_u8(C, Q.astype(np.float32), 12)[0]
        np.testing.assert_array_equal(ids, want_ids)
        assert s.tensor_core_path == 0
        assert L.mdh_index_destroy(h) == 0
    finally:
        L.mdh_set_scan_path(0)


@pytest.mark.parametrize("metric", [1, 0])
def test_verification_counts_zero_violations(metric):
    """mdh_set_verify: an exact unpruned re-scan of sampled queries finds no misplaced rows."""
    L = capi()
    assert L.mdh_set_verify(48) == 0
    try:
        C = cases.gmm_u8(150_000, 128, 64, seed=27)
        Q = cases.gmm_u8_queries(300, 128, 64, seed_means=27, seed_q=28)
        h = _create_u8(L, C, metric=metric)
        ids, _, s = _search_u8(L, h, Q, 10)
        assert s.verified_queries == 48
        assert s.bound_violations == 0
        assert 300 * 10 <= s.candidates <= 300 * 16384
        if metric == 1:
            np.testing.assert_array_equal(ids, oracle.l2_exact_u8_int(C, Q, 10)[0])
        assert L.mdh_index_destroy(h) == 0
    finally:
        assert L.mdh_set_verify(0) == 0
    assert L.mdh_set_verify(-1) != 0


def test_device_api_and_merge():
    torch = pytest.importorskip("torch")
    L = capi()
    C = cases.gmm_u8(120_000, 128, 64, seed=31)
    Q = cases.gmm_u8_queries(257, 128, 64, seed_means=31, seed_q=32)
    k = 10
    want_ids, want_d = oracle.l2_exact_u8_int(C, Q, k)
    # Two shards with global ids, searched through the device API, merged on device.
    half = C.shape[0] // 2
    shards = [(C[:half], 0), (C[half:], half)]
    dq = torch.from_numpy(Q).cuda()
    all_d = torch.empty((2, len(Q), k), dtype=torch.int32, device="cuda")
    all_i = torch.empty((2, len(Q), k), dtype=torch.int32, device="cuda")
    handles = []
    for s, (part, off) in enumerate(shards):
        h = _create_u8(L, part, id_offset=off)
        handles.append(h)
        st = L.mdh_search_u8_device(h, ctypes.c_void_p(dq.data_ptr()), len(Q), k, ctypes.c_void_p(all_i[s].data_ptr()),
                                    ctypes.c_void_p(all_d[s].data_ptr()), None, None)
        assert st == 0, L.mdh_last_error()
    out_d = torch.empty((len(Q), k), dtype=torch.int32, device="cuda")
    out_i = torch.empty((len(Q), k), dtype=torch.int32, device="cuda")
    st = L.mdh_merge_topk_device(ctypes.c_void_p(all_d.data_ptr()), ctypes.c_void_p(all_i.data_ptr()), 2, len(Q), k,
                                 ctypes.c_void_p(out_d.data_ptr()), ctypes.c_void_p(out_i.data_ptr()), None)
    assert st == 0, L.mdh_last_error()
    np.testing.assert_array_equal(out_i.cpu().numpy(), want_ids)
    np.testing.assert_array_equal(out_d.cpu().numpy(), want_d)
    for h in handles:
        L.mdh_index_destroy(h)


def test_multi_device_index_matches_single():
    L = capi()
    n = L.mdh_device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    C = cases.gmm_u8(200_000, 128, 64, seed=41)
    Q = cases.gmm_u8_queries(64, 128, 64, seed_means=41, seed_q=42)
    h1 = _create_u8(L, C)
    hn = _create_u8(L, C, devices=list(range(min(n, 4))))
    a = _search_u8(L, h1, Q, 10)
    b = _search_u8(L, hn, Q, 10)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    L.mdh_index_destroy(h1)
    L.mdh_index_destroy(hn)


def test_float_queries_through_capi():
    L = capi()
    C, Q = cases.case_float_queries()
    h = _create_u8(L, C)
    ids = np.empty((len(Q), 10), np.int32)
    dist = np.empty((len(Q), 10), np.float32)
    st = L.mdh_search_f32(h, ptr(Q), len(Q), 10, 0, ptr(ids), ptr(dist), None)
    assert st == 0, L.mdh_last_error()
    want_ids, want_d = oracle.l2_exact_u8(C, Q, 10)
    np.testing.assert_array_equal(ids, want_ids)
    np.testing.assert_array_equal(dist, want_d)  # bit-identical float distances
    L.mdh_index_destroy(h)


@pytest.mark.parametrize("k", [10, 100])
def test_cooperative_thresholds_two_shards(k):
    """Two row shards (global ids) searched with shared thresholds:
    mdh_search_u8_device_sample on each, the lists merged on the device, then
    mdh_search_u8_device_bounded on each with the merged lists; merging the
    bounded results gives the oracle's exact top-k.  The searches plan for
    thresholds shared by 2 ranks (mdh_set_threshold_sharing), so each rank's
    sample chain stops at a smaller sample than it would alone."""
    torch = pytest.importorskip("torch")
    L = capi()
    C = cases.gmm_u8(400_000, 128, 256, seed=33)
    Q = np.ascontiguousarray(cases.gmm_u8_queries(300, 128, 256, seed_means=33, seed_q=34))
    want_ids, want_d = oracle.l2_topk_u8(C, Q, k)
    half = C.shape[0] // 2
    hs = [_create_u8(L, C[:half], id_offset=0), _create_u8(L, C[half:], id_offset=half)]
    assert L.mdh_set_threshold_sharing(2) == 0
    dq = torch.from_numpy(Q).cuda()
    nq = len(Q)

    def merged(lists):
        all_d = torch.stack([d for d, _ in lists]).contiguous()
        all_i = torch.stack([i for _, i in lists]).contiguous()
        out_d = torch.empty((nq, k), dtype=torch.int32, device="cuda")
        out_i = torch.empty_like(out_d)
        assert L.mdh_merge_topk_device(ctypes.c_void_p(all_d.data_ptr()), ctypes.c_void_p(all_i.data_ptr()), 2, nq,
                                       k, ctypes.c_void_p(out_d.data_ptr()), ctypes.c_void_p(out_i.data_ptr()),
                                       None) == 0, L.mdh_last_error()
        return out_d, out_i

    phase1 = []
    for h in hs:
        d = torch.empty((nq, k), dtype=torch.int32, device="cuda")
        i = torch.empty_like(d)
        s = Stats()
        assert L.mdh_search_u8_device_sample(h, ctypes.c_void_p(dq.data_ptr()), nq, k, ctypes.c_void_p(i.data_ptr()),
                                             ctypes.c_void_p(d.data_ptr()), None, ctypes.byref(s)) == 0, \
            L.mdh_last_error()
        assert s.full_scan_pairs < half * nq  # only sample rows were scanned
        phase1.append((d, i))
    thr_d, thr_i = merged(phase1)
    phase2 = []
    for h in hs:
        d = torch.empty((nq, k), dtype=torch.int32, device="cuda")
        i = torch.empty_like(d)
        s = Stats()
        assert L.mdh_search_u8_device_bounded(h, ctypes.c_void_p(dq.data_ptr()), nq, k,
                                              ctypes.c_void_p(thr_d.data_ptr()), ctypes.c_void_p(thr_i.data_ptr()),
                                              ctypes.c_void_p(i.data_ptr()), ctypes.c_void_p(d.data_ptr()), None,
                                              ctypes.byref(s)) == 0, L.mdh_last_error()
        assert s.levels == 1 and s.full_scan_pairs == half * nq
        phase2.append((d, i))
    out_d, out_i = merged(phase2)
    assert L.mdh_set_threshold_sharing(1) == 0
    np.testing.assert_array_equal(out_i.cpu().numpy(), want_ids)
    np.testing.assert_array_equal(out_d.cpu().numpy(), want_d)
    for h in hs:
        assert L.mdh_index_destroy(h) == 0
