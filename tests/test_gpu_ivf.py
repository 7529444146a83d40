"""GPU parity of the clustered (IVF) search against the oracle.

The cells are the reference's own: MiniBatchKMeans centroids and labels from
its MadHybrid build (tests/golden/hybrid.npz).  Routing must equal the
oracle's cell lists exactly (same fp64 order); results must equal the exact
top-k over the union of the probed cells, ids and squared distances.
"""
import ctypes

import numpy as np
import pytest

import cases
import oracle
from helpers import Stats, capi, load_fixture, ptr

pytestmark = pytest.mark.gpu


def _ivf(L, C, cen, labels):
    C = np.ascontiguousarray(C, dtype=np.uint8)
    cen = np.ascontiguousarray(cen, dtype=np.float32)
    labels = np.ascontiguousarray(labels, dtype=np.int32)
    h = ctypes.c_void_p()
    st = L.mdh_ivf_create_u8(ptr(C), C.shape[0], C.shape[1], ptr(cen), cen.shape[0], ptr(labels), -1,
                             ctypes.byref(h))
    assert st == 0, L.mdh_last_error()
    return h


def _search(L, h, Q, k, nprobe):
    Q = np.ascontiguousarray(Q, dtype=np.uint8)
    ids = np.empty((len(Q), k), np.int32)
    dist = np.empty((len(Q), k), np.int32)
    s = Stats()
    st = L.mdh_ivf_search_u8(h, ptr(Q), len(Q), k, nprobe, ptr(ids), ptr(dist), ctypes.byref(s))
    assert st == 0, L.mdh_last_error()
    return ids, dist, s


def test_ivf_matches_oracle_on_reference_cells():
    L = capi()
    _, res = load_fixture("hybrid")
    C, Q = cases.case_hybrid()
    cen, labels, nprobe = res["centroids"], res["labels"], cases.HYBRID["nprobe"]
    h = _ivf(L, C, cen, labels)
    cells = np.empty((len(Q), nprobe), np.int32)
    assert L.mdh_ivf_route_u8(h, ptr(Q), len(Q), nprobe, ptr(cells)) == 0, L.mdh_last_error()
    np.testing.assert_array_equal(cells, oracle.ivf_route(cen, Q, nprobe))
    for k in (1, 10, 100):
        ids, dist, s = _search(L, h, Q, k, nprobe)
        want_ids, want_d = oracle.ivf_exact(C, labels, cen, Q, k, nprobe)
        np.testing.assert_array_equal(ids, want_ids)
        np.testing.assert_array_equal(dist[want_ids >= 0], want_d[want_ids >= 0])
        assert s.levels == 3 and s.tensor_core_path == 1 and s.full_scan_pairs > 0  # coarse, sample, full passes
    # probing every cell is the plain exact search
    ids, dist, _ = _search(L, h, Q, 10, cases.HYBRID["nlist"])
    want_ids, want_d = oracle.l2_exact_u8_int(C, Q, 10)
    np.testing.assert_array_equal(ids, want_ids)
    np.testing.assert_array_equal(dist, want_d)
    n = ctypes.c_int64()
    nl = ctypes.c_int32()
    rows = np.empty(cases.HYBRID["nlist"], np.int64)
    assert L.mdh_ivf_info(h, ctypes.byref(n), None, ctypes.byref(nl), ptr(rows)) == 0
    assert n.value == len(C) and nl.value == cases.HYBRID["nlist"]
    np.testing.assert_array_equal(rows, np.bincount(labels, minlength=cases.HYBRID["nlist"]))
    assert L.mdh_ivf_destroy(h) == 0


def test_ivf_route_ties_and_one_lane_holding_the_best():
    """Routing order on ties and when one lane's cells are all the best:
    centroids repeated every 10 cells (each similarity appears 20 times, so
    the lower id decides), then cells 3, 35, 67, ... (one lane of the
    selecting warp) made the 7 best, and every cell probed."""
    L = capi()
    rng = np.random.default_rng(77)
    nlist = 200
    C = rng.integers(0, 256, (2_000, 128), dtype=np.uint8)
    labels = rng.integers(0, nlist, len(C)).astype(np.int32)
    Q = rng.integers(0, 256, (50, 128), dtype=np.uint8)
    base = rng.uniform(0, 1, (10, 128)).astype(np.float32)
    tied = np.ascontiguousarray(np.tile(base, (nlist // 10, 1)))
    one_lane = rng.uniform(0, 1, (nlist, 128)).astype(np.float32)
    one_lane[3::32] *= 10
    for cen, probes in ((tied, (1, 16, 45)), (one_lane, (12, nlist))):
        h = _ivf(L, C, cen, labels)
        for nprobe in probes:
            cells = np.empty((len(Q), nprobe), np.int32)
            assert L.mdh_ivf_route_u8(h, ptr(Q), len(Q), nprobe, ptr(cells)) == 0, L.mdh_last_error()
            np.testing.assert_array_equal(cells, oracle.ivf_route(cen, Q, nprobe), err_msg=f"nprobe {nprobe}")
        assert L.mdh_ivf_destroy(h) == 0


def test_ivf_edge_cells_and_batches():
    """Empty cells, cells smaller than k, a cell larger than a unit's 64 tiles,
    one query and a 700-query batch."""
    L = capi()
    C = cases.gmm_u8(60_000, 128, 64, seed=73)
    Q = cases.gmm_u8_queries(700, 128, 64, seed_means=73, seed_q=74)
    rng = np.random.default_rng(75)
    nlist = 40
    cen = rng.uniform(0, 60, (nlist, 128)).astype(np.float32)
    labels = rng.integers(0, 30, len(C)).astype(np.int32)  # cells 30..39 stay empty
    labels[:20_000] = 5                                    # one cell of 20,000 rows (> 64 tiles)
    labels[20_000:20_003] = 31                             # a 3-row cell
    h = _ivf(L, C, cen, labels)
    for nq, k, nprobe in ((1, 10, 3), (700, 10, 6), (64, 16, 40)):
        ids, dist, _ = _search(L, h, Q[:nq], k, nprobe)
        want_ids, want_d = oracle.ivf_exact(C, labels, cen, Q[:nq], k, nprobe)
        np.testing.assert_array_equal(ids, want_ids)
        np.testing.assert_array_equal(dist[want_ids >= 0], want_d[want_ids >= 0])
    assert L.mdh_ivf_destroy(h) == 0


def test_ivf_chunk_buffer_overflow_reruns_exact():
    """The passes write their unsettled (query, 32-row chunk) blocks to a
    chunk buffer that a re-key kernel turns into candidates.  With a one-block
    buffer (injected, mdh_set_fault(3)) every pass overflows it: passes 0 and
    1 only get looser thresholds, and pass 2 reruns with keys formed in the
    scan, so the results stay the oracle's."""
    L = capi()
    C = cases.gmm_u8(60_000, 128, 64, seed=77)
    Q = cases.gmm_u8_queries(300, 128, 64, seed_means=77, seed_q=78)
    rng = np.random.default_rng(79)
    nlist = 24
    cen = rng.uniform(0, 60, (nlist, 128)).astype(np.float32)
    labels = rng.integers(0, nlist, len(C)).astype(np.int32)
    h = _ivf(L, C, cen, labels)
    want_ids, want_d = oracle.ivf_exact(C, labels, cen, Q, 10, 4)
    for fault in (0, 3, 0):
        assert L.mdh_set_fault(fault) == 0
        ids, dist, s = _search(L, h, Q, 10, 4)
        np.testing.assert_array_equal(ids, want_ids)
        np.testing.assert_array_equal(dist[want_ids >= 0], want_d[want_ids >= 0])
        # A rerun scans the probed cells a second time; the sample passes
        # alone stay far below one scan of them.
        assert (s.pairs_scored >= 2 * s.full_scan_pairs) == bool(fault)
    assert L.mdh_ivf_destroy(h) == 0


def test_ivf_all_keys_tied_large_k():
    """40,000 equal rows in one cell: the last pass's candidate lists hold
    ~2,000 entries with the same key, more than the large-k selection keeps in
    shared memory, so it takes the k smallest (key, id) one at a time."""
    L = capi()
    C = np.full((40_000, 128), 7, np.uint8)
    # Routing takes the largest inner product: the query goes to cell 0.
    cen = np.stack([np.full(128, 200.0), np.full(128, 7.0)]).astype(np.float32)
    labels = np.zeros(len(C), np.int32)  # cell 1 stays empty
    h = _ivf(L, C, cen, labels)
    Q = np.full((3, 128), 7, np.uint8)
    for k in (64, 128):
        ids, dist, _ = _search(L, h, Q, k, 1)
        np.testing.assert_array_equal(ids, np.tile(np.arange(k, dtype=np.int32), (3, 1)))
        np.testing.assert_array_equal(dist, 0)
    assert L.mdh_ivf_destroy(h) == 0


def test_ivf_rejects_bad_input():
    L = capi()
    C = np.zeros((100, 16), np.uint8)
    cen = np.zeros((4, 16), np.float32)
    labels = np.full(100, 4, np.int32)  # out of range
    h = ctypes.c_void_p()
    assert L.mdh_ivf_create_u8(ptr(C), 100, 16, ptr(cen), 4, ptr(labels), -1, ctypes.byref(h)) != 0
    assert b"label" in L.mdh_last_error()


def _structured(n=20_000, d=64, n_clusters=16, seed=7):
    """The reference's hybrid test corpus shape (tests/python/test_hybrid.py:23-38)."""
    rng = np.random.RandomState(seed)
    centers = rng.randn(n_clusters, d).astype(np.float32) * 5.0
    labels = rng.randint(0, n_clusters, n)
    X = centers[labels] + rng.randn(n, d).astype(np.float32) * 0.5
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    Xq = (X - X.min()) / (X.max() - X.min()) * 255
    return X.astype(np.float32), Xq.astype(np.uint8)


def test_hybrid_facade_uint8_l2():
    """build_engine(hybrid=True) on u8/L2 runs on the GPU IVF index; its results
    are the exact top-k over the probed cells of its own clustering, and the
    reference test assertions hold (tests/python/test_hybrid.py:57-67,121-128)."""
    pytest.importorskip("sklearn")
    import winnex_madhava as wm
    _, Xu = _structured()
    eng = wm.build_engine(Xu, dim=Xu.shape[1], k=10, hybrid=True, nlist=16, nprobe=5, metric="l2")
    assert type(eng).__name__ == "MadHybrid" and eng._ivf is not None
    assert eng.num_vectors() == Xu.shape[0] and eng.dim() == Xu.shape[1] and eng.built() is True
    res = eng.search(Xu[0].astype(np.float32), k=10)
    assert len(res.indices) == 10 and all(0 <= int(i) < Xu.shape[0] for i in res.indices)
    Q = Xu[:40]
    got = np.array(eng.search_batch(Q.astype(np.float32), k=10).indices).reshape(40, 10)
    want, _ = oracle.ivf_exact(Xu, eng._labels, eng._centroids, Q, 10, 5)
    np.testing.assert_array_equal(got, want)
    for i in range(5):
        assert eng.search(Q[i].astype(np.float32), k=10).indices == [int(v) for v in want[i] if v >= 0]
    # non-integral queries take the per-cell engines and rank the union by float L2
    qf = Xu[1].astype(np.float32) + 0.25
    r = eng.search(qf, k=10)
    assert len(r.indices) == 10
    default = wm.build_engine(Xu, dim=Xu.shape[1], k=10, metric="l2")
    assert type(default).__name__ == "MadhavaL2" and default.search(Xu[0].astype(np.float32)).bound_violations == 0


def test_ivf_inner_product_on_reference_cells():
    """Metric COSINE (MadHybrid's default): ranking by the inner product, the
    reference's merge `corpus[ids].astype(float32) @ q` (python/winnex_madhava/
    __init__.py:640-646), exact in integers for u8 rows and u8 queries.  The
    reference's own cells (tests/golden/hybrid.npz); ids and inner products
    equal the oracle's exact top-k over the probed cells, and probing every
    cell gives the exact inner-product top-k of the corpus."""
    L = capi()
    _, res = load_fixture("hybrid")
    C, Q = cases.case_hybrid()
    cen, labels, nprobe = res["centroids"], res["labels"], cases.HYBRID["nprobe"]
    Cc, cenc, labc = (np.ascontiguousarray(C, dtype=np.uint8), np.ascontiguousarray(cen, dtype=np.float32),
                      np.ascontiguousarray(labels, dtype=np.int32))
    h = ctypes.c_void_p()
    st = L.mdh_ivf_create_u8_metric(ptr(Cc), Cc.shape[0], Cc.shape[1], ptr(cenc), cenc.shape[0], ptr(labc), 0, -1,
                                    ctypes.byref(h))
    assert st == 0, L.mdh_last_error()
    for k in (1, 10, 100):
        ids, dots, s = _search(L, h, Q, k, nprobe)
        want_ids, want_d = oracle.ivf_exact(C, labels, cen, Q, k, nprobe, metric="ip")
        np.testing.assert_array_equal(ids, want_ids)
        np.testing.assert_array_equal(dots[want_ids >= 0], want_d[want_ids >= 0])
        assert 0 < s.pairs_pruned_by_bound < s.pairs_scored
    ids, dots, _ = _search(L, h, Q, 10, cases.HYBRID["nlist"])
    full = C.astype(np.int64) @ Q.astype(np.int64).T  # [n][nq]
    for i in range(len(Q)):
        order = np.lexsort((np.arange(len(C)), -full[:, i]))[:10]
        np.testing.assert_array_equal(ids[i], order)
        np.testing.assert_array_equal(dots[i], full[order, i])
    assert L.mdh_ivf_destroy(h) == 0


def test_hybrid_facade_default_metric_on_gpu():
    """build_engine(hybrid=True) with the default metric ("cosine") on a u8
    corpus runs one batched call on the GPU IVF index; results are the exact
    inner-product top-k over the probed cells of its own clustering."""
    pytest.importorskip("sklearn")
    import winnex_madhava as wm
    _, Xu = _structured()
    eng = wm.build_engine(Xu, dim=Xu.shape[1], k=10, hybrid=True, nlist=16, nprobe=5)
    assert type(eng).__name__ == "MadHybrid" and eng._ivf is not None and eng._metric == "cosine"
    Q = Xu[:40]
    got = np.array(eng.search_batch(Q.astype(np.float32), k=10).indices).reshape(40, 10)
    want, _ = oracle.ivf_exact(Xu, eng._labels, eng._centroids, Q, 10, 5, metric="ip")
    np.testing.assert_array_equal(got, want)
    assert eng.search(Q[3].astype(np.float32), k=10).indices == [int(v) for v in want[3] if v >= 0]
    assert not eng._cells  # no per-cell engines were built


# ---------------------------------------------------------------- float32 corpora
def _ivf_f32(L, X, cen, labels):
    X = np.ascontiguousarray(X, dtype=np.float32)
    cen = np.ascontiguousarray(cen, dtype=np.float32)
    labels = np.ascontiguousarray(labels, dtype=np.int32)
    h = ctypes.c_void_p()
    st = L.mdh_ivf_create_f32(ptr(X), X.shape[0], X.shape[1], ptr(cen), cen.shape[0], ptr(labels), -1,
                              ctypes.byref(h))
    assert st == 0, L.mdh_last_error()
    return h


def _search_f32(L, h, Q, k, nprobe):
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    ids = np.empty((len(Q), k), np.int32)
    sc = np.empty((len(Q), k), np.float64)
    s = Stats()
    st = L.mdh_ivf_search_f32(h, ptr(Q), len(Q), k, nprobe, ptr(ids), ptr(sc), ctypes.byref(s))
    assert st == 0, L.mdh_last_error()
    return ids, sc, s


def test_ivf_f32_matches_oracle():
    """Float32 cells (the reference's float hybrid path): the exact top-k by
    float64 inner product over the union of the probed cells, ids and scores
    bit for bit (fp64, one fused multiply-add per dimension in order)."""
    L = capi()
    X, _ = _structured(n=20_000, d=64, n_clusters=16, seed=7)
    rng = np.random.default_rng(121)
    nlist = 24
    cen = X[rng.choice(len(X), nlist, replace=False)].astype(np.float32)
    labels = np.argmax(X @ cen.T, axis=1).astype(np.int32)
    Q = (X[rng.choice(len(X), 40, replace=False)] + 0.05 * rng.standard_normal((40, 64))).astype(np.float32)
    h = _ivf_f32(L, X, cen, labels)
    for k, nprobe in ((1, 1), (10, 3), (16, 5), (10, nlist)):
        ids, sc, s = _search_f32(L, h, Q, k, nprobe)
        want_ids, want_sc = oracle.ivf_ip_f32(X, labels, cen, Q, k, nprobe)
        np.testing.assert_array_equal(ids, want_ids)
        np.testing.assert_array_equal(sc[want_ids >= 0], want_sc[want_ids >= 0])
        cells = oracle.ivf_route_f32(cen, Q, nprobe)
        rows = np.bincount(labels, minlength=nlist)
        assert s.pairs_scored == int(rows[cells].sum())
    assert L.mdh_ivf_destroy_f32(h) == 0


def test_ivf_f32_edges():
    """Empty cells, cells holding fewer than k rows (-1 padding), k above 16
    refused, and a query batch of one."""
    L = capi()
    rng = np.random.default_rng(123)
    X = rng.standard_normal((300, 40)).astype(np.float32)
    cen = rng.standard_normal((6, 40)).astype(np.float32)
    labels = np.where(np.arange(300) < 5, 0, 1 + np.arange(300) % 2).astype(np.int32)  # cells 3..5 empty
    h = _ivf_f32(L, X, cen, labels)
    Q = rng.standard_normal((7, 40)).astype(np.float32)
    for k, nprobe in ((16, 1), (8, 2), (16, 6)):
        ids, sc, _ = _search_f32(L, h, Q, k, nprobe)
        want_ids, want_sc = oracle.ivf_ip_f32(X, labels, cen, Q, k, nprobe)
        np.testing.assert_array_equal(ids, want_ids)
        np.testing.assert_array_equal(sc[want_ids >= 0], want_sc[want_ids >= 0])
    ids, _, _ = _search_f32(L, h, Q[:1], 10, 6)
    np.testing.assert_array_equal(ids, oracle.ivf_ip_f32(X, labels, cen, Q[:1], 10, 6)[0])
    out = np.empty((1, 17), np.int32)
    assert L.mdh_ivf_search_f32(h, ptr(Q[:1]), 1, 17, 2, ptr(out), None, None) != 0
    assert b"k must be" in L.mdh_last_error()
    assert L.mdh_ivf_destroy_f32(h) == 0


def test_hybrid_facade_float32_on_gpu():
    """build_engine(X_float, hybrid=True): one batched GPU call per search,
    equal to the oracle's exact top-k over the union of the probed cells of
    the engine's own k-means cells (default metric, and L2: the float cells
    rank by inner product either way)."""
    import winnex_madhava as wm

    X, _ = _structured(n=12_000, d=48, n_clusters=12, seed=9)
    for metric in ("cosine", "l2"):
        eng = wm.build_engine(X, dim=48, k=10, hybrid=True, nlist=16, nprobe=4, metric=metric)
        assert eng._ivf_f32 is not None
        Q = X[:25] + 0.01
        want, _ = oracle.ivf_ip_f32(X, eng._labels, eng._centroids, Q, 10, 4)
        got = np.asarray(eng.search_batch(Q, k=10).indices).reshape(25, 10)
        np.testing.assert_array_equal(got, want)
        assert list(eng.search(Q[3], k=10).indices) == [int(i) for i in want[3] if i >= 0]
