"""GPU audits and commitments against the oracle.

Replaces MadhavaL2::search_audited / audit_json / search_with_commitment
(src/winnex_madhava.cpp:1258-1591); the checks follow the reference's own
tests (tests/python/test_audit_certificate.py, test_audit_commitment.py):
excluded rows are strictly worse than the k-th result, the certificate covers
the returned top k, max_sample is honoured, the commitment's count equals the
certificate's, and both are deterministic.  On this exact engine the oracle
pins every number: the top k, the threshold, the rows strictly worse than it
and the nearest of them in (distance, id) order.
"""
import ctypes
import json

import numpy as np
import pytest

import cases
from helpers import Audit, Stats, capi, ptr

pytestmark = pytest.mark.gpu


def _oracle_audit(C, q, k, m):
    """(top ids, top dists, threshold, rows within, record ids, record dists)
    from exact int64 distances ordered by (distance, id)."""
    Ci = C.astype(np.int64)
    d = (Ci * Ci).sum(1) + int((q.astype(np.int64) ** 2).sum()) - 2 * (Ci @ q.astype(np.int64))
    order = np.lexsort((np.arange(len(C)), d))
    kk = min(k, len(C))
    T = d[order[kk - 1]]
    rest = order[kk:][d[order[kk:]] > T][:m]
    return order[:kk], d[order[:kk]], T, int((d <= T).sum()), rest, d[rest]


def _index(L, C, devices=None):
    h = ctypes.c_void_p()
    dev = np.asarray(devices, np.int32) if devices else None
    st = L.mdh_index_create_u8(ptr(C), C.shape[0], C.shape[1], 1, ptr(dev), len(devices or []), 0, ctypes.byref(h))
    assert st == 0, L.mdh_last_error()
    return h


def _audit_u8(L, h, Q, k, m):
    nq = len(Q)
    ids = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.int32)
    rid = np.empty((nq, max(m, 1)), np.int32)
    rdist = np.empty((nq, max(m, 1)), np.int32)
    aud = (Audit * nq)()
    st = Stats()
    s = L.mdh_audit_u8(h, ptr(Q), nq, k, m, ptr(ids), ptr(dist), ptr(rid), ptr(rdist), aud, ctypes.byref(st))
    assert s == 0, L.mdh_last_error()
    return ids, dist, rid, rdist, aud, st


@pytest.fixture(scope="module")
def gmm():
    C = cases.gmm_u8(60_000, 128, 64, seed=101)
    Q = cases.gmm_u8_queries(6, 128, 64, seed_means=101, seed_q=102)
    return C, Q


@pytest.mark.parametrize("k,m", [(1, 0), (10, 5), (100, 50)])
def test_audit_u8_matches_oracle(gmm, k, m):
    L = capi()
    C, Q = gmm
    h = _index(L, C)
    ids, dist, rid, rdist, aud, st = _audit_u8(L, h, Q, k, m)
    for i, q in enumerate(Q):
        top, topd, T, within, rest, restd = _oracle_audit(C, q, k, m)
        a = aud[i]
        np.testing.assert_array_equal(ids[i], top)
        np.testing.assert_array_equal(dist[i], topd)
        assert a.threshold == T and a.rows == len(C) and a.within == within
        assert a.excluded == len(C) - within and a.violations == 0
        assert a.n_records == len(rest)
        np.testing.assert_array_equal(rid[i, :a.n_records], rest)
        np.testing.assert_array_equal(rdist[i, :a.n_records], restd)
        # The tensor scan's block bound settles most of the clustered rows.
        assert 0 < a.excluded_by_bound <= a.excluded
    assert st.bound_violations == 0 and st.verified_queries == len(Q)
    assert L.mdh_index_destroy(h) == 0


def test_audit_ties_at_the_threshold():
    """3,000 rows at distance 0 from the query: the threshold is 0, all 3,000
    are within it (only k are returned), and the records start after them."""
    L = capi()
    rng = np.random.default_rng(103)
    C = rng.integers(0, 256, (20_000, 128), dtype=np.uint8)
    C[5_000:8_000] = 7
    q = np.full((1, 128), 7, np.uint8)
    h = _index(L, C)
    ids, dist, rid, rdist, aud, _ = _audit_u8(L, h, q, 10, 20)
    top, topd, T, within, rest, restd = _oracle_audit(C, q[0], 10, 20)
    assert T == 0 and within == 3_000
    np.testing.assert_array_equal(ids[0], top)
    assert aud[0].within == 3_000 and aud[0].excluded == len(C) - 3_000
    np.testing.assert_array_equal(rid[0, :aud[0].n_records], rest)
    np.testing.assert_array_equal(rdist[0, :aud[0].n_records], restd)
    assert L.mdh_index_destroy(h) == 0


def test_audit_two_shards_agree(gmm):
    """Rows split over two shards (one GPU): the audit pass sums the shards'
    counts against the merged threshold."""
    L = capi()
    C, Q = gmm
    h1 = _index(L, C)
    h2 = _index(L, C, [0, 0])
    a1 = _audit_u8(L, h1, Q, 10, 20)
    a2 = _audit_u8(L, h2, Q, 10, 20)
    for x, y in zip(a1[:4], a2[:4]):
        np.testing.assert_array_equal(x, y)
    for i in range(len(Q)):
        for f in ("within", "excluded", "threshold", "n_records"):
            assert getattr(a1[4][i], f) == getattr(a2[4][i], f), f
        # Each shard sorts its own rows by norm, so the 64-row blocks (and the
        # rows their bound settles) differ between the two layouts.
        for a in (a1[4][i], a2[4][i]):
            assert 0 < a.excluded_by_bound <= a.excluded
    assert L.mdh_index_destroy(h1) == 0 and L.mdh_index_destroy(h2) == 0


def test_audit_cosine_index_matches_oracle():
    """A u8 index ranked by MadhavaL2's cosine score, float queries
    (mdh_audit_f32): the threshold is the k-th score, `within` counts the rows
    scoring at least that, and the records are the next rows by (score
    descending, id) -- all from the oracle's full ranking."""
    import oracle

    L = capi()
    rng = np.random.default_rng(107)
    C = rng.integers(0, 256, (4_000, 64), dtype=np.uint8)
    Q = (rng.random((3, 64)) * 200).astype(np.float32)
    h = ctypes.c_void_p()
    assert L.mdh_index_create_u8(ptr(C), len(C), 64, 0, None, 0, 0, ctypes.byref(h)) == 0, L.mdh_last_error()
    k, m = 10, 25
    ids = np.empty((3, k), np.int32)
    val = np.empty((3, k), np.float32)
    rid = np.empty((3, m), np.int32)
    rval = np.empty((3, m), np.float32)
    aud = (Audit * 3)()
    st = L.mdh_audit_f32(h, ptr(Q), 3, k, m, ptr(ids), ptr(val), ptr(rid), ptr(rval), aud, None)
    assert st == 0, L.mdh_last_error()
    all_ids, all_sc = oracle.cosine_exact_u8(C, Q, len(C))
    for i in range(3):
        T = all_sc[i, k - 1]
        np.testing.assert_array_equal(ids[i], all_ids[i, :k])
        np.testing.assert_array_equal(val[i], all_sc[i, :k])
        within = int((all_sc[i] >= T).sum())
        assert aud[i].threshold == T and aud[i].within == within and aud[i].excluded == len(C) - within
        assert aud[i].excluded_by_bound == -1 and aud[i].violations == 0
        assert aud[i].n_records == m
        np.testing.assert_array_equal(rid[i], all_ids[i, within:within + m])
        np.testing.assert_array_equal(rval[i], all_sc[i, within:within + m])
    assert L.mdh_index_destroy(h) == 0


def test_audit_edges():
    """k at least n (every row returned, none excluded), no queries, and no
    records requested."""
    L = capi()
    rng = np.random.default_rng(109)
    C = rng.integers(0, 256, (100, 128), dtype=np.uint8)
    q = rng.integers(0, 256, (2, 128), dtype=np.uint8)
    h = _index(L, C)
    ids, dist, rid, rdist, aud, _ = _audit_u8(L, h, q, 150, 5)
    for i in range(2):
        top, topd, T, within, _, _ = _oracle_audit(C, q[i], 150, 0)
        np.testing.assert_array_equal(ids[i, :100], top)
        assert (ids[i, 100:] == -1).all()
        assert aud[i].within == 100 and aud[i].excluded == 0 and aud[i].n_records == 0 and aud[i].threshold == T
    ids, dist, rid, rdist, aud, _ = _audit_u8(L, h, q, 10, 0)
    top, topd, T, within, _, _ = _oracle_audit(C, q[0], 10, 0)
    np.testing.assert_array_equal(ids[0], top)
    assert aud[0].n_records == 0 and aud[0].excluded == 100 - within
    st = Stats()
    assert L.mdh_audit_u8(h, ptr(q), 0, 10, 5, None, None, None, None, None, ctypes.byref(st)) == 0
    assert L.mdh_index_destroy(h) == 0


def test_audit_rejects_bad_arguments(gmm):
    L = capi()
    C, Q = gmm
    h = _index(L, C)
    aud = (Audit * 1)()
    ids = np.empty(10, np.int32)
    assert L.mdh_audit_u8(h, ptr(Q[:1]), 1, 0, 5, ptr(ids), None, None, None, aud, None) != 0
    assert L.mdh_audit_u8(h, ptr(Q[:1]), 1, 10, 5, ptr(ids), None, None, None, aud, None) != 0  # no record ids
    assert b"record" in L.mdh_last_error()
    assert L.mdh_index_destroy(h) == 0


# ---------------------------------------------------------------- the facade
@pytest.fixture(scope="module")
def l2_engine():
    """The reference's L2 audit engine (test_audit_certificate.py:25-31)."""
    import winnex_madhava as wm

    rng = np.random.default_rng(42)
    corpus = rng.integers(0, 256, size=(5000, 128)).astype(np.uint8)
    eng = wm.build_engine(corpus, dim=128, metric="l2", quant="int8", stage1_dim=64, stage2_dim=0, k=10,
                          k1_fraction=0.10)
    return eng, corpus


def test_facade_search_audited_l2(l2_engine):
    eng, C = l2_engine
    for q in (np.zeros(128, np.float32), (C[17] // 2 + 3).astype(np.float32)):
        r = eng.search_audited(q, k=10, max_audit_records=500)
        top, topd, T, within, rest, restd = _oracle_audit(C, q.astype(np.uint8), 10, 500)
        assert r["indices"] == list(top) and r["bound_violations"] == 0
        assert r["audit_candidates"] == len(C) and r["audit_excluded"] == len(C) - within
        required = {"doc_id", "true_cosine", "projected_cosine", "residual_norm", "upper_bound", "threshold",
                    "excluded", "stage"}
        recs = r["audit"]
        assert all(required <= set(x) for x in recs)
        excl = [x for x in recs if x["excluded"]]
        assert [x["doc_id"] for x in excl] == list(rest)
        assert all(x["true_cosine"] > x["threshold"] for x in excl)  # L2: a larger distance is outside
        assert {x["doc_id"] for x in recs if x["stage"] == "in_topk"} == set(r["indices"])
        assert r["audit_threshold"] == T
        r2 = eng.search_audited(q, k=10, max_audit_records=500)
        assert [x["doc_id"] for x in r2["audit"]] == [x["doc_id"] for x in recs]
    # Full coverage: every excluded row gets a record.
    r = eng.search_audited(np.zeros(128, np.float32), k=10, max_audit_records=len(C))
    assert len([x for x in r["audit"] if x["excluded"]]) == r["audit_excluded"]


def test_facade_audit_json(l2_engine):
    eng, _ = l2_engine
    data = json.loads(eng.audit_json(np.zeros(128, np.float32), k=10, max_audit_records=50))
    assert "audit_trail" in data and len(data["results"]) == 10
    assert data["bound_violations"] == 0 and len(data["audit_trail"]) == 60


def test_facade_commitment(l2_engine):
    eng, C = l2_engine
    q = C[3].astype(np.float32)
    c = eng.search_with_commitment(q, k=10, max_sample=5)
    assert c["total_excluded_count"] > 0 and len(c["sampled_records"]) == 5
    assert all(s["excluded"] for s in c["sampled_records"])
    c50 = eng.search_with_commitment(q, k=10, max_sample=50)
    ar = eng.search_audited(q, k=10, max_audit_records=50)
    assert c50["total_excluded_count"] == ar["audit_excluded"]
    assert [s["doc_id"] for s in c50["sampled_records"]] == [x["doc_id"] for x in ar["audit"] if x["excluded"]]
    c2 = eng.search_with_commitment(q, k=10, max_sample=5)
    assert [s["doc_id"] for s in c["sampled_records"]] == [s["doc_id"] for s in c2["sampled_records"]]
    top, topd, T, _, _, _ = _oracle_audit(C, C[3], 10, 0)
    assert c["global_threshold"] == T and c["bound_violations"] == 0 and c["indices"] == list(top)
    assert all(s["upper_bound"] > c["global_threshold"] for s in c50["sampled_records"])


def test_facade_audit_cosine():
    """A cosine engine over re-quantized float rows, float queries: the
    excluded records score strictly below the threshold, in descending score,
    and with full coverage they are every excluded row."""
    import winnex_madhava as wm

    rng = np.random.default_rng(42)
    corpus = rng.standard_normal((3000, 64)).astype(np.float32)
    corpus /= np.linalg.norm(corpus, axis=1, keepdims=True)
    eng = wm.build_engine(corpus, dim=64, metric="cosine", quant="int8", k=10)
    q = corpus[5] + 0.1 * rng.standard_normal(64).astype(np.float32)
    r = eng.search_audited(q, k=10, max_audit_records=len(corpus))
    assert r["indices"] == list(eng.search_exact(q).indices)
    excl = [x for x in r["audit"] if x["excluded"]]
    vals = [x["true_cosine"] for x in excl]
    assert all(v < r["audit_threshold"] for v in vals) and vals == sorted(vals, reverse=True)
    assert len(excl) == r["audit_excluded"] and r["bound_violations"] == 0
    assert r["audit_excluded_by_bound"] == -1  # no block bound on the float path
