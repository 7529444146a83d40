"""The oracle (CPU restatement) against the golden fixtures made by the reference itself.

Pins the oracle before any GPU result is compared with it: every fixture
was produced by the reference's own compiled CPU code (make_golden.py), and
the oracle must reproduce it -- ordered lists for MadhavaL2.search_exact
(ties go to the lower index), id sets for SpeedEngine (whose tie order is
unspecified, src/speed_cpu.cpp:346-347).
"""
import numpy as np
import pytest

import cases
import oracle
from helpers import load_fixture


def _check_sha(meta, *arrays):
    assert cases.sha(*arrays) == meta["sha256"], "input generator drifted from the fixture"


def _cmp_exact(got, want):
    assert got.shape == want.shape
    np.testing.assert_array_equal(got, want)


def _cmp_sets(got, want):
    assert got.shape == want.shape
    for i in range(len(got)):
        assert sorted(got[i].tolist()) == sorted(want[i].tolist()), f"query {i}"


def _k(key):
    return int(key.rsplit("_k", 1)[1])


def _run_oracle(key, C, Q):
    k = _k(key)
    if key.startswith("exact_l2"):
        return oracle.l2_exact_u8(C, Q, k)[0]
    if key.startswith("exact_cos"):
        return oracle.cosine_exact_u8(C, Q, k)[0]
    cosine = "_cos_" in key
    return oracle.speed_exact(C, Q, k, cosine)[0]


CASES = {
    "api": cases.case_api,
    "quickstart": cases.case_quickstart,
    "gmm": cases.case_gmm,
    "float_queries": cases.case_float_queries,
    "dups": cases.case_dups,
    "small": cases.case_small,
    "f32_corpus": cases.case_f32_corpus,
}
for _d in cases.DIMS:
    CASES[f"dim{_d}"] = (lambda d=_d: cases.case_dim(d))


def _cmp_speed(key, C, Q, got, want):
    kind = "speed_cos" if "_cos_" in key else "speed_l2"
    bad = oracle.equivalent_topk(kind, C, Q, got, want)
    assert not bad, f"{key}: queries {bad} differ beyond tie order"


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_fixture(name):
    meta, res = load_fixture(name)
    C, Q = CASES[name]()
    _check_sha(meta, C, Q)
    for key, want in res.items():
        got = _run_oracle(key, C, Q)
        if key.startswith("exact"):
            _cmp_exact(got, want)
        else:
            _cmp_speed(key, C, Q, got, want)


def test_oracle_matches_reference_fixture_clustered():
    X, Xu = cases.case_clustered()
    meta, res = load_fixture("clustered_u8")
    _check_sha(meta, Xu, Xu[:16].astype(np.float32))
    Qu = Xu[:16].astype(np.float32)
    for key, want in res.items():
        got = _run_oracle(key, Xu, Qu)
        if key.startswith("exact"):
            _cmp_exact(got, want)
        else:
            _cmp_speed(key, Xu, Qu, got, want)
    meta, res = load_fixture("clustered_f32")
    _check_sha(meta, X, X[:16])
    for key, want in res.items():
        _cmp_speed(key, X, X[:16], _run_oracle(key, X, X[:16]), want)


def test_integer_oracle_agrees_with_float_oracle():
    """For u8 queries the int64 ranking equals the reference float ranking."""
    C, Q = cases.case_api()
    a, da = oracle.l2_exact_u8(C, Q, 32)
    b, db = oracle.l2_exact_u8_int(C, Q.astype(np.uint8), 32)
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(da.astype(np.int64), db)


def test_oracle_brute_force_numpy():
    """Cross-check the oracle with an independent numpy lexsort (dist, id)."""
    C, Q = cases.case_dups()
    ids, dist = oracle.l2_exact_u8_int(C, Q.astype(np.uint8), 64)
    Ci = C.astype(np.int64)
    for i, q in enumerate(Q.astype(np.int64)):
        d = ((Ci - q) ** 2).sum(1)
        o = np.lexsort((np.arange(len(d)), d))[:64]
        np.testing.assert_array_equal(ids[i], o)
        np.testing.assert_array_equal(dist[i], d[o])


def test_oracle_edge_cases():
    C = np.zeros((10, 16), np.uint8)  # all rows identical: ties everywhere
    ids, dist = oracle.l2_exact_u8_int(C, np.zeros((2, 16), np.uint8), 4)
    np.testing.assert_array_equal(ids, [[0, 1, 2, 3]] * 2)
    ids, _ = oracle.l2_exact_u8(C[:3], np.zeros((1, 16), np.float32), 5)  # k > n
    np.testing.assert_array_equal(ids, [[0, 1, 2, -1, -1]])
    ids, _ = oracle.l2_exact_u8(C[:0], np.zeros((1, 16), np.float32), 3)  # empty corpus
    np.testing.assert_array_equal(ids, [[-1, -1, -1]])


def test_ivf_routing_matches_reference():
    """The routing restatement (fp64, fixed order, lower cell id on ties) picks
    the reference's cells, `argsort(-(centroids @ q))[:nprobe]`
    (python/winnex_madhava/__init__.py:631-632), on the reference's own
    MiniBatchKMeans centroids; positions where the reference's float32 sums
    leave two cells within rounding of each other are the only exemptions."""
    meta, res = load_fixture("hybrid")
    C, Q = cases.case_hybrid()
    assert cases.sha(C, Q) == meta["sha256"]
    got = oracle.ivf_route(res["centroids"], Q, cases.HYBRID["nprobe"])
    want = res["route_ref"]
    sims = res["sims64"]
    differ = 0
    for i in range(len(Q)):
        if (got[i] == want[i]).all():
            continue
        s = np.sort(sims[i])[::-1]
        gaps = np.abs(np.diff(s[: cases.HYBRID["nprobe"] + 1]))
        assert gaps.min() < 1e-3 * abs(s[0]), (i, got[i], want[i])
        differ += 1
    assert differ <= 2
    # every row has a cell, every cell index is valid
    assert res["labels"].min() >= 0 and res["labels"].max() < cases.HYBRID["nlist"]


def test_ivf_exact_oracle_full_probe_is_brute_force():
    """Probing every cell makes the IVF oracle the plain exact search."""
    meta, res = load_fixture("hybrid")
    C, Q = cases.case_hybrid()
    ids, dist = oracle.ivf_exact(C, res["labels"], res["centroids"], Q[:12], 10, cases.HYBRID["nlist"])
    want_ids, want_d = oracle.l2_exact_u8_int(C, Q[:12], 10)
    np.testing.assert_array_equal(ids, want_ids)
    np.testing.assert_array_equal(dist, want_d)


def test_sliced_topk_oracle_matches_int_oracle():
    """oracle.L2TopK (one pass over the rows for all queries, fed in slices)
    ranks exactly like the per-query int64 oracle, ties and short corpora
    included."""
    C = cases.gmm_u8(60_000, 128, 64, seed=21)
    Q = cases.gmm_u8_queries(40, 128, 64, seed_means=21, seed_q=22)
    for corpus, q, k, sl in ((C, Q, 10, 7_001), (np.repeat(C[:500], 5, axis=0), Q[:9], 37, 777),
                             (C[:20], Q[:3], 30, 7)):
        a = oracle.l2_exact_u8_int(corpus, q, k)
        b = oracle.l2_topk_u8(corpus, q, k, slice_rows=sl)
        np.testing.assert_array_equal(a[0], b[0])
        np.testing.assert_array_equal(a[1], b[1])


def test_ivf_inner_product_oracle_full_probe_is_brute_force():
    """ivf_exact(metric="ip") probing every cell is the exact inner-product
    top-k by (q.v descending, id)."""
    C = cases.gmm_u8(3_000, 32, 8, seed=81)
    Q = cases.gmm_u8_queries(12, 32, 8, seed_means=81, seed_q=82)
    rng = np.random.default_rng(83)
    cen = rng.uniform(0, 60, (6, 32)).astype(np.float32)
    labels = rng.integers(0, 6, len(C))
    ids, dots = oracle.ivf_exact(C, labels, cen, Q, 7, 6, metric="ip")
    full = C.astype(np.int64) @ Q.astype(np.int64).T
    for i in range(len(Q)):
        order = np.lexsort((np.arange(len(C)), -full[:, i]))[:7]
        np.testing.assert_array_equal(ids[i], order)
        np.testing.assert_array_equal(dots[i], full[order, i])
