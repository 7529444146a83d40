"""GPU parity: the CUDA path against the reference fixtures and the oracle.

Exact-scan results (MadhavaL2.search_exact, Metric::L2) must equal the
reference's ordered lists bit for bit.  Score metrics (cosine, SpeedEngine)
equal the oracle's ordered lists (both break ties by the lower id) and are
equivalent to the reference's lists up to the order of ties at the k-th
score, which the reference leaves unspecified (src/speed_cpu.cpp:346-347).
"""
import numpy as np
import pytest

import cases
import oracle
import winnex_madhava as wm
from helpers import load_fixture

pytestmark = pytest.mark.gpu


def _exact_engine(C, metric, k):
    cfg = wm.Config()
    cfg.dim = C.shape[1]
    cfg.k = k
    cfg.metric = metric
    e = wm.MadhavaL2(cfg)
    e.build_numpy(np.ascontiguousarray(C))
    return e


def _run_exact(C, Q, k, metric):
    e = _exact_engine(C, metric, k)
    out = np.full((len(Q), k), -1, np.int32)
    for i, q in enumerate(Q):
        r = e.search_exact(q)
        out[i, :len(r.indices)] = r.indices
        assert r.bound_violations == 0
    batch = np.array(e.search_batch(np.ascontiguousarray(Q), len(Q), k)).reshape(len(Q), k)
    np.testing.assert_array_equal(batch, out)
    return out


def _run_speed(C, Q, k, metric, batch=False):
    s = wm._native.SpeedEngine(np.ascontiguousarray(C), C.shape[1], metric)
    out = np.full((len(Q), k), -1, np.int32)
    kk = min(k, len(C))
    if batch:
        out[:, :kk] = np.array(s.search_batch(np.ascontiguousarray(Q), len(Q), k)["indices"]).reshape(len(Q), kk)
    else:
        for i, q in enumerate(Q):
            ids = s.search(q, k)["indices"]
            out[i, :len(ids)] = ids
    return out


def _check_case(C, Q, res):
    for key, want in res.items():
        k = int(key.rsplit("_k", 1)[1])
        if key.startswith("exact_l2"):
            got = _run_exact(C, Q, k, wm.Metric.L2)
            np.testing.assert_array_equal(got, want, err_msg=key)
        elif key.startswith("exact_cos"):
            got = _run_exact(C, Q, k, wm.Metric.COSINE)
            np.testing.assert_array_equal(got, oracle.cosine_exact_u8(C, Q, k)[0], err_msg=key)
            assert not oracle.equivalent_topk("exact_cos", C, Q, got, want), key
        else:
            metric = 0 if "_cos_" in key else 1
            got = _run_speed(C, Q, k, metric, batch=key.startswith("speedb"))
            kind = "speed_cos" if metric == 0 else "speed_l2"
            np.testing.assert_array_equal(got, oracle.speed_exact(C, Q, k, metric == 0)[0], err_msg=key)
            assert not oracle.equivalent_topk(kind, C, Q, got, want), key


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


@pytest.fixture(autouse=True)
def _default_options():
    wm._native.set_scan_path(0)
    yield
    wm._native.set_scan_path(0)


@pytest.mark.parametrize("name", sorted(CASES))
def test_fixture_parity(name):
    meta, res = load_fixture(name)
    C, Q = CASES[name]()
    assert cases.sha(C, Q) == meta["sha256"]
    _check_case(C, Q, res)


def test_fixture_parity_clustered():
    X, Xu = cases.case_clustered()
    _, res = load_fixture("clustered_u8")
    _check_case(Xu, Xu[:16].astype(np.float32), res)
    _, res = load_fixture("clustered_f32")
    _check_case(X, X[:16], res)


@pytest.mark.parametrize("path", [1, 2, 3])
def test_scan_paths_agree(path):
    """CUDA-core, single-SM and SM-pair tensor-core scans give identical lists."""
    C, Q = cases.case_gmm()
    wm._native.set_scan_path(path)
    got = _run_exact(C, Q, 10, wm.Metric.L2)
    _, res = load_fixture("gmm")
    np.testing.assert_array_equal(got, res["exact_l2_k10"])


def test_reference_test_semantics():
    """The reference's own test assertions, restated (tests/python/test_speed.py:43-95,
    test_python_api.py:41-73)."""
    X = cases.clustered_f32(n=20_000)
    eng = wm.build_engine(X, dim=X.shape[1], k=10, metric="cosine", speed=True)
    assert type(eng).__name__ == "MadhavaSpeed" and eng.num_vectors() == X.shape[0] and eng.built() is True
    q = X[0]
    qn = q / max(np.linalg.norm(q), 1e-12)
    s = X.astype(np.float32) @ qn
    exp = np.argsort(-s)[:10]
    assert set(eng.search(q, k=10).indices) == set(exp.tolist())
    assert list(eng.search(q, k=10).indices) == list(eng.search_exact(q, k=10).indices)
    Xu = cases.to_u8(X)
    eng = wm.build_engine(Xu, dim=Xu.shape[1], k=10, metric="l2", speed=True)
    qu = Xu[0].astype(np.float32)
    d2 = ((Xu.astype(np.float32) - qu) ** 2).sum(axis=1)
    assert list(eng.search(qu, k=10).indices) == list(np.argsort(d2, kind="stable")[:10])
    Q = X[:50]
    rb = np.array(wm.build_engine(X, dim=64, k=10, metric="cosine", speed=True).search_batch(Q, k=10, chunk=25).indices)
    assert rb.shape == (500,)
    # self is top-1 under exact L2 on a one-row corpus
    corpus = np.random.default_rng(7).integers(0, 256, size=(1, 64), dtype=np.uint8)
    e = _exact_engine(corpus, wm.Metric.L2, 10)
    assert e.search(corpus[0].astype(np.float32)).indices == [0]


def test_speed_engine_counters_with_verification():
    """build_engine(..., speed=True) with set_verify(n): the result reports
    the verified queries and their measured violations (0), and on a
    clustered u8 corpus the tensor scan's block bound settles pairs without
    forming their distance (pruned_by_bound > 0).  The reference declares
    these counters (include/winnex_madhava/speed_engine.hpp:36-41) but never
    measures them."""
    C = cases.gmm_u8(120_000, 128, 64, seed=111)
    Q = cases.gmm_u8_queries(256, 128, 64, seed_means=111, seed_q=112)
    eng = wm.build_engine(C, dim=128, k=10, metric="l2", speed=True)
    wm.set_verify(32)
    try:
        r = eng.search_batch(Q.astype(np.float32), k=10)
    finally:
        wm.set_verify(0)
    assert r.verified_queries == 32 and r.bound_violations == 0
    # Pairs settled by the block bound, over every level scanned (the sample
    # levels too), so it is compared with the pairs of all levels.
    assert r.pruned_by_bound > len(C) * len(Q) // 2
    assert r.bound_pairs == len(C) * len(Q)
    want, _ = oracle.l2_exact_u8_int(C, Q, 10)
    np.testing.assert_array_equal(np.asarray(r.indices).reshape(len(Q), 10), want)
    one = eng.search(Q[0].astype(np.float32), k=10)
    assert one.verified_queries == 0 and one.pruned_by_bound >= 0


@pytest.mark.parametrize("metric", ["l2", "cosine"])
def test_speed_engine_anchors_scan_exactly(metric):
    """speed_n_anchors / speed_nprobe are accepted and the scan stays exact,
    as in the reference on a machine with a CUDA device: enable_gpu sets
    use_gpu_ (src/speed_gpu.cu:136-160) and search / search_batch take the
    brute-force GPU top-k (src/speed_cpu.cpp:426-448) without the anchor
    cells."""
    C = cases.gmm_u8(30_000, 128, 64, seed=113)
    Q = cases.gmm_u8_queries(12, 128, 64, seed_means=113, seed_q=114).astype(np.float32)
    plain = wm.build_engine(C, dim=128, k=10, metric=metric, speed=True)
    anch = wm.build_engine(C, dim=128, k=10, metric=metric, speed=True, speed_n_anchors=16, speed_nprobe=2)
    got = np.asarray(anch.search_batch(Q, k=10).indices).reshape(len(Q), 10)
    np.testing.assert_array_equal(got, np.asarray(plain.search_batch(Q, k=10).indices).reshape(len(Q), 10))
    want, _ = oracle.speed_exact(C, Q, 10, metric == "cosine")
    np.testing.assert_array_equal(got, want)
    for i in (0, 5):
        assert list(anch.search(Q[i], k=10).indices) == list(want[i])


def test_overflow_rerun_keeps_results_exact():
    """Tiny candidate lists force the overflow / tighter-threshold reruns."""
    C, Q = cases.case_dups()
    _, res = load_fixture("dups")
    lib = wm._native
    try:
        from helpers import capi
        L = capi()
        assert L.mdh_set_candidate_cap_limit(64) == 0
        np.testing.assert_array_equal(_run_exact(C, Q, 10, wm.Metric.L2), res["exact_l2_k10"])
        np.testing.assert_array_equal(_run_exact(C, Q, 64, wm.Metric.L2), res["exact_l2_k64"])
        Cq, Qq = cases.case_quickstart()
        _, rq = load_fixture("quickstart")
        np.testing.assert_array_equal(_run_exact(Cq, Qq, 10, wm.Metric.L2), rq["exact_l2_k10"])
    finally:
        L.mdh_set_candidate_cap_limit(0)
    assert lib is not None


def test_all_equal_rows_and_edge_shapes():
    C = np.full((3000, 32), 7, np.uint8)
    ids = _run_exact(C, np.full((2, 32), 7, np.float32), 16, wm.Metric.L2)
    np.testing.assert_array_equal(ids, [list(range(16))] * 2)
    # k in (16, 128] with every key tied: more than 1,024 entries share the
    # bound, so the selection takes the k smallest (key, id) one at a time.
    for k in (64, 128):
        ids = _run_exact(C, np.full((2, 32), 7, np.float32), k, wm.Metric.L2)
        np.testing.assert_array_equal(ids, [list(range(k))] * 2)
    # k > n and k == n
    C = np.random.default_rng(0).integers(0, 256, (6, 16), dtype=np.uint8)
    Q = C[:2].astype(np.float32)
    ids = _run_exact(C, Q, 9, wm.Metric.L2)
    np.testing.assert_array_equal(ids[:, 6:], -1)
    np.testing.assert_array_equal(ids, oracle.l2_exact_u8(C, Q, 9)[0])
    # a single query with an all-zero corpus row set and large ids
    C = np.zeros((70_000, 128), np.uint8)
    C[-1] = 255
    ids = _run_exact(C, np.full((1, 128), 255, np.float32), 3, wm.Metric.L2)
    np.testing.assert_array_equal(ids, [[69_999, 0, 1]])
