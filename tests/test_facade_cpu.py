"""Host-side checks of the drop-in Python facade (no GPU needed)."""
import os
import struct
import tempfile

import numpy as np
import pytest

import oracle
import winnex_madhava as wm


def test_public_names_match_reference_facade():
    for name in ("Config", "SearchResult", "MadhavaL2", "MadHybrid", "MadhavaSpeed", "Metric", "QuantMode",
                 "BasisMode", "recall_at_k", "ndcg_at_k", "read_bigann_groundtruth", "build_engine", "retrieve",
                 "benchmark_vs_groundtruth"):
        assert hasattr(wm, name), name
    assert int(wm.Metric.COSINE) == 0 and int(wm.Metric.L2) == 1


def test_config_defaults_match_reference():
    ours = wm.Config()
    R = oracle.reference_module()
    if R is None:
        pytest.skip("reference module not built")
    ref = R.Config()
    for f in ("dim", "seed", "pca_sample", "stage1_dim", "stage2_dim", "k", "k1_fraction", "k2_fraction", "k1_min",
              "k2_min", "k2_max", "modulation", "postfilter", "normalize_input", "early_exit", "n_threads"):
        assert getattr(ours, f) == getattr(ref, f), f
    assert int(ours.metric) == int(ref.metric)
    assert int(ours.quant) == int(ref.quant)
    assert int(ours.basis) == int(ref.basis)


def test_metric_helpers_match_reference():
    R = oracle.reference_module()
    rng = np.random.default_rng(0)
    for _ in range(50):
        gt = rng.choice(50, size=rng.integers(0, 12), replace=False).tolist()
        res = rng.choice(50, size=rng.integers(0, 12), replace=False).tolist()
        k = int(rng.integers(1, 12))
        r, n = wm.recall_at_k(res, gt, k), wm.ndcg_at_k(res, gt, k)
        if R is not None:
            assert r == R.recall_at_k(res, gt, k)
            assert n == pytest.approx(R.ndcg_at_k(res, gt, k), abs=0, rel=1e-15)
    assert wm.recall_at_k([5, 7, 100, 200, 300], [5, 7], 5) == 1.0
    assert wm.recall_at_k([], [5, 7, 9], 3) == 0.0


def test_l2_sq():
    # The reference binds l2_sq(const uint8_t*, const float*, int) with raw
    # pointers (bindings/py_module.cpp:344), which pybind11 exposes as scalar
    # arguments; ours takes arrays.  Integral inputs are exact; float inputs
    # follow the scalar FMA chain to float32 rounding.
    rng = np.random.default_rng(1)
    for d in (7, 64, 128, 130):
        v = rng.integers(0, 256, d, dtype=np.uint8)
        qi = rng.integers(0, 256, d).astype(np.float32)
        assert wm.l2_sq(v, qi, d) == float(((v.astype(np.int64) - qi.astype(np.int64)) ** 2).sum())
        q = (rng.random(d) * 255).astype(np.float32)
        want = float(((v.astype(np.float64) - q.astype(np.float64)) ** 2).sum())
        assert wm.l2_sq(v, q, d) == pytest.approx(want, rel=1e-5)


def test_read_bigann_groundtruth():
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "gt.bin")
        ids = np.arange(6, dtype=np.int32).reshape(2, 3)
        with open(p, "wb") as f:
            f.write(struct.pack("ii", 2, 3))
            for i in range(2):
                f.write(ids[i].tobytes())
                f.write(np.zeros(3, np.float32).tobytes())
        assert wm.read_bigann_groundtruth(p, 0) == [[0, 1, 2], [3, 4, 5]]
        assert wm.read_bigann_groundtruth(p, 1) == [[0, 1, 2]]
        assert wm.read_bigann_groundtruth(os.path.join(td, "missing"), 1) == []


def test_engines_refuse_to_run_without_gpu():
    if wm._native.device_count() > 0:
        pytest.skip("a GPU is present")
    C = np.zeros((16, 8), np.uint8)
    with pytest.raises(RuntimeError, match="no CUDA device"):
        wm.build_engine(C, dim=8, metric="l2")
    with pytest.raises(RuntimeError, match="no CUDA device"):
        wm.build_engine(C, dim=8, metric="l2", speed=True)


def test_bound_engine_only_features_raise():
    e = wm.MadhavaL2(wm.Config())
    # Like the reference, an unbuilt engine saves nothing and a missing file
    # does not load.
    assert e.save_index("/nonexistent-dir/x.idx") is False
    assert e.load_index("/nonexistent-dir/x.idx") is False and e.built() is False
    with pytest.raises(NotImplementedError):
        e.basis1()
    # An unbuilt engine audits nothing (src/winnex_madhava.cpp:1266).
    r = e.search_audited(np.zeros(128, np.float32))
    assert r["indices"] == [] and r["audit"] == [] and r["audit_excluded"] == 0
    assert e.search_with_commitment(np.zeros(128, np.float32))["sampled_records"] == []
    # An unbuilt engine returns an empty result like the reference.
    assert e.search(np.zeros(128, np.float32)).indices == []
    with pytest.raises(RuntimeError, match="query must be float32 of length dim"):
        e.search(np.zeros(3, np.float32))
