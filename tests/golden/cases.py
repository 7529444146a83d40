"""Seeded inputs for the golden fixtures (shared by make_golden.py and the tests).

Each case regenerates its corpus and queries from fixed seeds; the fixture
stores a sha256 of the generated arrays so a change in a random generator
is detected instead of silently comparing different data.  Shapes follow the
reference's own tests (tests/python/test_python_api.py:12-26, :58-73;
tests/python/test_speed.py:24-30; tests/test_winnex_madhava.cpp:158-191 uses
d = 48) and the quickstart (examples/quickstart.py:19-24).
"""
from __future__ import annotations

import hashlib

import numpy as np


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def clustered_f32(n=20_000, d=64, n_clusters=16, seed=7):
    """Normalized clustered float corpus (the shape of test_speed.py's fixture)."""
    rng = np.random.RandomState(seed)
    centers = rng.randn(n_clusters, d).astype(np.float32) * 5.0
    labels = rng.randint(0, n_clusters, n)
    X = centers[labels] + rng.randn(n, d).astype(np.float32) * 0.5
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    return X.astype(np.float32)


def to_u8(X):
    """Min-max quantization to u8 used by the reference tests for their L2 corpus."""
    Xu = (X - X.min()) / (X.max() - X.min()) * 255
    return Xu.astype(np.uint8)


def gmm_u8(n, d, comps, seed, chunk=1_000_000):
    """Clipped Gaussian-mixture u8 rows: means U[0,60], per-dim std 15, rounded and clipped."""
    rng = np.random.default_rng(seed)
    means = rng.uniform(0, 60, size=(comps, d))
    out = np.empty((n, d), np.uint8)
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        lab = rng.integers(0, comps, size=m)
        out[s:s + m] = np.clip(np.rint(means[lab] + rng.normal(0, 15, size=(m, d))), 0, 255)
    return out


def gmm_u8_queries(nq, d, comps, seed_means, seed_q):
    """Queries from the same mixture means as gmm_u8(seed=seed_means), fresh labels/noise."""
    rng_m = np.random.default_rng(seed_means)
    means = rng_m.uniform(0, 60, size=(comps, d))
    rng = np.random.default_rng(seed_q)
    lab = rng.integers(0, comps, size=nq)
    return np.clip(np.rint(means[lab] + rng.normal(0, 15, size=(nq, d))), 0, 255).astype(np.uint8)


def case_api():
    corpus = np.random.default_rng(42).integers(0, 256, size=(5000, 64), dtype=np.uint8)
    q0 = np.random.default_rng(0).integers(0, 256, size=(1, 64), dtype=np.uint8)
    qs = np.random.default_rng(1).integers(0, 256, size=(15, 64), dtype=np.uint8)
    return corpus, np.concatenate([q0, qs]).astype(np.float32)


def case_clustered():
    X = clustered_f32()
    return X, to_u8(X)


def case_quickstart():
    corpus = np.random.default_rng(0).integers(0, 256, size=(100_000, 128), dtype=np.uint8)
    qidx = np.random.default_rng(7).choice(100_000, 100, replace=False)
    return corpus, corpus[qidx].astype(np.float32)


def case_gmm():
    corpus = gmm_u8(200_000, 128, 256, seed=1)
    queries = gmm_u8_queries(48, 128, 256, seed_means=1, seed_q=2).astype(np.float32)
    return corpus, queries


def case_float_queries():
    corpus = np.random.default_rng(5).integers(0, 256, size=(3000, 128), dtype=np.uint8)
    queries = (np.random.default_rng(6).random((16, 128)) * 255).astype(np.float32)
    return corpus, queries


def case_dups():
    rng = np.random.default_rng(3)
    base = rng.integers(0, 256, size=(40, 64), dtype=np.uint8)
    corpus = base[rng.integers(0, 40, size=2000)]
    queries = np.concatenate([base[:8], rng.integers(0, 256, size=(8, 64), dtype=np.uint8)]).astype(np.float32)
    return corpus, queries


def case_dim(d, n=4000, seed=11):
    rng = np.random.default_rng(seed + d)
    corpus = rng.integers(0, 256, size=(n, d), dtype=np.uint8)
    queries = rng.integers(0, 256, size=(8, d), dtype=np.uint8).astype(np.float32)
    return corpus, queries


def case_small():
    rng = np.random.default_rng(9)
    corpus = rng.integers(0, 256, size=(5, 32), dtype=np.uint8)
    queries = rng.integers(0, 256, size=(3, 32), dtype=np.uint8).astype(np.float32)
    return corpus, queries


def case_hybrid():
    """MadHybrid (uint8, L2): 24,000 x 64 clipped-GMM rows, 96 queries from the
    same mixture; the reference clusters them into nlist=16 cells."""
    C = gmm_u8(24_000, 64, 32, seed=71)
    Q = gmm_u8_queries(96, 64, 32, seed_means=71, seed_q=72)
    return C, Q


HYBRID = {"nlist": 16, "nprobe": 4, "seed": 42}


def case_f32_corpus():
    X = clustered_f32(n=12_000, d=96, n_clusters=24, seed=13)
    rng = np.random.default_rng(14)
    Q = np.concatenate([X[:8], rng.standard_normal((8, 96)).astype(np.float32)])
    return X, Q


def cos_gmm_f32(n, d, comps, seed, stream=0):
    """Row-normalized isotropic Gaussian mixture: unit-normalized random means,
    component std 0.3 (the float cosine workload's generator); `stream`
    selects an independent draw of rows from the same means."""
    rng = np.random.default_rng(seed)
    means = rng.standard_normal((comps, d))
    means /= np.linalg.norm(means, axis=1, keepdims=True)
    r = np.random.default_rng([seed, stream])
    lab = r.integers(0, comps, n)
    X = means[lab] + r.normal(0, 0.3, (n, d))
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    return X.astype(np.float32)


DIMS = (48, 7, 200, 300)
