"""Oracle bindings -- TEST INFRASTRUCTURE ONLY.

ctypes wrappers over ``oracle/liboracle.so`` (the C restatement in
``exact_scan.c``) plus a loader for the compiled reference module in
``oracle/_ref/`` when it was built.  Only ``tests/``, ``__graft_entry__.smoke``
and ``bench.py``'s CPU-baseline leg import this module; the product package
never does.

Each wrapper names the reference function it restates:

* :func:`l2_exact_u8`      -- ``MadhavaL2::search_exact``, Metric::L2
  (src/winnex_madhava.cpp:1224-1246, l2_sq_avx :119-146)
* :func:`cosine_exact_u8`  -- ``MadhavaL2::search_exact``, Metric::Cosine on a
  u8 base (src/winnex_madhava.cpp:714-763)
* :func:`speed_exact_u8` / :func:`speed_exact_f32` -- ``SpeedEngine`` CPU scan
  (src/speed_cpu.cpp:81-144 construction, :271-398 search)
* :func:`l2_exact_u8_int`  -- the same L2 ranking in int64 for u8 queries.
"""
from __future__ import annotations

import ctypes
import importlib.util
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
# Where the reference's sources lie (the one setting for every script that
# reads them: this module, oracle/Makefile, tests/golden/make_golden.py and
# __graft_entry__.build); override with MDH_REFERENCE_DIR.
REFERENCE_DIR = os.environ.get("MDH_REFERENCE_DIR", "/root/reference")
REF_DIR = os.path.join(HERE, "_ref")

_lib = None


def build() -> None:
    """Compile liboracle.so (and the reference module when its sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    if os.path.isdir(os.path.join(REFERENCE_DIR, "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        i64, i32, f32 = ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.oracle_l2_exact_u8.argtypes = [P, i64, i32, P, i32, i32, P, P]
        L.oracle_l2_exact_u8_int.argtypes = [P, i64, i32, P, i32, i32, P, P]
        L.oracle_l2_topk_u8_update.argtypes = [P, i64, i32, i64, P, i32, i32, P, P]
        L.oracle_cosine_exact_u8.argtypes = [P, i64, i32, P, i32, i32, P, P]
        L.oracle_speed_exact.argtypes = [P, P, i64, i32, i32, P, i32, i32, P, P]
        L.oracle_speed_prepare_u8.argtypes = [P, i64, i32, i32, P, P]
        L.oracle_speed_prepare_f32.argtypes = [P, i64, i32, i32, P, P]
        L.oracle_l2_sq_u8.argtypes = [P, P, i32]
        L.oracle_l2_sq_u8.restype = f32
        L.oracle_num_threads.restype = i32
        L.oracle_score_ids.argtypes = [i32, i32, P, P, P, i32, P, P, i32, P]
        L.oracle_ivf_route.argtypes = [P, i32, i32, P, i32, i32, P]
        L.oracle_ivf_route_f32.argtypes = [P, i32, i32, P, i32, i32, P]
        L.oracle_ivf_ip_f32.argtypes = [P, i64, i32, P, P, i32, P, i32, i32, P, P]
        L.oracle_score_ids.restype = None
        for fn in ("oracle_l2_exact_u8", "oracle_l2_exact_u8_int", "oracle_l2_topk_u8_update", "oracle_cosine_exact_u8",
                   "oracle_speed_exact", "oracle_speed_prepare_u8", "oracle_speed_prepare_f32"):
            getattr(L, fn).restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _prep(corpus, queries, dtype_c=np.uint8):
    C = np.ascontiguousarray(corpus, dtype=dtype_c)
    Q = np.ascontiguousarray(queries, dtype=np.float32)
    if Q.ndim == 1:
        Q = Q[None, :]
    assert C.ndim == 2 and Q.shape[1] == C.shape[1]
    return C, Q


def l2_exact_u8(corpus, queries, k):
    """(ids [nq,k] int32, dist [nq,k] float32), ascending (dist, id)."""
    C, Q = _prep(corpus, queries)
    nq = Q.shape[0]
    ids = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.float32)
    lib().oracle_l2_exact_u8(_p(C), C.shape[0], C.shape[1], _p(Q), nq, k, _p(ids), _p(dist))
    return ids, dist


def l2_exact_u8_int(corpus, queries_u8, k):
    """(ids [nq,k] int32, dist [nq,k] int64) for u8 queries, int64 arithmetic."""
    C = np.ascontiguousarray(corpus, dtype=np.uint8)
    Q = np.ascontiguousarray(queries_u8, dtype=np.uint8)
    if Q.ndim == 1:
        Q = Q[None, :]
    assert C.shape[1] <= 258, "float-key selection is exact only for d <= 258"
    nq = Q.shape[0]
    ids = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.int64)
    lib().oracle_l2_exact_u8_int(_p(C), C.shape[0], C.shape[1], _p(Q), nq, k, _p(ids), _p(dist))
    return ids, dist


class L2TopK:
    """Exact L2 top-k of u8 queries over a corpus fed one row slice at a time
    (``oracle_l2_topk_u8_update``): the same (distance, id) ranking as
    :func:`l2_exact_u8_int`, for corpora too large to hold on the host at once.
    ``update(rows, id_base)`` folds in rows with global ids starting at
    ``id_base``; ``ids`` / ``dist`` ([nq, k]) hold the result (-1 past the rows
    seen)."""

    def __init__(self, queries_u8, k):
        self.Q = np.ascontiguousarray(queries_u8, dtype=np.uint8)
        if self.Q.ndim == 1:
            self.Q = self.Q[None, :]
        self.k = k
        self.ids = np.full((self.Q.shape[0], k), -1, np.int32)
        self.dist = np.full((self.Q.shape[0], k), -1, np.int64)

    def update(self, rows_u8, id_base=0):
        C = np.ascontiguousarray(rows_u8, dtype=np.uint8)
        assert C.ndim == 2 and C.shape[1] == self.Q.shape[1]
        lib().oracle_l2_topk_u8_update(_p(C), C.shape[0], C.shape[1], int(id_base), _p(self.Q), self.Q.shape[0],
                                       self.k, _p(self.ids), _p(self.dist))
        return self


def l2_topk_u8(corpus, queries_u8, k, slice_rows=1 << 22):
    """(ids, dist) like :func:`l2_exact_u8_int`, scanning the corpus once for
    all queries (row slices of ``slice_rows``)."""
    t = L2TopK(queries_u8, k)
    for s in range(0, corpus.shape[0], slice_rows):
        t.update(corpus[s:s + slice_rows], s)
    return t.ids, t.dist


def cosine_exact_u8(corpus, queries, k):
    """(ids, score) for MadhavaL2 cosine on a u8 base, descending score."""
    C, Q = _prep(corpus, queries)
    nq = Q.shape[0]
    ids = np.empty((nq, k), np.int32)
    sc = np.empty((nq, k), np.float32)
    lib().oracle_cosine_exact_u8(_p(C), C.shape[0], C.shape[1], _p(Q), nq, k, _p(ids), _p(sc))
    return ids, sc


def speed_prepare(corpus, is_cosine):
    """SpeedEngine's internal float corpus and norms."""
    n, d = corpus.shape
    f = np.empty((n, d), np.float32)
    nr = np.empty(n, np.float32)
    if corpus.dtype == np.uint8:
        C = np.ascontiguousarray(corpus)
        lib().oracle_speed_prepare_u8(_p(C), n, d, int(is_cosine), _p(f), _p(nr))
    else:
        C = np.ascontiguousarray(corpus, dtype=np.float32)
        lib().oracle_speed_prepare_f32(_p(C), n, d, int(is_cosine), _p(f), _p(nr))
    return f, nr


def speed_exact(corpus, queries, k, is_cosine, prepared=None):
    """(ids, score) for SpeedEngine's CPU exact scan; descending score."""
    f, nr = prepared if prepared is not None else speed_prepare(corpus, is_cosine)
    Q = np.ascontiguousarray(queries, dtype=np.float32)
    if Q.ndim == 1:
        Q = Q[None, :]
    nq = Q.shape[0]
    ids = np.empty((nq, k), np.int32)
    sc = np.empty((nq, k), np.float32)
    lib().oracle_speed_exact(_p(f), _p(nr), f.shape[0], f.shape[1], int(is_cosine), _p(Q), nq, k,
                             _p(ids), _p(sc))
    return ids, sc


def score_ids(kind: str, corpus, queries, ids, prepared=None):
    """Reference-arithmetic scores of given ids, [nq][m] float32 (NaN for id < 0).

    kind: "exact_l2" | "exact_cos" | "speed_l2" | "speed_cos"."""
    Q = np.ascontiguousarray(queries, dtype=np.float32)
    if Q.ndim == 1:
        Q = Q[None, :]
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out = np.empty(ids.shape, np.float32)
    d = Q.shape[1]
    cos = kind.endswith("cos")
    if kind.startswith("exact"):
        C = np.ascontiguousarray(corpus, dtype=np.uint8)
        for i in range(len(Q)):
            lib().oracle_score_ids(0 if kind == "exact_l2" else 1, int(cos), _p(C), None, None, d, _p(Q[i]),
                                   _p(ids[i]), ids.shape[1], _p(out[i]))
    else:
        f, nr = prepared if prepared is not None else speed_prepare(np.ascontiguousarray(corpus), cos)
        for i in range(len(Q)):
            lib().oracle_score_ids(2, int(cos), None, _p(f), _p(nr), d, _p(Q[i]), _p(ids[i]), ids.shape[1],
                                   _p(out[i]))
    return out


def equivalent_topk(kind: str, corpus, queries, got, want, prepared=None) -> list:
    """Queries where `got` is not an equally good top-k as `want`.

    Two lists are equivalent when their score multisets match and they agree
    on every id whose score beats the k-th score (ids tied at the k-th score
    may differ: the reference leaves that choice unspecified)."""
    sg = score_ids(kind, corpus, queries, got, prepared)
    sw = score_ids(kind, corpus, queries, want, prepared)
    bad = []
    asc = kind == "exact_l2"
    for i in range(len(sg)):
        a, b = np.sort(sg[i]), np.sort(sw[i])
        if not np.array_equal(np.nan_to_num(a, nan=np.inf), np.nan_to_num(b, nan=np.inf)):
            bad.append(i)
            continue
        valid = ~np.isnan(sw[i])
        if not valid.any():
            continue
        edge = sw[i][valid].max() if asc else sw[i][valid].min()
        strict_w = set(want[i][(sw[i] < edge) if asc else (sw[i] > edge)].tolist())
        strict_g = set(got[i][(sg[i] < edge) if asc else (sg[i] > edge)].tolist())
        if strict_w != strict_g:
            bad.append(i)
    return bad


def ivf_route(centroids, queries_u8, nprobe):
    """[nq, nprobe] cells per query, best first (MadHybrid routing,
    python/winnex_madhava/__init__.py:631-632, fp64 in dimension order)."""
    Cn = np.ascontiguousarray(centroids, dtype=np.float32)
    Q = np.ascontiguousarray(queries_u8, dtype=np.uint8)
    if Q.ndim == 1:
        Q = Q[None, :]
    out = np.empty((Q.shape[0], nprobe), np.int32)
    lib().oracle_ivf_route(_p(Cn), Cn.shape[0], Cn.shape[1], _p(Q), Q.shape[0], nprobe, _p(out))
    return out


def ivf_exact(corpus, labels, centroids, queries_u8, k, nprobe, metric="l2"):
    """(ids, dist) [nq, k]: exact top-k over the union of each query's probed
    cells; -1 past the rows available.  metric "l2": by (squared L2, row id);
    "ip": by (inner product descending, row id), dist = the inner product
    (MadHybrid's merge for metric "cosine", python/winnex_madhava/__init__.py:640-646)."""
    C = np.ascontiguousarray(corpus, dtype=np.uint8)
    Q = np.ascontiguousarray(queries_u8, dtype=np.uint8)
    probe = ivf_route(centroids, Q, nprobe)
    labels = np.asarray(labels)
    ids = np.full((Q.shape[0], k), -1, np.int32)
    dist = np.full((Q.shape[0], k), -1, np.int64)
    C64 = C.astype(np.int64)
    for i in range(Q.shape[0]):
        rows = np.flatnonzero(np.isin(labels, probe[i]))
        if metric == "ip":
            d = C64[rows] @ Q[i].astype(np.int64)
            order = np.lexsort((rows, -d))[:k]
        else:
            d = ((C64[rows] - Q[i].astype(np.int64)) ** 2).sum(axis=1)
            order = np.lexsort((rows, d))[:k]
        ids[i, :len(order)] = rows[order]
        dist[i, :len(order)] = d[order]
    return ids, dist


def ivf_route_f32(centroids, queries, nprobe):
    """[nq, nprobe] cells per float query, best first (fp64 in dimension
    order, as ivf_route)."""
    Cn = np.ascontiguousarray(centroids, dtype=np.float32)
    Q = np.ascontiguousarray(queries, dtype=np.float32)
    if Q.ndim == 1:
        Q = Q[None, :]
    out = np.empty((Q.shape[0], nprobe), np.int32)
    lib().oracle_ivf_route_f32(_p(Cn), Cn.shape[0], Cn.shape[1], _p(Q), Q.shape[0], nprobe, _p(out))
    return out


def ivf_ip_f32(rows, labels, centroids, queries, k, nprobe):
    """(ids int32, scores float64) [nq, k]: the exact top-k by float64 inner
    product (descending, then row id) over the union of each float query's
    probed cells -- MadHybrid over a float corpus with every probed row
    scored (python/winnex_madhava/__init__.py:526, :650); -1 / -inf past
    the rows available."""
    X = np.ascontiguousarray(rows, dtype=np.float32)
    Q = np.ascontiguousarray(queries, dtype=np.float32)
    if Q.ndim == 1:
        Q = Q[None, :]
    lab = np.ascontiguousarray(labels, dtype=np.int32)
    cells = ivf_route_f32(centroids, Q, nprobe)
    ids = np.empty((Q.shape[0], k), np.int32)
    sc = np.empty((Q.shape[0], k), np.float64)
    lib().oracle_ivf_ip_f32(_p(X), X.shape[0], X.shape[1], _p(lab), _p(cells), nprobe, _p(Q), Q.shape[0], k,
                            _p(ids), _p(sc))
    return ids, sc


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def reference_module():
    """The compiled reference module (_winnex_madhava) from oracle/_ref, or None."""
    if not os.path.isdir(REF_DIR):
        return None
    for fn in os.listdir(REF_DIR):
        if fn.startswith("_winnex_madhava") and fn.endswith(".so"):
            name = "_oracle_ref_winnex_madhava"
            if name in sys.modules:
                return sys.modules[name]
            spec = importlib.util.spec_from_file_location("_winnex_madhava", os.path.join(REF_DIR, fn))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            sys.modules[name] = mod
            return mod
    return None
