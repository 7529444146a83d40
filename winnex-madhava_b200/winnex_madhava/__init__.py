"""winnex_madhava -- exact top-K vector search on NVIDIA B200.

Drop-in replacement for the Python API of winnex-madhava
(python/winnex_madhava/__init__.py): ``build_engine``, ``MadhavaL2``,
``MadhavaSpeed``, ``MadHybrid``, ``retrieve``, ``benchmark_vs_groundtruth`` and
the re-exported ``Config`` / ``SearchResult`` / enums / metric helpers keep
their names and arguments.  Every search runs on the GPU through
``libwinnex_madhava_b200.so`` (hand-written sm_100a kernels behind a C ABI);
there is no CPU or torch fallback -- without a B200 the engines raise.

Semantics:

* Searches are exact.  ``MadhavaL2.search`` returns the same list as
  ``search_exact``; L2 ranks by (squared distance, row id), so the lower id
  wins a tie, as in the reference's ``search_exact``
  (src/winnex_madhava.cpp:1237-1239).  ``bound_violations`` is 0 because no
  pair is excluded without an exact comparison.
* u8 corpora with integral queries use integer arithmetic (exact for every
  metric); float queries reproduce the reference's float evaluation order.
"""
from __future__ import annotations

import math
import os
import sys
import time
import weakref as _weakref

import numpy as np

_this_dir = os.path.dirname(os.path.abspath(__file__))
try:
    from . import _winnex_madhava as _native
except ImportError as exc:  # the product has no fallback path
    raise ImportError(
        "winnex_madhava: native module _winnex_madhava (and libwinnex_madhava_b200.so) not found next to "
        f"{__file__}; build it with `python winnex-madhava_b200/build.py`"
    ) from exc

# Engines copy the corpus to device memory, so the caller's buffer does not
# have to outlive them; the side table is kept for API compatibility with
# code that calls _attach_buffer (python/winnex_madhava/__init__.py:52-71).
_BUFFER_REF_TABLE: dict[int, object] = {}
_ENGINE_WEAKREFS: list = []


def _release_engine(ref):
    _BUFFER_REF_TABLE.pop(id(ref), None)


def _attach_buffer(engine, arr):
    _BUFFER_REF_TABLE[id(engine)] = arr
    try:
        _ENGINE_WEAKREFS.append(_weakref.ref(engine, _release_engine))
    except TypeError:
        pass
    return engine


Config = _native.Config
SearchResult = _native.SearchResult
MadhavaL2 = _native.MadhavaL2
Metric = _native.Metric
QuantMode = _native.QuantMode
BasisMode = _native.BasisMode
recall_at_k = _native.recall_at_k
ndcg_at_k = _native.ndcg_at_k
read_bigann_groundtruth = _native.read_bigann_groundtruth
l2_sq = _native.l2_sq
# Not in the reference API: re-check up to n queries of every search with an
# exact unpruned scan and report misplaced rows in bound_violations (0 = off).
set_verify = _native.set_verify

__version__ = "1.9.3+b200"
__all__ = [
    "Config",
    "SearchResult",
    "MadhavaL2",
    "MadHybrid",
    "MadhavaSpeed",
    "Metric",
    "QuantMode",
    "BasisMode",
    "recall_at_k",
    "ndcg_at_k",
    "read_bigann_groundtruth",
    "build_engine",
    "retrieve",
    "benchmark_vs_groundtruth",
    "set_verify",
    "__version__",
]


def _metric_enum(metric: str):
    return Metric.COSINE if metric.lower() == "cosine" else Metric.L2


def build_engine(
    corpus: np.ndarray,
    *,
    dim: int | None = None,
    metric: str = "cosine",
    quant: str = "int8",
    basis: str = "random",
    pca_sample: int = 10000,
    stage1_dim: int = 64,
    stage2_dim: int = 128,
    k: int = 10,
    k1_fraction: float = 0.05,
    k2_fraction: float = 0.01,
    k2_max: int = 2000,
    modulation: bool = True,
    postfilter: bool = True,
    normalize_input: bool = True,
    early_exit: bool | None = None,
    seed: int = 42,
    hybrid: bool = False,
    nlist: int = 64,
    nprobe: int = 5,
    speed: bool = False,
    gpu_dtype: str = "float32",
    require_gpu: bool = False,
    speed_n_anchors: int = 0,
    speed_nprobe: int = 4,
    speed_opencl_lib: str = "",
    devices=None,
):
    """Build an exact search engine over ``corpus`` (same arguments as the reference).

    Routing follows the reference (python/winnex_madhava/__init__.py:105-342):
    ``hybrid=True`` returns a :class:`MadHybrid`, ``speed=True`` a
    :class:`MadhavaSpeed`, otherwise a :class:`MadhavaL2`.  A float corpus
    goes through ``MadhavaL2.build_float32``.  The bound-cascade knobs
    (``quant``, ``stage*_dim``, ``k*_fraction``, ``modulation``,
    ``postfilter``, ``early_exit``, ``basis``, ``pca_sample``) are stored in the
    Config for introspection; the search itself is exact.  ``gpu_dtype``,
    ``speed_n_anchors``, ``speed_nprobe`` and ``speed_opencl_lib`` are accepted
    and ignored (the GPU scan is always exact).  ``devices`` (new): a device
    count or list to shard the corpus over.
    """
    arr = np.ascontiguousarray(corpus)
    if arr.ndim != 2:
        raise ValueError("corpus must be a 2D array of shape (n, dim)")
    if dim is None:
        dim = arr.shape[1]
    is_float = arr.dtype in (np.float32, np.float64)
    if not (hybrid or speed) and not is_float:
        arr = np.ascontiguousarray(arr, dtype=np.uint8)

    cfg = Config()
    cfg.dim = int(dim)
    cfg.metric = _metric_enum(metric)
    cfg.quant = QuantMode.INT8 if quant.lower() == "int8" else QuantMode.NONE
    cfg.basis = BasisMode.PCA_CORPUS if basis.lower() == "pca_corpus" else BasisMode.RANDOM
    cfg.pca_sample = int(pca_sample)
    cfg.stage1_dim = int(stage1_dim)
    cfg.stage2_dim = int(stage2_dim)
    cfg.k = int(k)
    cfg.k1_fraction = float(k1_fraction)
    cfg.k2_fraction = float(k2_fraction)
    cfg.k2_max = int(k2_max)
    cfg.modulation = bool(modulation)
    cfg.postfilter = bool(postfilter)
    cfg.normalize_input = bool(normalize_input)
    cfg.early_exit = bool(early_exit) if early_exit is not None else False
    cfg.seed = int(seed)

    if hybrid:
        return MadHybrid(arr, nlist=nlist, nprobe=nprobe, metric=metric, seed=seed, k=k, devices=devices)
    if speed:
        return MadhavaSpeed(arr, k=int(k), metric=metric, dtype=gpu_dtype, n_anchors=int(speed_n_anchors),
                            nprobe=int(speed_nprobe), require_gpu=require_gpu, opencl_lib=speed_opencl_lib,
                            devices=devices)
    engine = MadhavaL2(cfg)
    if devices is not None:
        engine._set_devices(devices)
    if is_float:
        engine.build_float32(np.ascontiguousarray(arr, dtype=np.float32))
    else:
        engine.build_numpy(arr)
    return engine


def retrieve(engine, query: np.ndarray, corpus_text: list[str] | None = None, k: int | None = None) -> dict:
    """Top-K ids (and texts) for one query, with the search counters.

    Same keys as the reference helper (python/winnex_madhava/__init__.py:345-402).
    ``scores`` holds zeros like the reference (exact scores are not exposed
    through ``search``).
    """
    kk = k or engine.config().k
    res = engine.search(np.ascontiguousarray(query, dtype=np.float32))
    ids = list(res.indices[:kk])
    out = {
        "indices": ids,
        "scores": [0.0] * len(ids),
        "bound_violations": int(res.bound_violations),
        "k1": int(res.k1),
        "k2": int(res.k2),
        "k3": int(res.k3),
        "latency_ms": float(res.latency_ms),
        "proof": (
            "exact scan: every corpus row was compared exactly with the query on the GPU; "
            "no row was excluded by a bound (bound_violations == 0), recall vs exhaustive scan is 1.0"
        ),
    }
    if corpus_text is not None:
        out["contents"] = [corpus_text[i] if 0 <= i < len(corpus_text) else None for i in ids]
    return out


def benchmark_vs_groundtruth(engine, queries: np.ndarray, gt_ids, *, query_alignment: int = 1,
                             k: int | None = None) -> dict:
    """Recall@K / NDCG@K / mean latency of ``engine.search`` against id lists.

    Mirrors python/winnex_madhava/__init__.py:405-457 (query i*alignment is
    scored against gt_ids[i], ids outside the corpus are dropped).
    """
    k = k or engine.config().k
    q = np.ascontiguousarray(queries, dtype=np.float32)
    if q.ndim != 2:
        raise ValueError("queries must be (n_queries*alignment, dim) float32")
    n_queries = len(gt_ids)
    rs = ns = ls = 0.0
    per_query = []
    nv = engine.num_vectors()
    for i in range(n_queries):
        qi = i * query_alignment
        res = engine.search(q[qi])
        gset = [v for v in gt_ids[i] if 0 <= v < nv]
        r = recall_at_k(res.indices, gset, k)
        n = ndcg_at_k(res.indices, gset, k)
        rs += r
        ns += n
        ls += res.latency_ms
        per_query.append({"query": qi, "recall": r, "ndcg": n})
    m = max(n_queries, 1)
    return {"recall_at_k": rs / m, "ndcg_at_k": ns / m, "latency_ms": ls / m, "n_queries": n_queries, "k": k,
            "per_query": per_query}


class _SimpleResult:
    """Result object of MadhavaSpeed / MadHybrid (python/winnex_madhava/__init__.py:682-693)."""

    def __init__(self, indices, bound_violations):
        self.indices = indices
        self.bound_violations = bound_violations
        self.k1 = 0
        self.k2 = 0
        self.k3 = 0
        self.latency_ms = 0.0
        self.bound_pairs = 0
        self.modulation_gain = 0.0
        self.pruned_by_bound = 0
        self.verified_queries = 0


def _speed_result(res):
    """_SimpleResult from a native SpeedEngine dict, keeping its measured
    counters (bound_violations is measured when set_verify is on)."""
    out = _SimpleResult(res["indices"], int(res.get("bound_violations", 0)))
    out.latency_ms = res["latency_ms"]
    out.bound_pairs = int(res.get("bound_pairs", 0))
    out.pruned_by_bound = int(res.get("pruned_by_bound", 0))
    out.verified_queries = int(res.get("verified_queries", 0))
    return out


class MadhavaSpeed:
    """Exact GPU scan engine returned by ``build_engine(..., speed=True)``.

    Backed by the native ``SpeedEngine``: u8 corpora (L2) stay u8 in HBM,
    float corpora are prepared with the reference's arithmetic
    (src/speed_cpu.cpp:81-144).  Scores follow SpeedEngine: inner product of
    normalized vectors (cosine) or 2*dot - |v|^2 (L2).
    """

    def __init__(self, corpus, *, k=10, metric="cosine", dtype="float32", n_anchors=0, nprobe=4,
                 require_gpu=False, opencl_lib="", devices=None):
        self._k = int(k)
        self._metric = metric.lower()
        arr = np.ascontiguousarray(corpus)
        self._n, self._dim = arr.shape
        t0 = time.time()
        m = 1 if self._metric == "l2" else 0
        if arr.dtype == np.uint8:
            self._native = _native.SpeedEngine(arr, self._dim, m, int(n_anchors), int(nprobe), bool(require_gpu),
                                               str(opencl_lib or ""), devices)
        else:
            self._native = _native.SpeedEngine(np.ascontiguousarray(arr, dtype=np.float32), self._dim, m,
                                               int(n_anchors), int(nprobe), bool(require_gpu), str(opencl_lib or ""),
                                               devices)
        self._build_time = time.time() - t0

    def search(self, query, k: int | None = None):
        kk = k or self._k
        q = np.ascontiguousarray(query, dtype=np.float32).reshape(-1)
        return _speed_result(self._native.search(q, kk))

    def search_batch(self, queries, k: int | None = None, chunk: int = 128):
        kk = k or self._k
        Q = np.ascontiguousarray(queries, dtype=np.float32)
        if Q.ndim == 1:
            Q = Q.reshape(1, -1)
        return _speed_result(self._native.search_batch(Q, len(Q), kk))

    def search_exact(self, query, k: int | None = None):
        return self.search(query, k=k)

    def num_vectors(self):
        return self._n

    def dim(self):
        return self._dim

    def build_seconds(self):
        return self._build_time

    def built(self):
        return True

    @property
    def backend(self):
        return "native"


class MadHybrid:
    """Clustered (IVF) search returned by ``build_engine(..., hybrid=True)``.

    Cells come from scikit-learn MiniBatchKMeans with the reference's settings
    (python/winnex_madhava/__init__.py:577-593); a query is routed to the
    ``nprobe`` cells whose centroids have the largest inner product with it
    (:631-632), and the result is the exact top-k over the union of those
    cells.  For a uint8 corpus (dim <= 128) with integral queries that runs
    entirely on the GPU index ``IvfIndex`` in one batched call (routing in
    fp64, ties to the lower cell id): under L2 ranked by (squared distance,
    row id), under the default metric "cosine" by (inner product, row id) --
    the reference merges a u8 corpus by ``corpus[ids] @ q`` (:640-646), exact
    in integers here.  A float32 corpus runs on the GPU index ``IvfIndexF32``,
    also in one batched call: the reference's float cells score their rows by
    the float64 inner product ``vecs @ q`` and the merge orders by that score
    (:526, :650), so the result is the top-k of the probed cells' union by
    (float64 inner product, row id), for k <= 16.  Larger k and non-integral
    queries on a uint8 corpus use one exact GPU engine per cell.
    """

    def __init__(self, corpus, *, nlist: int = 64, nprobe: int = 5, dtype: str | None = None,
                 metric: str = "cosine", stage1_dim: int = 32, stage2_dim: int = 64, keep_fraction: float = 0.40,
                 k2: int = 200, seed: int = 42, native_builder=None, k: int = 10, devices=None):
        self._nprobe = int(nprobe)
        self._nlist = int(nlist)
        self._metric = metric.lower()
        arr = np.ascontiguousarray(corpus)
        if dtype is None:
            self._dtype = "uint8" if arr.dtype == np.uint8 else "float32"
        else:
            self._dtype = dtype.lower()
        self._corpus = arr
        self._n, self._dim = arr.shape
        self._k = int(k)
        try:
            from sklearn.cluster import MiniBatchKMeans
        except ImportError as exc:  # pragma: no cover
            raise ImportError("hybrid mode requires scikit-learn") from exc
        E = arr.astype(np.float32)
        km = MiniBatchKMeans(n_clusters=self._nlist, random_state=seed, batch_size=min(10000, self._n), n_init=3,
                             max_iter=50)
        labels = km.fit_predict(E)
        self._centroids = km.cluster_centers_.astype(np.float32)
        self._labels = labels
        self._members = {}
        self._cells = {}
        self._devices = devices
        self._ivf = None
        self._ivf_f32 = None
        t0 = time.time()
        if self._dtype != "uint8":
            dev = int(devices[0]) if devices else -1
            self._ivf_f32 = _native.IvfIndexF32(np.ascontiguousarray(E, dtype=np.float32), self._centroids,
                                                np.ascontiguousarray(labels, dtype=np.int32), dev)
            for cid in range(self._nlist):
                idxs = np.where(labels == cid)[0]
                if len(idxs):
                    self._members[cid] = idxs
            self._build_time = time.time() - t0
            return
        if self._dtype == "uint8" and self._dim <= 128:
            # metric "cosine" merges by the raw inner product corpus @ q
            # (python/winnex_madhava/__init__.py:640-646): the index's
            # inner-product form (metric 0); otherwise L2 (metric 1).
            dev = int(devices[0]) if devices else -1
            self._ivf = _native.IvfIndex(np.ascontiguousarray(arr, dtype=np.uint8), self._centroids,
                                         np.ascontiguousarray(labels, dtype=np.int32), dev,
                                         0 if self._metric == "cosine" else 1)
            for cid in range(self._nlist):
                idxs = np.where(labels == cid)[0]
                if len(idxs):
                    self._members[cid] = idxs
            self._build_time = time.time() - t0
            return
        self._build_cells()
        self._build_time = time.time() - t0

    def _build_cells(self):
        arr, labels, devices = self._corpus, self._labels, self._devices
        E = arr.astype(np.float32)
        for cid in range(self._nlist):
            idxs = np.where(labels == cid)[0]
            if len(idxs) == 0:
                continue
            self._members[cid] = idxs
            if self._dtype == "uint8":
                cell = np.ascontiguousarray(arr[idxs], dtype=np.uint8)
                self._cells[cid] = MadhavaSpeed(cell, k=self._k, metric=self._metric, devices=devices)
            else:
                cell = np.ascontiguousarray(E[idxs], dtype=np.float32)
                self._cells[cid] = MadhavaSpeed(cell, k=self._k, metric="cosine" if self._metric == "cosine" else "l2",
                                                devices=devices)

    @staticmethod
    def _ivf_result(indices, st):
        r = _SimpleResult(indices, int(st.get("bound_violations", 0)))
        r.latency_ms = float(st["latency_ms"])
        r.bound_pairs = int(st.get("pairs_scored", 0))
        r.pruned_by_bound = int(st.get("pruned_by_bound", 0))
        return r

    def _probe(self, q, nprobe):
        sims = self._centroids @ q
        return np.argsort(-sims, kind="stable")[:nprobe]

    def search(self, query, k: int | None = None, nprobe: int | None = None):
        np_ = min(self._nprobe if nprobe is None else int(nprobe), self._nlist)
        kk = k or self._k
        q = np.ascontiguousarray(query, dtype=np.float32).reshape(-1)
        if self._ivf is not None and np.all((q >= 0) & (q <= 255) & (q == np.round(q))):
            ids, _, st = self._ivf.search(q.astype(np.uint8)[None, :], kk, np_)
            return self._ivf_result([int(i) for i in ids[0] if i >= 0], st)
        if self._ivf_f32 is not None and kk <= 16:
            ids, _, st = self._ivf_f32.search(q[None, :], kk, np_)
            return self._ivf_result([int(i) for i in ids[0] if i >= 0], st)
        if not self._cells:
            self._build_cells()
        cands = []
        for cid in self._probe(q, np_):
            cell = self._cells.get(int(cid))
            if cell is None:
                continue
            local = np.asarray(cell.search(q, k=kk).indices, dtype=np.int64)
            gids = self._members[int(cid)][local]
            cands.extend(gids.tolist())
        out = self._rank(np.asarray(cands, dtype=np.int64), q, kk)
        return _SimpleResult(out, 0)

    def _rank(self, ids, q, kk):
        if len(ids) == 0:
            return []
        if self._dtype == "uint8" and self._metric != "cosine":
            d = self._corpus[ids].astype(np.int64) - q.astype(np.int64) if np.all(q == np.round(q)) else None
            if d is not None:
                key = (d * d).sum(axis=1)
            else:
                dd = self._corpus[ids].astype(np.float64) - q.astype(np.float64)
                key = (dd * dd).sum(axis=1)
            order = np.lexsort((ids, key))
        else:
            s = self._corpus[ids].astype(np.float64) @ q.astype(np.float64)
            order = np.lexsort((ids, -s))
        return [int(i) for i in ids[order[:kk]]]

    def search_batch(self, queries, k: int | None = None, nprobe: int | None = None):
        """Batch form of ``search`` (not in the reference API): ``indices`` is
        the flat [nq * k] list, -1 where the probed cells hold fewer than k rows."""
        np_ = min(self._nprobe if nprobe is None else int(nprobe), self._nlist)
        kk = k or self._k
        Q = np.ascontiguousarray(queries, dtype=np.float32).reshape(-1, self._dim)
        if self._ivf is not None and np.all((Q >= 0) & (Q <= 255) & (Q == np.round(Q))):
            ids, _, st = self._ivf.search(Q.astype(np.uint8), kk, np_)
            return self._ivf_result([int(i) for i in ids.reshape(-1)], st)
        if self._ivf_f32 is not None and kk <= 16:
            ids, _, st = self._ivf_f32.search(Q, kk, np_)
            return self._ivf_result([int(i) for i in ids.reshape(-1)], st)
        out = []
        for q in Q:
            got = self.search(q, k=kk, nprobe=np_).indices
            out.extend(list(got) + [-1] * (kk - len(got)))
        return _SimpleResult(out, 0)

    def search_exact(self, query, k: int | None = None):
        """Exact scan of the whole corpus (the recall ceiling), on the GPU."""
        kk = k or self._k
        if not hasattr(self, "_full"):
            m = "l2" if (self._dtype == "uint8" and self._metric != "cosine") else "cosine"
            src = self._corpus if self._dtype == "uint8" else self._corpus.astype(np.float32)
            self._full = MadhavaSpeed(src, k=kk, metric=m)
        return _SimpleResult(list(self._full.search(query, k=kk).indices), 0)

    def num_vectors(self):
        return self._n

    def dim(self):
        return self._dim

    def build_seconds(self):
        return self._build_time

    def built(self):
        return True
