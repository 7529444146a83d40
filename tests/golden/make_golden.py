"""Generate the golden fixtures by running the reference's own CPU code.

Requires oracle/_ref/_winnex_madhava*.so (built by `make -C oracle ref` from
the reference sources).  For each case in cases.py this records the ids the
reference returns, the sha256 of the generated inputs, and writes
tests/golden/<case>.npz.  Keys:
  exact_l2_k<K>    MadhavaL2(metric=L2).search_exact ids  [nq][K]
  exact_cos_k<K>   MadhavaL2(metric=Cosine).search_exact ids
  speed_l2_k<K>    SpeedEngine(metric=1).search ids (tie order unspecified)
  speed_cos_k<K>   SpeedEngine(metric=0).search ids (tie order unspecified)
  speedb_*         the same through search_batch
Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))

import cases  # noqa: E402
import oracle  # noqa: E402


def exact(R, C, Q, k, metric):
    cfg = R.Config()
    cfg.dim = C.shape[1]
    cfg.k = k
    cfg.metric = metric
    e = R.MadhavaL2(cfg)
    e.build_numpy(np.ascontiguousarray(C))
    out = np.full((len(Q), k), -1, np.int32)
    for i, q in enumerate(Q):
        ids = e.search_exact(np.ascontiguousarray(q, dtype=np.float32)).indices
        out[i, :len(ids)] = ids
    return out


def speed(R, C, Q, k, metric, batch=False):
    s = R.SpeedEngine(np.ascontiguousarray(C), C.shape[1], metric, 0, 4, False, "")
    kk = min(k, C.shape[0])
    out = np.full((len(Q), k), -1, np.int32)
    if batch:
        ids = np.array(s.search_batch(np.ascontiguousarray(Q, dtype=np.float32), len(Q), k)["indices"]).reshape(len(Q), kk)
        out[:, :kk] = ids
    else:
        for i, q in enumerate(Q):
            ids = s.search(np.ascontiguousarray(q, dtype=np.float32), k)["indices"]
            out[i, :len(ids)] = ids
    return out


def reference_hybrid(C, Q):
    """The reference's own MadHybrid (python/winnex_madhava/__init__.py:547-654)
    built on the u8 case: its MiniBatchKMeans centroids and cell labels, and
    its routing expression `argsort(-(centroids @ q))[:nprobe]` (:631-632)
    evaluated here on those centroids."""
    import shutil
    import tempfile

    ref_py = os.path.join(oracle.REFERENCE_DIR, "python", "winnex_madhava", "__init__.py")
    so = [f for f in os.listdir(oracle.REF_DIR) if f.startswith("_winnex_madhava") and f.endswith(".so")][0]
    tmp = tempfile.mkdtemp()
    try:
        pkg = os.path.join(tmp, "winnex_madhava")
        os.mkdir(pkg)
        os.symlink(ref_py, os.path.join(pkg, "__init__.py"))
        os.symlink(os.path.join(oracle.REF_DIR, so), os.path.join(pkg, so))
        sys.path.insert(0, tmp)
        import winnex_madhava as refwm  # the reference package, not this repository's

        h = cases.HYBRID
        eng = refwm.build_engine(np.ascontiguousarray(C), dim=C.shape[1], metric="l2", hybrid=True,
                                 nlist=h["nlist"], nprobe=h["nprobe"], seed=h["seed"])
        centroids = np.asarray(eng._centroids, dtype=np.float32)
        labels = np.full(C.shape[0], -1, np.int32)
        for cid, idxs in eng._members.items():
            labels[np.asarray(idxs)] = cid
        assert (labels >= 0).all()
        route = np.stack([np.argsort(-(centroids @ np.ascontiguousarray(q, dtype=np.float32).flatten()))[:h["nprobe"]]
                          for q in Q]).astype(np.int32)
        sims = (centroids.astype(np.float64) @ Q.astype(np.float64).T).T
        return {"centroids": centroids, "labels": labels, "route_ref": route, "sims64": sims}
    finally:
        sys.path.remove(tmp)
        shutil.rmtree(tmp)


def main():
    R = oracle.reference_module()
    if R is None:
        raise SystemExit("oracle/_ref not built: run `make -C oracle ref` first")
    M = R.Metric
    todo = {}

    C, Q = cases.case_api()
    todo["api"] = ((C, Q), {f"exact_l2_k{k}": exact(R, C, Q, k, M.L2) for k in (1, 10, 64)} |
                   {"exact_cos_k10": exact(R, C, Q, 10, M.COSINE), "speed_l2_k10": speed(R, C, Q, 10, 1),
                    "speed_cos_k10": speed(R, C, Q, 10, 0), "speedb_l2_k10": speed(R, C, Q, 10, 1, True)})

    X, Xu = cases.case_clustered()
    Qu = Xu[:16].astype(np.float32)
    Qf = X[:16]
    todo["clustered_u8"] = ((Xu, Qu), {"speed_l2_k10": speed(R, Xu, Qu, 10, 1),
                                      "speedb_l2_k10": speed(R, Xu, Qu, 10, 1, True),
                                      "exact_l2_k10": exact(R, Xu, Qu, 10, M.L2)})
    todo["clustered_f32"] = ((X, Qf), {"speed_cos_k10": speed(R, X, Qf, 10, 0),
                                      "speedb_cos_k10": speed(R, X, Qf, 10, 0, True),
                                      "speed_l2_k10": speed(R, X, Qf, 10, 1)})

    C, Q = cases.case_quickstart()
    todo["quickstart"] = ((C, Q), {"exact_l2_k10": exact(R, C, Q, 10, M.L2),
                                   "exact_cos_k10": exact(R, C, Q, 10, M.COSINE)})

    C, Q = cases.case_gmm()
    todo["gmm"] = ((C, Q), {"exact_l2_k10": exact(R, C, Q, 10, M.L2), "exact_l2_k100": exact(R, C, Q, 100, M.L2),
                            "speedb_l2_k10": speed(R, C, Q, 10, 1, True)})

    C, Q = cases.case_float_queries()
    todo["float_queries"] = ((C, Q), {"exact_l2_k10": exact(R, C, Q, 10, M.L2),
                                      "exact_cos_k10": exact(R, C, Q, 10, M.COSINE),
                                      "speed_l2_k10": speed(R, C, Q, 10, 1),
                                      "speed_cos_k10": speed(R, C, Q, 10, 0)})

    C, Q = cases.case_dups()
    todo["dups"] = ((C, Q), {"exact_l2_k10": exact(R, C, Q, 10, M.L2), "exact_l2_k64": exact(R, C, Q, 64, M.L2)})

    for d in cases.DIMS:
        C, Q = cases.case_dim(d)
        todo[f"dim{d}"] = ((C, Q), {"exact_l2_k10": exact(R, C, Q, 10, M.L2),
                                    "exact_cos_k10": exact(R, C, Q, 10, M.COSINE)})

    C, Q = cases.case_small()
    todo["small"] = ((C, Q), {"exact_l2_k10": exact(R, C, Q, 10, M.L2)})

    X, Q = cases.case_f32_corpus()
    todo["f32_corpus"] = ((X, Q), {"speed_cos_k10": speed(R, X, Q, 10, 0), "speed_l2_k10": speed(R, X, Q, 10, 1),
                                   "speedb_cos_k10": speed(R, X, Q, 10, 0, True)})

    C, Q = cases.case_hybrid()
    todo["hybrid"] = ((C, Q), reference_hybrid(C, Q))

    for name, ((C, Q), res) in todo.items():
        meta = {"case": name, "sha256": cases.sha(C, Q), "corpus_shape": list(C.shape), "corpus_dtype": str(C.dtype),
                "nq": int(len(Q)), "generator": "reference oracle/_ref (_winnex_madhava compiled from the reference sources)"}
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), meta=json.dumps(meta), **res)
        print(name, {k: v.shape for k, v in res.items()})


if __name__ == "__main__":
    main()
