#!/usr/bin/env python3
"""Throughput benchmark: exact top-10 L2 over 100M x 128 u8 rows, 10K queries.

Workload (one "step"): 10,000 u8 queries against a 100,000,000 x 128 u8
corpus drawn from a clipped 4,096-component Gaussian mixture (means U[0,60],
per-dim std 15, rounded, clipped to [0,255]); exact top-10 by (squared L2,
row id).  Synthetic data of the BIGANN-like shape; the corpus is generated
on the GPU in fixed 3.125M-row chunks so every GPU count sees the same rows.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun: rank r holds rows [r*N/G, (r+1)*N/G), scans them
for all queries and the ranks exchange their top-10 lists with one NCCL
all_gather, merged on the GPU.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "winnex-madhava_b200"))

N_DEFAULT = 100_000_000
DIM = 128
COMPONENTS = 4096
SEED = 20261201
CHUNK = 3_125_000
L2_BYTES = 126 << 20        # B200 L2
L2_FLUSH_BYTES = 512 << 20
TRAFFIC_BYTES_PER_ROW = (1.288255e9 + 35.171072e6) / 10_000_000
METRIC = "queries/sec, 100M×128 u8 exact top-10, 10K-query batch at 1/2/4/8 B200; % roofline"


# --------------------------------------------------------------------------- data
def mixture_means(comps=COMPONENTS):
    return np.random.default_rng(SEED).uniform(0, 60, size=(comps, DIM))


def make_queries(nq, comps=COMPONENTS):
    means = mixture_means(comps)
    rng = np.random.default_rng(SEED + 1)
    lab = rng.integers(0, comps, size=nq)
    return np.clip(np.rint(means[lab] + rng.normal(0, 15, size=(nq, DIM))), 0, 255).astype(np.uint8)


def make_rows_gpu(torch, start, end, device, comps=COMPONENTS):
    """Rows [start, end) of the corpus on `device` (u8 [end-start][128])."""
    means = torch.tensor(mixture_means(comps), dtype=torch.float32, device=device)
    out = torch.empty((end - start, DIM), dtype=torch.uint8, device=device)
    c0, c1 = start // CHUNK, (end + CHUNK - 1) // CHUNK
    g = torch.Generator(device=device)
    for c in range(c0, c1):
        s, e = c * CHUNK, (c + 1) * CHUNK
        g.manual_seed(SEED * 1000 + c)
        lab = torch.randint(0, comps, (CHUNK,), generator=g, device=device)
        x = means[lab]
        x.add_(torch.randn((CHUNK, DIM), generator=g, device=device), alpha=15.0)
        x = x.round_().clamp_(0, 255).to(torch.uint8)
        lo, hi = max(s, start), min(e, end)
        if lo < hi:
            out[lo - start:hi - start] = x[lo - s:hi - s]
        del x, lab
    return out


# --------------------------------------------------------------------------- library
class Stats(ctypes.Structure):
    _fields_ = [("latency_ms", ctypes.c_double), ("pairs_scored", ctypes.c_int64),
                ("pairs_pruned_by_bound", ctypes.c_int64), ("bound_violations", ctypes.c_int64),
                ("candidates", ctypes.c_int64), ("tensor_core_path", ctypes.c_int32), ("levels", ctypes.c_int32),
                ("full_scan_ms", ctypes.c_double), ("full_scan_pairs", ctypes.c_int64),
                ("kernel_launches", ctypes.c_int64), ("verified_queries", ctypes.c_int64),
                ("sample_ms", ctypes.c_double), ("select_ms", ctypes.c_double), ("rescore_ms", ctypes.c_double),
                ("prep_ms", ctypes.c_double), ("blocks_tested", ctypes.c_int64), ("blocks_passed", ctypes.c_int64)]


def load_lib():
    path = os.path.join(ROOT, "winnex-madhava_b200", "winnex_madhava", "libwinnex_madhava_b200.so")
    if not os.path.exists(path):
        raise SystemExit(f"{path} missing: run python winnex-madhava_b200/build.py")
    L = ctypes.CDLL(path)
    P, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    L.mdh_index_create_u8_device.argtypes = [P, i64, i32, i32, i64, ctypes.POINTER(P)]
    L.mdh_index_destroy.argtypes = [P]
    L.mdh_search_u8.argtypes = [P, P, i32, i32, P, P, ctypes.POINTER(Stats)]
    L.mdh_index_create_u8.argtypes = [P, i64, i32, i32, P, i32, i64, ctypes.POINTER(P)]
    L.mdh_index_create_u8.restype = ctypes.c_int
    L.mdh_search_u8_device.argtypes = [P, P, i32, i32, P, P, P, ctypes.POINTER(Stats)]
    L.mdh_search_u8_device_sample.argtypes = [P, P, i32, i32, P, P, P, ctypes.POINTER(Stats)]
    L.mdh_search_u8_device_bounded.argtypes = [P, P, i32, i32, P, P, P, P, P, ctypes.POINTER(Stats)]
    L.mdh_search_u8_device_sample.restype = ctypes.c_int
    L.mdh_search_u8_device_bounded.restype = ctypes.c_int
    L.mdh_merge_topk_device.argtypes = [P, P, i32, i32, i32, P, P, P]
    L.mdh_set_scan_path.argtypes = [i32]
    L.mdh_set_sample_ratio.argtypes = [i32]
    L.mdh_set_threshold_sharing.argtypes = [i32]
    L.mdh_ivf_create_u8.argtypes = [P, i64, i32, P, i32, P, i32, ctypes.POINTER(P)]
    L.mdh_ivf_search_u8.argtypes = [P, P, i32, i32, i32, P, P, ctypes.POINTER(Stats)]
    L.mdh_ivf_destroy.argtypes = [P]
    L.mdh_ivf_route_u8.argtypes = [P, P, i32, i32, P]
    L.mdh_ivf_info.argtypes = [P, P, P, P, P]
    L.mdh_index_save.argtypes = [P, ctypes.c_char_p]
    L.mdh_index_load.argtypes = [ctypes.c_char_p, P, i32, ctypes.POINTER(P)]
    L.mdh_index_create_f32.argtypes = [P, i64, i32, i32, P, i32, i64, ctypes.POINTER(P)]
    L.mdh_index_create_f32.restype = ctypes.c_int
    L.mdh_search_f32.argtypes = [P, P, i32, i32, i32, P, P, ctypes.POINTER(Stats)]
    L.mdh_search_f32.restype = ctypes.c_int
    L.mdh_search_u8.restype = ctypes.c_int
    L.mdh_last_error.restype = ctypes.c_char_p
    for f in ("mdh_index_create_u8_device", "mdh_index_destroy", "mdh_search_u8", "mdh_search_u8_device",
              "mdh_merge_topk_device", "mdh_set_scan_path", "mdh_set_sample_ratio", "mdh_set_threshold_sharing",
              "mdh_ivf_create_u8",
              "mdh_ivf_search_u8",
              "mdh_ivf_destroy"):
        getattr(L, f).restype = ctypes.c_int
    return L


def check(L, st, what):
    if st != 0:
        raise RuntimeError(f"{what} failed ({st}): {L.mdh_last_error().decode()}")


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock / throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = str(gpu_index)
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = self.rows
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "", 1).isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "", 1).isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        pw = [float(r[3]) for r in rows if r[3].replace(".", "", 1).isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(pw) if pw else None}


# --------------------------------------------------------------------------- peaks
def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# --------------------------------------------------------------------------- reference arm / cpu baseline
def cpu_reference_qps(corpus_slice, n_total, queries, k, steps=1, warmup=0):
    """Time the reference's own CPU exact scan (SpeedEngine.search_batch, OpenMP over
    all host cores) on a row slice; QPS is scaled to the full corpus (the scan is
    linear in the number of rows)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # test infrastructure: CPU baseline only

    R = oracle.reference_module()
    n_slice = corpus_slice.shape[0]
    cores = os.cpu_count()
    Q = np.ascontiguousarray(queries.astype(np.float32))
    if R is not None:
        os.environ.setdefault("OMP_NUM_THREADS", str(cores))
        eng = R.SpeedEngine(np.ascontiguousarray(corpus_slice), DIM, 1, 0, 4, False, "")
        run = lambda: eng.search_batch(Q, len(Q), k)  # noqa: E731
        kind = "reference"
    else:
        run = lambda: oracle.l2_exact_u8_int(corpus_slice, queries, k)  # noqa: E731
        kind = "port"
        cores = oracle.num_threads()
    for _ in range(warmup):
        run()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    qps = len(Q) / t * (n_slice / n_total)
    sample = (f"reference SpeedEngine.search_batch (CPU, OpenMP) on rows [0, {n_slice}) of the corpus with "
              f"{len(Q)} queries per step; QPS scaled by {n_slice}/{n_total} rows (linear scan)")
    if kind == "port":
        sample = sample.replace("reference SpeedEngine.search_batch (CPU, OpenMP)", "oracle C port (OpenMP)")
    return qps, {"value": qps, "unit": "queries/sec", "cores": cores, "kind": kind, "sample": sample,
                 "seconds_per_step": t}


# --------------------------------------------------------------------------- IVF workload
IVF_COMPS, IVF_NLIST, IVF_NPROBE = 1024, 1024, 16


def run_ivf(args, torch, device, L, warmup):
    """Clustered search: 10M x 128 u8 clipped GMM (1,024 components), nlist
    1,024, nprobe 16, exact top-k over the probed cells; one GPU."""
    from sklearn.cluster import MiniBatchKMeans

    n = args.n if args.n != N_DEFAULT else 10_000_000
    nq, k = args.nq, args.k
    rows = make_rows_gpu(torch, 0, n, device, IVF_COMPS)
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 7)
    sample = rows[torch.randperm(n, generator=g, device=device)[:200_000]].cpu().numpy().astype(np.float32)
    t0 = time.time()
    km = MiniBatchKMeans(n_clusters=IVF_NLIST, random_state=42, batch_size=10_000, n_init=1, max_iter=20)
    km.fit(sample)
    cen = km.cluster_centers_.astype(np.float32)
    cen_t = torch.from_numpy(cen).to(device)
    cn = (cen_t * cen_t).sum(1)
    labels = torch.empty(n, dtype=torch.int32, device=device)
    for s in range(0, n, 1_000_000):  # nearest centroid, as MiniBatchKMeans.predict
        x = rows[s:s + 1_000_000].float()
        labels[s:s + 1_000_000] = (cn[None, :] - 2.0 * (x @ cen_t.T)).argmin(dim=1).to(torch.int32)
    host_rows = rows.cpu().numpy()
    host_labels = labels.cpu().numpy()
    cluster_s = time.time() - t0
    del rows, labels, x
    torch.cuda.empty_cache()
    h = ctypes.c_void_p()
    t0 = time.time()
    check(L, L.mdh_ivf_create_u8(ctypes.c_void_p(host_rows.ctypes.data), n, DIM, ctypes.c_void_p(cen.ctypes.data),
                                 IVF_NLIST, ctypes.c_void_p(host_labels.ctypes.data), device.index or 0,
                                 ctypes.byref(h)), "ivf build")
    build_s = time.time() - t0
    queries = make_queries(nq, IVF_COMPS)
    ids = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.int32)
    st = Stats()

    def step():
        check(L, L.mdh_ivf_search_u8(h, ctypes.c_void_p(queries.ctypes.data), nq, k, IVF_NPROBE,
                                     ctypes.c_void_p(ids.ctypes.data), ctypes.c_void_p(dist.ctypes.data),
                                     ctypes.byref(st)), "ivf search")

    for _ in range(warmup):
        step()
    sampler = ClockSampler(device.index or 0)
    sampler.start()
    scan_ms, pairs = [], []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
        scan_ms.append(st.full_scan_ms)
        pairs.append(st.full_scan_pairs)
    elapsed = time.perf_counter() - t0
    clocks = sampler.stop()
    launches = int(st.kernel_launches) * args.steps
    ivf_block = {"blocks_tested": int(st.blocks_tested), "blocks_passed": int(st.blocks_passed),
                 "pass_rate": (st.blocks_passed / st.blocks_tested) if st.blocks_tested else None,
                 "pairs_pruned_by_bound": int(st.pairs_pruned_by_bound), "pairs_scanned": int(st.pairs_scored),
                 "final_candidates": int(st.candidates), "block": "(query, 32-row chunk) of a probed cell, all passes"}
    # Recall of the clustered search against the exact scan, on 1,000 queries.
    m = min(nq, 1000)
    flat = ctypes.c_void_p()
    check(L, L.mdh_index_create_u8(ctypes.c_void_p(host_rows.ctypes.data), n, DIM, 1, None, 0, 0, ctypes.byref(flat)),
          "flat build")
    fids = np.empty((m, k), np.int32)
    check(L, L.mdh_search_u8(flat, ctypes.c_void_p(queries.ctypes.data), m, k, ctypes.c_void_p(fids.ctypes.data),
                             None, None), "flat search")
    check(L, L.mdh_index_destroy(flat), "flat destroy")
    recall = float(np.mean([len(set(ids[i]) & set(fids[i])) / k for i in range(m)]))
    # Bytes pass 2 must stream: each unit (one cell, up to 128 of the queries
    # probing it) reads the cell's padded rows once.
    cells = np.empty((nq, IVF_NPROBE), np.int32)
    check(L, L.mdh_ivf_route_u8(h, ctypes.c_void_p(queries.ctypes.data), nq, IVF_NPROBE,
                                ctypes.c_void_p(cells.ctypes.data)), "ivf route")
    cell_rows = np.empty(IVF_NLIST, np.int64)
    check(L, L.mdh_ivf_info(h, None, None, None, ctypes.c_void_p(cell_rows.ctypes.data)), "ivf info")
    q_per_cell = np.bincount(cells.ravel(), minlength=IVF_NLIST)
    unit_rows = int(np.sum(-(-q_per_cell // 128) * (-(-cell_rows // 256)) * 256))
    pass2_bytes = unit_rows * DIM
    check(L, L.mdh_ivf_destroy(h), "ivf destroy")
    peaks, peak_src = measured_peaks()
    int8_peak = 2.0 * peaks["bf16_tflops"]
    ms = statistics.median(scan_ms)
    achieved = 2.0 * pairs[0] * DIM / (ms / 1e3) / 1e12 if ms > 0 else None
    qps = nq * args.steps / elapsed
    line = {
        "metric": f"queries/sec, {n // 1_000_000}M x {DIM} u8 IVF (nlist {IVF_NLIST}, nprobe {IVF_NPROBE}) "
                  f"exact top-{k} over the probed cells, {nq}-query batch",
        "value": qps, "unit": "queries/sec", "n_gpus": 1, "steps": args.steps, "warmup": warmup,
        "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": f"IVF: {n} x {DIM} u8 clipped-GMM ({IVF_COMPS} comps), nlist {IVF_NLIST}, "
                               f"nprobe {IVF_NPROBE}, {nq} queries, k={k}",
                   "centroids": "MiniBatchKMeans on a 200,000-row sample (n_init 1, max_iter 20); labels = nearest "
                                "centroid", "recall_at_k_vs_exact": recall, "cluster_s": round(cluster_s, 1),
                   "index_build_s": round(build_s, 2),
                   "l2_flush": f"inputs larger than L2 (cells {n * DIM / 1e9:.2f} GB)",
                   "timing": "wall clock around the host-buffer call (queries in, ids and distances out)"},
        "e2e": {"value": qps, "unit": "queries/sec", "h2d_bytes_per_step": int(nq * DIM),
                "d2h_bytes_per_step": int(nq * k * 8)},
        "gpu_launches": launches,
        "stages_ms": {"route_and_plan": round(st.prep_ms, 3), "passes_0_1": round(st.sample_ms, 3),
                      "pass_2_scan_and_rekey": round(st.full_scan_ms, 3), "select": round(st.select_ms, 3),
                      "call_wall": round(st.latency_ms, 3),
                      "note": "last timed step; CUDA events per stage inside the library; route_and_plan includes "
                              "the query upload"},
        "block_bound": ivf_block,
        "clocks": clocks,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOP/s",
                     "frac": (achieved / int8_peak) if achieved else None, "traffic": None,
                     "kernel": "pass-2 scan over the probed cells (k_filter_tc_u8_l2, unit table) and its "
                               "re-key pass (k_rekey_chunks)",
                     "algorithmic": "2 * (query, row) pairs of the probed cells * D",
                     "peak_source": f"2 x {peak_src} bf16 dense ({peaks['bf16_tflops']} TF/s)", "kernel_ms": ms,
                     "hbm": {"achieved": pass2_bytes / (ms / 1e3) / 1e9 if ms > 0 else None,
                             "peak": peaks["hbm_gbs"], "unit": "GB/s",
                             "frac": (pass2_bytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]) if ms > 0 else None,
                             "bytes_per_launch": pass2_bytes,
                             "algorithmic": "sum over units of the cell's padded rows x 128 B (each unit streams "
                                            "its cell once)"}},
    }
    emit(line)


# --------------------------------------------------------------------------- index files
def run_persist(args, torch, device, L):
    """Index files: build a 10M x 128 u8 index from host rows, save it, load it
    back twice (from the disk after dropping the file's cached pages, then from
    the page cache) and check that the loaded index answers 1,000 queries
    exactly as the built one."""
    import shutil
    import tempfile

    n = args.n if args.n != N_DEFAULT else 10_000_000
    rows = make_rows_gpu(torch, 0, n, device, args.comps)
    host = rows.cpu().numpy()
    del rows
    torch.cuda.empty_cache()
    h = ctypes.c_void_p()
    t0 = time.perf_counter()
    check(L, L.mdh_index_create_u8(ctypes.c_void_p(host.ctypes.data), n, DIM, 1, None, 0, 0, ctypes.byref(h)), "build")
    build_s = time.perf_counter() - t0
    tmp = tempfile.mkdtemp(prefix="mdh_index_")
    path = os.path.join(tmp, "index.mdh")
    try:
        t0 = time.perf_counter()
        check(L, L.mdh_index_save(h, path.encode()), "save")
        save_s = time.perf_counter() - t0
        size = os.path.getsize(path)
        # The storage ceiling: the same file read by 8 threads in 8 MB pieces
        # (the library's own I/O shape) into host memory, after dropping its
        # cached pages, then again from the page cache.
        raw = [plain_read_seconds(path, size), plain_read_seconds(path, size, drop=False)]
        loads = []
        for i in range(2):
            if i == 0:
                drop_cached_pages(path)
            h2 = ctypes.c_void_p()
            t0 = time.perf_counter()
            check(L, L.mdh_index_load(path.encode(), None, 0, ctypes.byref(h2)), "load")
            loads.append(time.perf_counter() - t0)
            if len(loads) < 2:
                check(L, L.mdh_index_destroy(h2), "destroy")
        m = 1000
        queries = make_queries(m, args.comps)
        out = []
        for hx in (h, h2):
            ids = np.empty((m, args.k), np.int32)
            dd = np.empty((m, args.k), np.int32)
            check(L, L.mdh_search_u8(hx, ctypes.c_void_p(queries.ctypes.data), m, args.k,
                                     ctypes.c_void_p(ids.ctypes.data), ctypes.c_void_p(dd.ctypes.data), None), "search")
            out.append((ids, dd))
        same = bool(np.array_equal(out[0][0], out[1][0]) and np.array_equal(out[0][1], out[1][1]))
        check(L, L.mdh_index_destroy(h2), "destroy")
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    check(L, L.mdh_index_destroy(h), "destroy")
    line = {
        "metric": f"index file load throughput, {n // 1_000_000}M x {DIM} u8 (file bytes / load time)",
        "value": size / loads[0] / 1e9, "unit": "GB/s", "n_gpus": 1, "steps": 1, "warmup": 0,
        "higher_is_better": True, "dtype": "u8", "data": "synthetic",
        "config": {"workload": f"{n} x {DIM} u8 clipped-GMM ({args.comps} comps) index: build from host rows, "
                               f"save, load", "file_bytes": size, "build_from_host_s": round(build_s, 3),
                   "save_s": round(save_s, 3), "save_GBps": round(size / save_s / 1e9, 2),
                   "load_after_page_drop_s": round(loads[0], 3), "load_page_cache_s": round(loads[1], 3),
                   "load_page_cache_GBps": round(size / loads[1] / 1e9, 2),
                   "plain_read_after_page_drop_GBps": round(size / raw[0] / 1e9, 2),
                   "plain_read_page_cache_GBps": round(size / raw[1] / 1e9, 2),
                   "loaded_index_equals_built": same,
                   "timing": "wall clock around each C-ABI call; save includes fsync; the first load follows "
                             "POSIX_FADV_DONTNEED on the file"},
    }
    line["roofline"] = {"bound": "storage read", "achieved": size / loads[0] / 1e9,
                        "peak": size / raw[0] / 1e9, "unit": "GB/s", "frac": raw[0] / loads[0], "traffic": size,
                        "peak_source": "plain 8-thread read of the same file after dropping its cached pages"}
    emit(line)
    if not same:
        raise SystemExit("loaded index answered differently from the built index")


def drop_cached_pages(path):
    fd = os.open(path, os.O_RDONLY)
    try:
        os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
    finally:
        os.close(fd)


def plain_read_seconds(path, size, drop=True, lanes=8, piece=8 << 20):
    """Seconds to read a file into host memory with `lanes` threads taking
    `piece`-byte pieces in turn (no GPU work)."""
    if drop:
        drop_cached_pages(path)
    bufs = [bytearray(piece) for _ in range(lanes)]
    fd = os.open(path, os.O_RDONLY)

    def lane(t):
        mv = memoryview(bufs[t])
        for off in range(t * piece, size, lanes * piece):
            got = 0
            want = min(piece, size - off)
            while got < want:
                r = os.preadv(fd, [mv[got:want]], off + got)
                if r <= 0:
                    raise OSError("short read")
                got += r

    try:
        t0 = time.perf_counter()
        th = [threading.Thread(target=lane, args=(t,)) for t in range(lanes)]
        for x in th:
            x.start()
        for x in th:
            x.join()
        return time.perf_counter() - t0
    finally:
        os.close(fd)


# --------------------------------------------------------------------------- float cosine workload
COS_DIM, COS_COMPS = 768, 1024


def make_cos_rows_gpu(torch, n, device, seed):
    """Row-normalized isotropic Gaussian mixture (1,024 unit-normalized random
    means, component std 0.3), float32 [n][768], generated on the GPU."""
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 11)
    means = torch.randn((COS_COMPS, COS_DIM), generator=g, device=device)
    means /= means.norm(dim=1, keepdim=True)
    out = torch.empty((n, COS_DIM), dtype=torch.float32, device=device)
    g.manual_seed(seed)
    step = 1_000_000
    for s in range(0, n, step):
        e = min(n, s + step)
        lab = torch.randint(0, COS_COMPS, (e - s,), generator=g, device=device)
        x = means[lab] + 0.3 * torch.randn((e - s, COS_DIM), generator=g, device=device)
        out[s:e] = x / x.norm(dim=1, keepdim=True)
    return out


def run_cos(args, torch, device, L, warmup):
    """Float32 cosine (SpeedEngine cosine semantics) over 10M x 768, batch
    4,096, k=10: bf16 tcgen05 pass + exact fp32 rescore."""
    n = args.n if args.n != N_DEFAULT else 10_000_000
    nq = args.nq if args.nq != 10_000 else 4096
    k = args.k
    rows = make_cos_rows_gpu(torch, n, device, SEED + 12).cpu().numpy()
    queries = make_cos_rows_gpu(torch, nq, device, SEED + 13).cpu().numpy()
    torch.cuda.empty_cache()
    check(L, L.mdh_set_scan_path(args.scan_path), "set_scan_path")
    check(L, L.mdh_set_sample_ratio(args.sample_ratio), "set_sample_ratio")
    h = ctypes.c_void_p()
    t0 = time.time()
    check(L, L.mdh_index_create_f32(ctypes.c_void_p(rows.ctypes.data), n, COS_DIM, 0, None, 0, 0, ctypes.byref(h)),
          "index build")
    build_s = time.time() - t0
    del rows
    ids = np.empty((nq, k), np.int32)
    score = np.empty((nq, k), np.float32)
    st = Stats()

    def step():
        check(L, L.mdh_search_f32(h, ctypes.c_void_p(queries.ctypes.data), nq, k, 2, ctypes.c_void_p(ids.ctypes.data),
                                  ctypes.c_void_p(score.ctypes.data), ctypes.byref(st)), "search")

    for _ in range(warmup):
        step()
    sampler = ClockSampler(device.index or 0)
    sampler.start()
    scan_ms, pairs = [], []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
        scan_ms.append(st.full_scan_ms)
        pairs.append(st.full_scan_pairs)
    elapsed = time.perf_counter() - t0
    clocks = sampler.stop()
    check(L, L.mdh_index_destroy(h), "destroy")
    peaks, peak_src = measured_peaks()
    ms = statistics.median(scan_ms)
    achieved = 2.0 * pairs[0] * COS_DIM / (ms / 1e3) / 1e12 if ms > 0 else None
    qps = nq * args.steps / elapsed
    cos_stages = {"prep": round(st.prep_ms, 3), "samples": round(st.sample_ms, 3),
                  "full_scan": round(st.full_scan_ms, 3), "rescore_in_full_scan": round(st.rescore_ms, 3),
                  "select": round(st.select_ms, 3), "call_wall": round(st.latency_ms, 3),
                  "final_candidates": int(st.candidates), "sample_ratio": args.sample_ratio or 8,
                  "note": "last timed step; CUDA events per stage, prep includes the host query normalization"}
    path = {0: "CUDA cores (fp32 replica)", 3: "bf16 tcgen05 pass + exact fp32 rescore"}.get(int(st.tensor_core_path),
                                                                                           str(st.tensor_core_path))
    line = {
        "metric": f"queries/sec, {n // 1_000_000}M x {COS_DIM} f32 cosine top-{k}, {nq}-query batch",
        "value": qps, "unit": "queries/sec", "n_gpus": 1, "steps": args.steps, "warmup": warmup,
        "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (bf16 tensor pass, fp32 rescore)", "data": "synthetic",
        "config": {"workload": f"{n} x {COS_DIM} f32 row-normalized GMM ({COS_COMPS} comps, std 0.3), {nq} queries, "
                               f"k={k}, SpeedEngine cosine semantics", "scan": path,
                   "index_build_s": round(build_s, 1), "levels": int(st.levels),
                   "l2_flush": f"inputs larger than L2 (bf16 rows {n * COS_DIM * 2 / 1e9:.1f} GB)",
                   "timing": "wall clock around the host-buffer call (queries in, ids and scores out)"},
        "e2e": {"value": qps, "unit": "queries/sec", "h2d_bytes_per_step": int(nq * COS_DIM * 4),
                "d2h_bytes_per_step": int(nq * k * 8)},
        "gpu_launches": int(st.kernel_launches) * args.steps,
        "stages_ms": cos_stages,
        "clocks": clocks,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": (achieved / peaks["bf16_tflops"]) if achieved else None, "traffic": None,
                     "kernel": "full-corpus scan (k_filter_tc_bf16_cos + k_rescore_speed_cos)",
                     "algorithmic": "2*N*Q*D flop per launch", "peak_source": f"{peak_src} bf16 dense",
                     "kernel_ms": ms},
    }
    emit(line)


# --------------------------------------------------------------------------- result checks
def result_digest(dist_arr, ids_arr):
    """sha256 (first 16 hex digits) of the [Q][k] int32 distances then ids."""
    import hashlib

    h = hashlib.sha256()
    h.update(np.ascontiguousarray(dist_arr, dtype=np.int32).tobytes())
    h.update(np.ascontiguousarray(ids_arr, dtype=np.int32).tobytes())
    return h.hexdigest()[:16]


def check_parity(torch, device, args, queries, res_d, res_i):
    """Check `--parity-queries` of the timed queries (spread over the batch)
    against the oracle's exact int64 top-k over the whole corpus.  The corpus
    is regenerated slice by slice on this GPU (the same rows the index was
    built from) and folded into the oracle's running top-k on the host."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # test infrastructure: the checker, outside the timed region

    m = max(1, min(args.parity_queries, args.nq))
    pick = np.unique(np.linspace(0, args.nq - 1, m).astype(np.int64))
    t0 = time.perf_counter()
    ref = oracle.L2TopK(queries[pick], args.k)
    step = 4 * CHUNK
    for s0 in range(0, args.n, step):
        e0 = min(args.n, s0 + step)
        rows = make_rows_gpu(torch, s0, e0, device, args.comps).cpu().numpy()
        ref.update(rows, s0)
        del rows
    torch.cuda.empty_cache()
    got_i, got_d = res_i[pick], res_d[pick]
    bad = [int(q) for j, q in enumerate(pick)
           if not (np.array_equal(got_i[j], ref.ids[j]) and np.array_equal(got_d[j], ref.dist[j]))]
    return {"queries": int(len(pick)), "match": not bad, "mismatched_queries": bad[:8],
            "oracle": "oracle.L2TopK: int64 (distance, id) ranking of MadhavaL2::search_exact over every row",
            "seconds": round(time.perf_counter() - t0, 1)}


# --------------------------------------------------------------------------- output
_RESULT_OUT = None  # the process's original stdout, kept for the result line


def keep_stdout_for_result():
    """From here on the result line is the only output on stdout: file
    descriptor 1 is pointed at stderr, so NCCL's banner, library messages and
    prints all go there, and emit() writes to a duplicate of the original."""
    global _RESULT_OUT
    try:
        sys.stdout.flush()
        _RESULT_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)
    except OSError:
        _RESULT_OUT = None


def emit(line):
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


# --------------------------------------------------------------------------- main
def main():
    keep_stdout_for_result()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--n", type=int, default=N_DEFAULT)
    ap.add_argument("--nq", type=int, default=10_000)
    ap.add_argument("--k", type=int, default=10)
    ap.add_argument("--comps", type=int, default=COMPONENTS, help="mixture components of the synthetic corpus")
    ap.add_argument("--scan-path", type=int, default=0, help="0 auto, 1 CUDA cores, 2 tensor cores")
    ap.add_argument("--cpu-slice", type=int, default=4_000_000)
    ap.add_argument("--cpu-queries", type=int, default=16)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the oracle check of the timed results (flat workload)")
    ap.add_argument("--parity-queries", type=int, default=16)
    ap.add_argument("--no-coop", action="store_true",
                    help="N > 1: each rank uses its own sample thresholds (no exchange of sample results)")
    ap.add_argument("--sample-ratio", type=int, default=0,
                    help="largest sample = shard / ratio (0 = the library default)")
    ap.add_argument("--workload", default="flat", choices=["flat", "ivf", "cos", "persist"],
                    help="flat: exact u8 L2 scan (the headline); ivf: clustered search (nlist 1024, nprobe 16); "
                         "cos: float32 cosine scan (10M x 768, 4,096 queries); persist: index file save/load "
                         "(10M x 128)")
    args = ap.parse_args()
    warmup = max(3, args.warmup)

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n_gpus = max(args.gpus, world)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    queries = make_queries(args.nq, args.comps)
    config = {"workload": f"{args.n // 1_000_000}M x {DIM} u8 clipped-GMM ({args.comps} comps), {args.nq} queries, "
                          f"exact top-{args.k} L2",
              "n": args.n, "dim": DIM, "nq": args.nq, "k": args.k,
              "parallelism": f"row-shard x{n_gpus} + NCCL all_gather of top-k"}
    # A corpus under twice the L2 could be served from L2 across steps: then
    # a buffer larger than L2 is written before every timed step, outside the
    # timed interval.
    shard_bytes = (args.n + n_gpus - 1) // n_gpus * DIM
    small_corpus = shard_bytes < 2 * L2_BYTES
    if small_corpus:
        config["l2_flush"] = (f"{L2_FLUSH_BYTES >> 20} MB buffer written before each timed step, outside the timed "
                              f"interval (corpus {shard_bytes / 1e6:.0f} MB per rank < 2 x L2)")
    else:
        config["l2_flush"] = f"inputs larger than L2 (corpus {shard_bytes / 1e9:.1f} GB per rank per step)"

    if args.impl == "reference":
        if rank != 0:
            if dist is not None:
                dist.destroy_process_group()
            return
        n_slice = min(args.cpu_slice, args.n)
        rows = make_rows_gpu(torch, 0, n_slice, device, args.comps).cpu().numpy()
        qps, cb = cpu_reference_qps(rows, args.n, queries[:args.cpu_queries], args.k, steps=args.steps,
                                    warmup=min(warmup, 1))
        line = {"metric": METRIC, "value": qps, "unit": "queries/sec", "n_gpus": n_gpus, "steps": args.steps,
                "warmup": warmup, "ms_per_step": cb["seconds_per_step"] * 1e3, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
                "impl": "reference", "cpu_baseline": cb,
                "e2e": {"value": qps, "unit": "queries/sec", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        emit(line)
        if dist is not None:
            dist.destroy_process_group()
        return

    L = load_lib()
    if args.workload == "ivf":
        run_ivf(args, torch, device, L, warmup)
        return
    if args.workload == "cos":
        run_cos(args, torch, device, L, warmup)
        return
    if args.workload == "persist":
        run_persist(args, torch, device, L)
        return
    sys.path.insert(0, os.path.join(ROOT, "winnex-madhava_b200"))
    from winnex_madhava.sharding import cooperative_topk, device_phases, gather_topk, merge_topk_device, row_range

    check(L, L.mdh_set_scan_path(args.scan_path), "set_scan_path")
    # With G ranks sharing their sample results, each rank samples 1/G of what
    # it would alone for the same threshold: its largest sample is shard/(16 G).
    coop = world > 1 and not args.no_coop
    ratio = args.sample_ratio
    check(L, L.mdh_set_sample_ratio(ratio), "set_sample_ratio")
    check(L, L.mdh_set_threshold_sharing(world if coop else 1), "set_threshold_sharing")
    config["threshold_exchange"] = ("each rank scans its samples, the ranks all_gather and merge their sample top-k "
                                    "lists, every rank scans its shard under the merged k-th distance, then the "
                                    "final lists are all_gathered and merged" if coop else "none")
    config["sample_ratio"] = ratio or 8
    start, end = row_range(args.n, rank, world)
    flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device) if small_corpus else None
    rows = make_rows_gpu(torch, start, end, device, args.comps)
    torch.cuda.synchronize()
    h = ctypes.c_void_p()
    t0 = time.time()
    check(L, L.mdh_index_create_u8_device(ctypes.c_void_p(rows.data_ptr()), end - start, DIM, 1, start,
                                          ctypes.byref(h)), "index build")
    build_s = time.time() - t0
    del rows
    torch.cuda.empty_cache()

    nq, k = args.nq, args.k
    dq = torch.from_numpy(queries).to(device)
    ids = torch.empty((nq, k), dtype=torch.int32, device=device)
    dd = torch.empty((nq, k), dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)
    sp = ctypes.c_void_p(stream.cuda_stream)
    st = Stats()
    st1 = Stats()  # the sample phase of a cooperative search
    scan_ms, scan_pairs, launches, stages, blocks = [], [], [], [], []
    merge = lambda d, i: merge_topk_device(L, d, i, stream)  # noqa: E731
    if coop:
        sample_phase = device_phases(L, h, dq, stream, ctypes.byref(st1))[0]
        bounded_phase = device_phases(L, h, dq, stream, ctypes.byref(st))[1]

    def search(q):
        if coop:
            return cooperative_topk(sample_phase, bounded_phase, merge, q, k)
        check(L, L.mdh_search_u8_device(h, ctypes.c_void_p(q.data_ptr()), nq, k, ctypes.c_void_p(ids.data_ptr()),
                                        ctypes.c_void_p(dd.data_ptr()), sp, ctypes.byref(st)), "search")
        if world > 1:
            return merge(*gather_topk(dd, ids))
        return dd, ids

    def step(record):
        out = search(dq)
        if record:
            scan_ms.append(st.full_scan_ms)
            scan_pairs.append(st.full_scan_pairs)
            # + the merge kernels (two with shared thresholds)
            launches.append(st.kernel_launches + st1.kernel_launches + (0 if world == 1 else (2 if coop else 1)))
            stages.append({"prep": st.prep_ms + st1.prep_ms,
                           "samples": (st1.sample_ms + st1.full_scan_ms + st1.select_ms) if coop else st.sample_ms,
                           "full_scan": st.full_scan_ms, "select": st.select_ms})
            blocks.append((st.blocks_tested + st1.blocks_tested, st.blocks_passed + st1.blocks_passed,
                           st.pairs_pruned_by_bound + st1.pairs_pruned_by_bound, st.pairs_scored + st1.pairs_scored,
                           st.candidates))
        return out

    for _ in range(warmup):
        step(False)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    result = None
    if flush_buf is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            result = step(True)
        e1.record(stream)
        torch.cuda.synchronize()
        elapsed = e0.elapsed_time(e1) / 1e3
    else:
        evs = []
        for i in range(args.steps):
            flush_buf.fill_(i & 255)
            a_ev, b_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a_ev.record(stream)
            result = step(True)
            b_ev.record(stream)
            evs.append((a_ev, b_ev))
        torch.cuda.synchronize()
        elapsed = sum(a_ev.elapsed_time(b_ev) for a_ev, b_ev in evs) / 1e3
    clocks = sampler.stop()
    if dist is not None:
        t = torch.tensor([elapsed], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
        dist.barrier()
    tensor_path = bool(st.tensor_core_path)
    levels = int(st.levels + st1.levels)
    # The timed steps' merged result, identical for every GPU count: its digest
    # goes into the line so runs at different N can be compared.
    res_d = result[0].cpu().numpy()
    res_i = result[1].cpu().numpy()
    digest = result_digest(res_d, res_i)

    # End to end through the C ABI with host buffers (pinned queries in, ids out).
    hq = torch.from_numpy(queries).pin_memory()
    hid = torch.empty((nq, k), dtype=torch.int32).pin_memory()
    hdist = torch.empty((nq, k), dtype=torch.int32).pin_memory()
    e2e_steps = max(1, min(args.steps, 3))

    def e2e_step():
        if world == 1:
            check(L, L.mdh_search_u8(h, ctypes.c_void_p(hq.data_ptr()), nq, k, ctypes.c_void_p(hid.data_ptr()),
                                     ctypes.c_void_p(hdist.data_ptr()), None), "e2e search")
            return
        # The sharded public path: queries from pinned host memory to this
        # rank's GPU, the search with its exchanges, the merged result back.
        q = hq.to(device, non_blocking=True)
        out_d, out_i = search(q)
        hid.copy_(out_i)
        hdist.copy_(out_d)

    e2e_step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    torch.cuda.synchronize()
    e2e_t = time.perf_counter() - t0
    if dist is not None:
        t = torch.tensor([e2e_t], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_t = float(t.item())

    peaks, peak_src = measured_peaks()
    ms_scan = statistics.median(scan_ms) if scan_ms else float("nan")
    pairs = scan_pairs[0] if scan_pairs else 0
    rows_scanned = pairs // nq if nq else 0
    int8_peak = 2.0 * peaks["bf16_tflops"]
    # Which roof bounds the scan: it does 2*Q int ops per corpus byte, so
    # below the ridge point (peak ops / peak bytes) it is HBM-bound.
    hbm_bound = 2.0 * nq < int8_peak * 1e12 / (peaks["hbm_gbs"] * 1e9)
    kernel_name = "k_filter_tc_u8_l2" if tensor_path else "k_scan_stream_u8"
    if not hbm_bound:
        # Batched path: u8 x u8 -> s32 on tcgen05, compute-bound at 2*N*Q*D ops.
        achieved = 2.0 * pairs * DIM / (ms_scan / 1e3) / 1e12 if ms_scan > 0 else None
        # DRAM traffic of the scan: ncu capture of the same kernel on a
        # 10M-row case (dram__bytes_read.sum + dram__bytes_write.sum =
        # 1.3234e9 B per launch for 10,000 queries); the corpus and norms cross
        # HBM once per launch, so traffic scales with the rows scanned.
        traffic = TRAFFIC_BYTES_PER_ROW * rows_scanned if pairs else None
        roofline = {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOP/s",
                    "frac": (achieved / int8_peak) if achieved else None, "traffic": traffic,
                    "traffic_source": "ncu dram bytes of a 10M-row launch, scaled by rows (profiles/)",
                    "kernel": f"full-corpus u8 L2 scan (filter) kernel, {kernel_name}",
                    "algorithmic": "2*N*Q*D int8 ops per launch",
                    "peak_source": f"2 x {peak_src} bf16 dense ({peaks['bf16_tflops']} TF/s): u8 MMA runs at twice "
                                   "the bf16 rate on sm_100",
                    "kernel_ms": ms_scan}
    else:
        # Small batches (the single-query GEMV end): bound by reading the u8
        # corpus (N*D bytes per launch) from HBM.
        bytes_alg = rows_scanned * DIM
        achieved = bytes_alg / (ms_scan / 1e3) / 1e9 if ms_scan > 0 else None
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": (achieved / peaks["hbm_gbs"]) if achieved else None,
                    "traffic": rows_scanned * (DIM + 4) if pairs else None,
                    "traffic_source": "corpus + norms once per launch (rows x (D + 4) B)",
                    "kernel": f"full-corpus u8 L2 scan (filter) kernel, {kernel_name}",
                    "algorithmic": "N*D corpus bytes per launch",
                    "peak_source": f"{peak_src} HBM copy bandwidth (read + write)",
                    "kernel_ms": ms_scan}
    line = {
        "metric": METRIC,
        "value": nq * args.steps / elapsed,
        "unit": "queries/sec",
        "n_gpus": n_gpus,
        "steps": args.steps,
        "warmup": warmup,
        "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "u8",
        "data": "synthetic",
        "config": dict(config, scan=("tcgen05 tensor cores" if tensor_path else "CUDA cores (dp4a)"),
                       levels=levels, index_build_s=round(build_s, 2)),
        "e2e": {"value": nq * e2e_steps / e2e_t, "unit": "queries/sec", "h2d_bytes_per_step": int(nq * DIM),
                "d2h_bytes_per_step": int(nq * k * 8)},
        "gpu_launches": int(sum(launches)),
        "clocks": clocks,
        "roofline": roofline,
    }
    st_med = {key: statistics.median(x[key] for x in stages) for key in stages[0]} if stages else {}
    line["stages_ms"] = dict({key: round(v, 3) for key, v in st_med.items()},
                             step=round(elapsed / args.steps * 1e3, 3),
                             note="CUDA events per stage inside the library, median over the timed steps "
                                  "(rank 0); step = the device-timed step")
    if blocks:
        bt, bp, pruned, scored, cand = blocks[-1]
        line["block_bound"] = {"blocks_tested": int(bt), "blocks_passed": int(bp),
                               "pass_rate": (bp / bt) if bt else None, "pairs_pruned_by_bound": int(pruned),
                               "pairs_scanned": int(scored), "final_candidates": int(cand),
                               "block": "(query, 64-row block) of a norm-sorted level, every level"}
    line["result_digest"] = digest
    check(L, L.mdh_index_destroy(h), "destroy")
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            n_slice = min(args.cpu_slice, args.n)
            rows = make_rows_gpu(torch, 0, n_slice, device, args.comps).cpu().numpy()
            _, cb = cpu_reference_qps(rows, args.n, queries[:args.cpu_queries], k, steps=args.steps,
                                      warmup=min(warmup, 1))
            line["cpu_baseline"] = cb
        except Exception as exc:  # the baseline must not hide the GPU number
            line["cpu_baseline"] = {"value": None, "error": str(exc)[:200]}
    ok = True
    if rank == 0 and not args.no_parity:
        line["parity"] = check_parity(torch, device, args, queries, res_d, res_i)
        ok = line["parity"]["match"]
    if rank == 0:
        emit(line)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if not ok:
        raise SystemExit("parity check failed: the timed results differ from the oracle")


if __name__ == "__main__":
    main()
