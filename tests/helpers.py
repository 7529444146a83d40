"""Shared test helpers (fixture loading, ctypes access to the C ABI)."""
from __future__ import annotations

import ctypes
import json
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
PKG = os.path.join(ROOT, "winnex-madhava_b200", "winnex_madhava")
LIB = os.path.join(PKG, "libwinnex_madhava_b200.so")
HEADER = os.path.join(ROOT, "include", "winnex_madhava_b200.h")


def load_fixture(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    meta = json.loads(str(z["meta"]))
    return meta, {k: z[k] for k in z.files if k != "meta"}


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mdh_[a-z0-9_]+)\s*\(", src)))


class Stats(ctypes.Structure):
    _fields_ = [("latency_ms", ctypes.c_double), ("pairs_scored", ctypes.c_int64),
                ("pairs_pruned_by_bound", ctypes.c_int64), ("bound_violations", ctypes.c_int64),
                ("candidates", ctypes.c_int64), ("tensor_core_path", ctypes.c_int32), ("levels", ctypes.c_int32),
                ("full_scan_ms", ctypes.c_double), ("full_scan_pairs", ctypes.c_int64),
                ("kernel_launches", ctypes.c_int64), ("verified_queries", ctypes.c_int64),
                ("sample_ms", ctypes.c_double), ("select_ms", ctypes.c_double), ("rescore_ms", ctypes.c_double),
                ("prep_ms", ctypes.c_double), ("blocks_tested", ctypes.c_int64), ("blocks_passed", ctypes.c_int64)]


class Audit(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int64), ("within", ctypes.c_int64), ("excluded", ctypes.c_int64),
                ("excluded_by_bound", ctypes.c_int64), ("violations", ctypes.c_int64), ("threshold", ctypes.c_double),
                ("n_records", ctypes.c_int32), ("reserved", ctypes.c_int32)]


def capi():
    L = ctypes.CDLL(LIB)
    P, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    L.mdh_index_create_u8.argtypes = [P, i64, i32, i32, P, i32, i64, ctypes.POINTER(P)]
    L.mdh_index_create_f32.argtypes = [P, i64, i32, i32, P, i32, i64, ctypes.POINTER(P)]
    L.mdh_index_create_u8_device.argtypes = [P, i64, i32, i32, i64, ctypes.POINTER(P)]
    L.mdh_index_destroy.argtypes = [P]
    L.mdh_index_info.argtypes = [P, P, P, P, P]
    L.mdh_search_f32.argtypes = [P, P, i32, i32, i32, P, P, ctypes.POINTER(Stats)]
    L.mdh_search_u8.argtypes = [P, P, i32, i32, P, P, ctypes.POINTER(Stats)]
    L.mdh_audit_f32.argtypes = [P, P, i32, i32, i32, P, P, P, P, P, ctypes.POINTER(Stats)]
    L.mdh_audit_u8.argtypes = [P, P, i32, i32, i32, P, P, P, P, P, ctypes.POINTER(Stats)]
    L.mdh_search_u8_device.argtypes = [P, P, i32, i32, P, P, P, ctypes.POINTER(Stats)]
    L.mdh_search_u8_device_noalloc.argtypes = [P, P, i32, i32, P, P, P, ctypes.POINTER(Stats)]
    L.mdh_search_u8_device_sample.argtypes = [P, P, i32, i32, P, P, P, ctypes.POINTER(Stats)]
    L.mdh_search_u8_device_bounded.argtypes = [P, P, i32, i32, P, P, P, P, P, ctypes.POINTER(Stats)]
    L.mdh_merge_topk_device.argtypes = [P, P, i32, i32, i32, P, P, P]
    L.mdh_ivf_create_u8.argtypes = [P, i64, i32, P, i32, P, i32, ctypes.POINTER(P)]
    L.mdh_ivf_create_u8_metric.argtypes = [P, i64, i32, P, i32, P, i32, i32, ctypes.POINTER(P)]
    L.mdh_ivf_route_u8.argtypes = [P, P, i32, i32, P]
    L.mdh_ivf_search_u8.argtypes = [P, P, i32, i32, i32, P, P, ctypes.POINTER(Stats)]
    L.mdh_ivf_info.argtypes = [P, P, P, P, P]
    L.mdh_ivf_destroy.argtypes = [P]
    L.mdh_ivf_create_f32.argtypes = [P, i64, i32, P, i32, P, i32, ctypes.POINTER(P)]
    L.mdh_ivf_search_f32.argtypes = [P, P, i32, i32, i32, P, P, ctypes.POINTER(Stats)]
    L.mdh_ivf_destroy_f32.argtypes = [P]
    L.mdh_index_save.argtypes = [P, ctypes.c_char_p]
    L.mdh_index_load.argtypes = [ctypes.c_char_p, P, i32, ctypes.POINTER(P)]
    L.mdh_index_file_info.argtypes = [ctypes.c_char_p, P, P, P, P, P]
    L.mdh_set_scan_path.argtypes = [i32]
    L.mdh_set_verify.argtypes = [i32]
    L.mdh_set_candidate_cap_limit.argtypes = [i32]
    L.mdh_set_sample_ratio.argtypes = [i32]
    L.mdh_set_fault.argtypes = [i32]
    L.mdh_set_threshold_sharing.argtypes = [i32]
    L.mdh_check_wait_timeout.argtypes = [i32, i64]
    L.mdh_plan_level_count.argtypes = [i64, i32]
    L.mdh_plan_level_count.restype = i32
    L.mdh_index_id_base.argtypes = [P, P]
    L.mdh_index_memory.argtypes = [P, P, P]
    L.mdh_last_error.restype = ctypes.c_char_p
    L.mdh_version.restype = ctypes.c_char_p
    L.mdh_device_count.restype = i32
    for fn in ("mdh_index_create_u8", "mdh_index_create_u8_device", "mdh_index_create_f32", "mdh_index_destroy", "mdh_index_info", "mdh_search_f32",
               "mdh_search_u8", "mdh_search_u8_device", "mdh_search_u8_device_noalloc", "mdh_merge_topk_device", "mdh_set_scan_path",
               "mdh_set_verify", "mdh_ivf_create_u8", "mdh_ivf_route_u8", "mdh_ivf_search_u8", "mdh_ivf_info",
               "mdh_ivf_destroy", "mdh_index_save", "mdh_index_load", "mdh_index_file_info",
               "mdh_set_candidate_cap_limit", "mdh_set_sample_ratio", "mdh_index_id_base",
               "mdh_index_memory", "mdh_ivf_create_u8_metric", "mdh_search_u8_device_sample",
               "mdh_search_u8_device_bounded", "mdh_set_fault", "mdh_check_wait_timeout",
               "mdh_set_threshold_sharing"):
        getattr(L, fn).restype = ctypes.c_int
    return L


def ptr(a):
    """Data address of `a` for a C call.  The returned object keeps `a`
    alive, so ``ptr(np.ascontiguousarray(x))`` stays valid through the call
    even when that makes a temporary copy."""
    if a is None:
        return None
    p = ctypes.c_void_p(a.ctypes.data)
    p._keep = a
    return p


def sorted_by_key(ids, key, asc=True):
    """Re-sort ids per query by (key, id) -- the canonical tie order."""
    out = np.empty_like(ids)
    for i in range(ids.shape[0]):
        kk = key[i] if asc else -key[i]
        o = np.lexsort((ids[i], kk))
        out[i] = ids[i][o]
    return out
