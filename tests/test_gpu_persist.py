"""GPU tests of index files: save, load, and search the loaded index.

The file's bytes are compared with an independent statement of the layout
(tests/index_file.py: rows sorted by (|v|^2, id), norms, ids), and the
loaded index must return exactly what the saved one returned, which in turn
matches the oracle.
"""
import ctypes
import os

import numpy as np
import pytest

import cases
import index_file
import oracle
from helpers import Stats, capi, ptr

pytestmark = pytest.mark.gpu

MDH_ERR_IO = 9


def _create(L, C, metric=1, id_offset=0, devices=None, f32=False):
    h = ctypes.c_void_p()
    dev = np.asarray(devices, np.int32) if devices else None
    fn = L.mdh_index_create_f32 if f32 else L.mdh_index_create_u8
    st = fn(ptr(np.ascontiguousarray(C)), C.shape[0], C.shape[1], metric, ptr(dev), len(devices or []), id_offset,
            ctypes.byref(h))
    assert st == 0, L.mdh_last_error()
    return h


def _search_u8(L, h, Q, k):
    ids = np.empty((len(Q), k), np.int32)
    dist = np.empty((len(Q), k), np.int32)
    s = Stats()
    assert L.mdh_search_u8(h, ptr(np.ascontiguousarray(Q)), len(Q), k, ptr(ids), ptr(dist), ctypes.byref(s)) == 0, \
        L.mdh_last_error()
    return ids, dist, s


def _search_f32(L, h, Q, k, mode):
    ids = np.empty((len(Q), k), np.int32)
    val = np.empty((len(Q), k), np.float32)
    s = Stats()
    Q = np.ascontiguousarray(Q, np.float32)
    assert L.mdh_search_f32(h, ptr(Q), len(Q), k, mode, ptr(ids), ptr(val), ctypes.byref(s)) == 0, L.mdh_last_error()
    return ids, val, s


def _save(L, h, path):
    assert L.mdh_index_save(h, path.encode()) == 0, L.mdh_last_error()
    assert not os.path.exists(path + ".tmp")


def _load(L, path, devices=None):
    h = ctypes.c_void_p()
    dev = np.asarray(devices, np.int32) if devices else None
    st = L.mdh_index_load(path.encode(), ptr(dev), len(devices or []), ctypes.byref(h))
    return st, h


def test_roundtrip_u8_l2(tmp_path):
    """300K GMM rows (a chain of samples and the shard): the file holds
    the norm-sorted shard, and the loaded index answers bit for bit."""
    L = capi()
    C = cases.gmm_u8(300_000, 128, 256, seed=91)
    Q = cases.gmm_u8_queries(500, 128, 256, seed_means=91, seed_q=92)
    h = _create(L, C)
    ids0, d0, s0 = _search_u8(L, h, Q, 10)
    want_ids, want_d = oracle.l2_exact_u8_int(C, Q[:50], 10)
    np.testing.assert_array_equal(ids0[:50], want_ids)
    np.testing.assert_array_equal(d0[:50], want_d)
    path = str(tmp_path / "gmm.idx")
    _save(L, h, path)
    raw = open(path, "rb").read()
    head, table, size = index_file.header(0, len(C), 128, 1, [(len(C), 0)])
    assert len(raw) == size and raw[:len(head)] == head
    off, nbytes = table[0][2], table[0][3]
    assert raw[off:off + nbytes] == index_file.u8_sections(C, 0)
    assert L.mdh_index_destroy(h) == 0
    st, h2 = _load(L, path)
    assert st == 0, L.mdh_last_error()
    ids1, d1, s1 = _search_u8(L, h2, Q, 10)
    np.testing.assert_array_equal(ids1, ids0)
    np.testing.assert_array_equal(d1, d0)
    # The loaded index rebuilt the same samples, so it runs the same chain.
    assert s1.levels == s0.levels == L.mdh_plan_level_count(len(C), 10) >= 3
    assert s1.tensor_core_path == s0.tensor_core_path == 1
    n, dim, metric, nd = ctypes.c_int64(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    assert L.mdh_index_info(h2, ctypes.byref(n), ctypes.byref(dim), ctypes.byref(metric), ctypes.byref(nd)) == 0
    assert (n.value, dim.value, metric.value, nd.value) == (len(C), 128, 1, 1)
    # k = 100 through the large-k selection, and the float-query path
    ids_a, d_a, _ = _search_u8(L, h2, Q[:64], 100)
    want_ids, want_d = oracle.l2_exact_u8_int(C, Q[:64], 100)
    np.testing.assert_array_equal(ids_a, want_ids)
    np.testing.assert_array_equal(d_a, want_d)
    assert L.mdh_index_destroy(h2) == 0


def test_roundtrip_two_shards_cosine_dim96(tmp_path):
    """Two shards (both on this GPU), global ids offset by 1000, cosine metric,
    dim 96 (rows padded to a 128-byte stride)."""
    L = capi()
    C = cases.gmm_u8(60_001, 96, 64, seed=93)
    Q = cases.gmm_u8_queries(200, 96, 64, seed_means=93, seed_q=94)
    h = _create(L, C, metric=0, id_offset=1000, devices=[0, 0])
    ids0, sc0, _ = _search_f32(L, h, Q.astype(np.float32), 10, 0)
    path = str(tmp_path / "two.idx")
    _save(L, h, path)
    raw = open(path, "rb").read()
    half = len(C) // 2
    head, table, size = index_file.header(0, len(C), 96, 0, [(half, 1000), (len(C) - half, 1000 + half)])
    assert len(raw) == size and raw[:len(head)] == head
    for (rows, base, off, nbytes), part in zip(table, (C[:half], C[half:])):
        assert raw[off:off + nbytes] == index_file.u8_sections(part, base)
    # one device per shard, or none (every shard on the current device)
    st, bad = _load(L, path, devices=[0])
    assert st == 1 and b"one GPU per shard" in L.mdh_last_error() and not bad.value
    for devs in (None, [0, 0]):
        st, h2 = _load(L, path, devices=devs)
        assert st == 0, L.mdh_last_error()
        ids1, sc1, _ = _search_f32(L, h2, Q.astype(np.float32), 10, 0)
        np.testing.assert_array_equal(ids1, ids0)
        np.testing.assert_array_equal(sc1.view(np.uint32), sc0.view(np.uint32))
        assert L.mdh_index_destroy(h2) == 0
    want_ids, _ = oracle.cosine_exact_u8(C, Q[:40].astype(np.float32), 10)
    assert oracle.equivalent_topk("exact_cos", C, Q[:40].astype(np.float32), ids0[:40] - 1000, want_ids) == []
    assert L.mdh_index_destroy(h) == 0


def test_roundtrip_f32_l2_speed(tmp_path):
    """A float32 corpus (SpeedEngine L2 rows and norms in id order)."""
    L = capi()
    X = cases.clustered_f32(n=20_000, d=64)
    Qf = X[:30] + np.float32(0.01)
    h = _create(L, X, metric=1, f32=True)
    ids0, v0, _ = _search_f32(L, h, Qf, 10, 1)
    path = str(tmp_path / "f32.idx")
    _save(L, h, path)
    raw = open(path, "rb").read()
    head, table, size = index_file.header(1, len(X), 64, 1, [(len(X), 0)])
    assert len(raw) == size and raw[:len(head)] == head
    f, nr = oracle.speed_prepare(X, False)
    assert raw[table[0][2]:table[0][2] + table[0][3]] == index_file.f32_sections(f, nr, 0)
    st, h2 = _load(L, path)
    assert st == 0, L.mdh_last_error()
    ids1, v1, _ = _search_f32(L, h2, Qf, 10, 1)
    np.testing.assert_array_equal(ids1, ids0)
    np.testing.assert_array_equal(v1.view(np.uint32), v0.view(np.uint32))
    assert L.mdh_index_destroy(h2) == 0
    assert L.mdh_index_destroy(h) == 0


def test_load_rejects_damaged_rows(tmp_path):
    """A changed row byte, an id moved out of range, an id duplicated inside
    the range and two swapped rows each fail the load-time integrity check;
    the library stays usable afterwards."""
    L = capi()
    C = cases.gmm_u8(5_000, 128, 16, seed=95)
    h = _create(L, C)
    path = str(tmp_path / "ok.idx")
    _save(L, h, path)
    good = bytearray(open(path, "rb").read())
    _, table, _ = index_file.header(0, len(C), 128, 1, [(len(C), 0)])
    off = table[0][2]
    n = len(C)
    norms_at, ids_at = off + n * 128, off + n * 132

    def expect_rejected(raw, what):
        p = str(tmp_path / (what + ".idx"))
        open(p, "wb").write(bytes(raw))
        st, hb = _load(L, p)
        assert st == MDH_ERR_IO and b"integrity" in L.mdh_last_error(), (what, L.mdh_last_error())
        assert not hb.value

    raw = bytearray(good)
    raw[off + 77 * 128 + 5] ^= 0x01
    expect_rejected(raw, "row_byte")
    raw = bytearray(good)
    raw[ids_at + 4 * 10:ids_at + 4 * 11] = (n + 3).to_bytes(4, "little")
    expect_rejected(raw, "id_range")
    # An in-range id made equal to another row's id, at a row whose norm is
    # strictly between its neighbours' (so the (norm, id) order still holds):
    # a duplicate, caught by the permutation check.
    raw = bytearray(good)
    ids = np.frombuffer(bytes(raw[ids_at:ids_at + 4 * n]), np.int32)
    norms = np.frombuffer(bytes(raw[norms_at:norms_at + 4 * n]), np.int32)
    j = next(i for i in range(1, n - 201) if norms[i - 1] < norms[i] < norms[i + 1])
    raw[ids_at + 4 * j:ids_at + 4 * j + 4] = int(ids[j + 200]).to_bytes(4, "little")
    expect_rejected(raw, "id_duplicate")
    raw = bytearray(good)
    a, b = 100, 4000  # different norms: the order breaks
    ra, rb = bytes(raw[off + a * 128:off + (a + 1) * 128]), bytes(raw[off + b * 128:off + (b + 1) * 128])
    raw[off + a * 128:off + (a + 1) * 128], raw[off + b * 128:off + (b + 1) * 128] = rb, ra
    na, nb = bytes(raw[norms_at + 4 * a:norms_at + 4 * a + 4]), bytes(raw[norms_at + 4 * b:norms_at + 4 * b + 4])
    raw[norms_at + 4 * a:norms_at + 4 * a + 4], raw[norms_at + 4 * b:norms_at + 4 * b + 4] = nb, na
    ia, ib = bytes(raw[ids_at + 4 * a:ids_at + 4 * a + 4]), bytes(raw[ids_at + 4 * b:ids_at + 4 * b + 4])
    raw[ids_at + 4 * a:ids_at + 4 * a + 4], raw[ids_at + 4 * b:ids_at + 4 * b + 4] = ib, ia
    expect_rejected(raw, "swapped_rows")
    st, h2 = _load(L, path)
    assert st == 0, L.mdh_last_error()
    Q = C[:20]
    ids, dist, _ = _search_u8(L, h2, Q, 5)
    want_ids, want_d = oracle.l2_exact_u8_int(C, Q, 5)
    np.testing.assert_array_equal(ids, want_ids)
    np.testing.assert_array_equal(dist, want_d)
    assert L.mdh_index_destroy(h2) == 0
    assert L.mdh_index_destroy(h) == 0


def test_empty_index_roundtrip(tmp_path):
    L = capi()
    h = _create(L, np.zeros((0, 32), np.uint8))
    path = str(tmp_path / "empty.idx")
    _save(L, h, path)
    st, h2 = _load(L, path)
    assert st == 0, L.mdh_last_error()
    ids, _, _ = _search_u8(L, h2, np.zeros((2, 32), np.uint8), 3)
    assert (ids == -1).all()
    assert L.mdh_index_destroy(h2) == 0
    assert L.mdh_index_destroy(h) == 0


def test_facade_save_and_load_index(tmp_path):
    """MadhavaL2.save_index / load_index (the reference's bool API): a fresh
    engine that loads the file answers like the engine that saved it."""
    import winnex_madhava as wm
    C = cases.gmm_u8(40_000, 128, 32, seed=97)
    eng = wm.build_engine(C, dim=128, k=10, metric="l2")
    path = str(tmp_path / "facade.idx")
    assert eng.save_index(path) is True
    fresh = wm.MadhavaL2(wm.Config())
    assert fresh.built() is False
    assert fresh.load_index(path) is True
    assert fresh.built() and fresh.num_vectors() == len(C) and fresh.dim() == 128
    Q = C[:8].astype(np.float32)
    for i in range(8):
        assert fresh.search(Q[i]).indices == eng.search(Q[i]).indices
        assert fresh.search_exact(Q[i]).indices == eng.search_exact(Q[i]).indices
    assert fresh.search_batch(Q, 8, 10) == eng.search_batch(Q, 8, 10)
    # a damaged file leaves the engine unbuilt, as the reference's load_index does
    raw = bytearray(open(path, "rb").read())
    raw[:8] = b"WMADHAV1"
    bad = str(tmp_path / "bad.idx")
    open(bad, "wb").write(bytes(raw))
    assert fresh.load_index(bad) is False and fresh.built() is False


def test_roundtrip_across_devices(tmp_path):
    """Shards on two GPUs are saved and loaded back onto two GPUs (each shard's
    copies run on its own device), and onto one."""
    L = capi()
    if L.mdh_device_count() < 2:
        pytest.skip("needs two GPUs")
    C = cases.gmm_u8(80_000, 128, 64, seed=99)
    Q = cases.gmm_u8_queries(100, 128, 64, seed_means=99, seed_q=100)
    h = _create(L, C, devices=[0, 1])
    ids0, d0, _ = _search_u8(L, h, Q, 10)
    path = str(tmp_path / "two_gpus.idx")
    _save(L, h, path)
    for devs in ([1, 0], None):
        st, h2 = _load(L, path, devices=devs)
        assert st == 0, L.mdh_last_error()
        ids1, d1, _ = _search_u8(L, h2, Q, 10)
        np.testing.assert_array_equal(ids1, ids0)
        np.testing.assert_array_equal(d1, d0)
        assert L.mdh_index_destroy(h2) == 0
    assert L.mdh_index_destroy(h) == 0
