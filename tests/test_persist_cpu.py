"""Index-file header checks that need no GPU (mdh_index_file_info reads only
the header; mdh_index_load validates the header before it touches a device)."""
import ctypes
import os

import numpy as np
import pytest

import index_file
from helpers import capi

MDH_ERR_IO = 9


def _info(L, path):
    n, dim, metric, shards, isf = (ctypes.c_int64(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32(),
                                   ctypes.c_int32())
    st = L.mdh_index_file_info(path.encode(), ctypes.byref(n), ctypes.byref(dim), ctypes.byref(metric),
                               ctypes.byref(shards), ctypes.byref(isf))
    return st, (n.value, dim.value, metric.value, shards.value, isf.value)


def test_header_fields(tmp_path):
    L = capi()
    p = str(tmp_path / "a.idx")
    index_file.write(p, 0, 96, 1, [(300, 0), (0, 300), (201, 300)])
    st, got = _info(L, p)
    assert st == 0, L.mdh_last_error()
    assert got == (501, 96, 1, 3, 0)
    p2 = str(tmp_path / "b.idx")
    index_file.write(p2, 1, 768, 0, [(10, 5)])
    st, got = _info(L, p2)
    assert st == 0, L.mdh_last_error()
    assert got == (10, 768, 0, 1, 1)
    # data offsets are 4096-aligned and the file size is the end of the last shard
    _, table, size = index_file.layout(0, 96, [(300, 0), (0, 300), (201, 300)])
    assert all(off % 4096 == 0 for _, _, off, _ in table)
    assert os.path.getsize(p) == size == table[2][2] + 201 * (128 + 8)


@pytest.mark.parametrize("damage,msg", [
    ({"magic": b"WMADHAV1"}, b"bad magic"),
    ({"version": 2}, b"unsupported version"),
    ({"stride": 96}, b"row stride"),
    ({"n_field": 8}, b"do not add up"),
])
def test_damaged_headers(tmp_path, damage, msg):
    L = capi()
    p = str(tmp_path / "d.idx")
    index_file.write(p, 0, 96, 1, [(5, 0), (2, 5)], **damage)
    st, _ = _info(L, p)
    assert st == MDH_ERR_IO and msg in L.mdh_last_error(), L.mdh_last_error()
    out = ctypes.c_void_p()
    assert L.mdh_index_load(p.encode(), None, 0, ctypes.byref(out)) == MDH_ERR_IO
    assert not out.value


def test_truncated_and_padded_files(tmp_path):
    L = capi()
    p = str(tmp_path / "t.idx")
    index_file.write(p, 0, 128, 1, [(40, 0)])
    data = open(p, "rb").read()
    open(p, "wb").write(data[:-1])
    st, _ = _info(L, p)
    assert st == MDH_ERR_IO and b"truncated" in L.mdh_last_error()
    open(p, "wb").write(data + b"\0")
    st, _ = _info(L, p)
    assert st == MDH_ERR_IO and b"longer" in L.mdh_last_error()
    open(p, "wb").write(data[:40])
    st, _ = _info(L, p)
    assert st == MDH_ERR_IO and b"truncated" in L.mdh_last_error()


def test_bad_shard_table(tmp_path):
    L = capi()
    p = str(tmp_path / "s.idx")
    index_file.write(p, 0, 128, 1, [(40, 0), (8, 40)])
    raw = bytearray(open(p, "rb").read())
    # shard 1's offset moved off the 4096 grid
    e1 = 64 + 32
    good = bytes(raw)
    raw[e1 + 16:e1 + 24] = (int.from_bytes(raw[e1 + 16:e1 + 24], "little") + 8).to_bytes(8, "little")
    open(p, "wb").write(raw)
    st, _ = _info(L, p)
    assert st == MDH_ERR_IO and b"bad offset" in L.mdh_last_error()
    # shard 1's byte count disagrees with its rows
    raw = bytearray(good)
    raw[e1 + 24:e1 + 32] = (8 * 136 + 4).to_bytes(8, "little")
    open(p, "wb").write(raw)
    st, _ = _info(L, p)
    assert st == MDH_ERR_IO and b"row count" in L.mdh_last_error()
    # ids past int32
    raw = bytearray(good)
    raw[e1 + 8:e1 + 16] = (2**31 - 4).to_bytes(8, "little")
    open(p, "wb").write(raw)
    st, _ = _info(L, p)
    assert st == MDH_ERR_IO and b"int32" in L.mdh_last_error()


def test_missing_file_and_arguments(tmp_path):
    L = capi()
    st, _ = _info(L, str(tmp_path / "missing.idx"))
    assert st == MDH_ERR_IO and b"cannot open" in L.mdh_last_error()
    out = ctypes.c_void_p()
    assert L.mdh_index_load(b"", None, 0, ctypes.byref(out)) == 1
    assert L.mdh_index_load(b"x", None, 0, None) == 1
    assert L.mdh_index_save(None, b"x") == 1


def test_load_needs_a_gpu(tmp_path):
    L = capi()
    if L.mdh_device_count() > 0:
        pytest.skip("a GPU is present")
    p = str(tmp_path / "ok.idx")
    index_file.write(p, 0, 128, 1, [(16, 0)], payloads=[index_file.u8_sections(np.zeros((16, 128), np.uint8), 0)])
    out = ctypes.c_void_p()
    assert L.mdh_index_load(p.encode(), None, 0, ctypes.byref(out)) == 2
    assert b"no CUDA device" in L.mdh_last_error()
