"""The index-file header parser on damaged input (no GPU needed): random
byte changes in the header and shard table, and random truncations, must
give MDH_OK with a self-consistent layout or MDH_ERR_IO, never a crash."""
import ctypes

import numpy as np

import index_file
from helpers import capi

MDH_ERR_IO = 9


def _info(L, path):
    n, dim, metric, shards, isf = (ctypes.c_int64(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32(),
                                   ctypes.c_int32())
    st = L.mdh_index_file_info(path.encode(), ctypes.byref(n), ctypes.byref(dim), ctypes.byref(metric),
                               ctypes.byref(shards), ctypes.byref(isf))
    return st, (n.value, dim.value, metric.value, shards.value, isf.value)


def _accepted_layout_is_valid(raw: bytes) -> bool:
    """What an accepted file must satisfy, restated from the layout."""
    h = index_file.HEAD.unpack_from(raw, 0)
    magic, version, kind, n, dim, stride, metric, nsh, data_off, size, _ = h
    if magic != index_file.MAGIC or version != 1 or kind not in (0, 1) or metric not in (0, 1):
        return False
    if not (1 <= dim <= 4096) or stride != index_file.stride_of(kind, dim) or size != len(raw):
        return False
    per_row = (stride if kind == 0 else 4 * stride) + 8
    end, total, next_base = data_off, 0, None
    for i in range(nsh):
        rows, base, off, nbytes = index_file.ENTRY.unpack_from(raw, 64 + 32 * i)
        if rows < 0 or base < 0 or base + rows > 2**31 - 1 or nbytes != rows * per_row:
            return False
        if next_base is not None and base != next_base:  # id ranges tile one run in file order
            return False
        next_base = base + rows
        if off % 4096 or off < end or off + nbytes > len(raw):
            return False
        end, total = off + nbytes, total + rows
    return total == n and data_off % 4096 == 0


def test_header_fuzz(tmp_path):
    L = capi()
    rng = np.random.default_rng(2024)
    base = str(tmp_path / "base.idx")
    index_file.write(base, 0, 64, 1, [(7, 0), (0, 7), (5, 7)])
    good = open(base, "rb").read()
    data_off = index_file.layout(0, 64, [(7, 0), (0, 7), (5, 7)])[0]
    p = str(tmp_path / "fuzz.idx")
    accepted = rejected = 0
    for it in range(400):
        raw = bytearray(good)
        if it % 4 == 3:
            raw = raw[:int(rng.integers(0, len(raw)))]
        else:
            for _ in range(int(rng.integers(1, 4))):
                at = int(rng.integers(0, 64 + 32 * 3))
                raw[at] = int(rng.integers(0, 256))
        open(p, "wb").write(bytes(raw))
        st, got = _info(L, p)
        assert st in (0, MDH_ERR_IO), (it, st, L.mdh_last_error())
        if st == 0:
            accepted += 1
            assert len(raw) >= data_off and _accepted_layout_is_valid(bytes(raw)), it
            assert got[3] == index_file.HEAD.unpack_from(raw, 0)[7]
        else:
            rejected += 1
            assert L.mdh_last_error().startswith(b"index file ")
    assert rejected > 300 and accepted >= 1  # unchanged bytes (same value written back) are accepted


def test_shard_id_ranges_must_tile(tmp_path):
    """Shards whose id ranges overlap, leave a gap, or run out of order are
    refused; ranges that tile [first, first + n) are accepted, whatever the
    first id (a rank's slice of a larger corpus)."""
    L = capi()
    layouts = {"tiled": ([(7, 0), (0, 7), (5, 7)], 0), "offset_run": ([(4, 100), (6, 104)], 0),
               "overlap": ([(7, 0), (5, 3)], MDH_ERR_IO), "gap": ([(7, 0), (5, 9)], MDH_ERR_IO),
               "reversed": ([(5, 7), (7, 0)], MDH_ERR_IO)}
    for name, (shards, want) in layouts.items():
        p = str(tmp_path / (name + ".idx"))
        index_file.write(p, 0, 64, 1, shards)
        st, _ = _info(L, p)
        assert st == want, (name, st, L.mdh_last_error())
        if want:
            assert b"id range" in L.mdh_last_error()
