"""A second, independent statement of the index-file layout (the C header
include/winnex_madhava_b200.h documents it), used to write test files and to
predict the bytes the library writes.

Header (64 bytes, little-endian): magic "MDHB200I", u32 version 1, u32 kind
(0 u8 rows, 1 float32 rows), i64 n, i32 dim, i32 row stride, i32 metric,
i32 shards, u64 data offset, u64 file size, u64 0; then one 32-byte entry per
shard {i64 rows, i64 id_base, u64 offset, u64 bytes}.  Each shard's data starts
at a 4096-aligned offset: rows [rows][stride], norms [rows], ids [rows].
"""
from __future__ import annotations

import struct

import numpy as np

MAGIC = b"MDHB200I"
ALIGN = 4096
HEAD = struct.Struct("<8sIIqiiiiQQQ")
ENTRY = struct.Struct("<qqQQ")
assert HEAD.size == 64 and ENTRY.size == 32


def _align(x: int) -> int:
    return (x + ALIGN - 1) // ALIGN * ALIGN


def stride_of(kind: int, dim: int) -> int:
    return (dim + 127) // 128 * 128 if kind == 0 else dim


def layout(kind: int, dim: int, shards):
    """shards: [(rows, id_base)] -> (data_offset, [(rows, id_base, offset, bytes)], file_size)."""
    stride = stride_of(kind, dim)
    per_row = (stride if kind == 0 else 4 * stride) + 8
    data_off = _align(64 + 32 * len(shards))
    table, at = [], data_off
    for rows, id_base in shards:
        table.append((rows, id_base, at, rows * per_row))
        at = _align(at + rows * per_row)
    size = max([data_off] + [o + b for _, _, o, b in table])
    return data_off, table, size


def header(kind: int, n: int, dim: int, metric: int, shards, version: int = 1, magic: bytes = MAGIC,
           stride: int | None = None, n_field: int | None = None) -> tuple[bytes, list, int]:
    """Header + table padded to the data offset; fields can be overridden to
    build damaged files."""
    data_off, table, size = layout(kind, dim, shards)
    h = HEAD.pack(magic, version, kind, n if n_field is None else n_field, dim,
                  stride_of(kind, dim) if stride is None else stride, metric, len(table), data_off, size, 0)
    h += b"".join(ENTRY.pack(*t) for t in table)
    return h.ljust(data_off, b"\0"), table, size


def write(path: str, kind: int, dim: int, metric: int, shards, payloads=None, **overrides) -> None:
    """Write a file; payloads[i] (bytes, optional) fills shard i's data, zeros otherwise."""
    n = sum(r for r, _ in shards)
    head, table, size = header(kind, n, dim, metric, shards, **overrides)
    buf = bytearray(size)
    buf[:len(head)] = head
    for i, (_, _, off, nbytes) in enumerate(table):
        if payloads is not None and payloads[i] is not None:
            assert len(payloads[i]) == nbytes
            buf[off:off + nbytes] = payloads[i]
    with open(path, "wb") as f:
        f.write(bytes(buf))


def u8_sections(rows_u8: np.ndarray, id_base: int) -> bytes:
    """The data a u8 shard holds: rows sorted ascending by (|v|^2, row id),
    zero padded to the stride, then int32 norms, then int32 global ids."""
    n, dim = rows_u8.shape
    norms = (rows_u8.astype(np.int64) ** 2).sum(1)
    order = np.lexsort((np.arange(n), norms))
    padded = np.zeros((n, stride_of(0, dim)), np.uint8)
    padded[:, :dim] = rows_u8[order]
    return padded.tobytes() + norms[order].astype("<i4").tobytes() + (order + id_base).astype("<i4").tobytes()


def f32_sections(rows_f32: np.ndarray, norms_f32: np.ndarray, id_base: int) -> bytes:
    """The data a float shard holds: rows and norms in id order, then ids."""
    n = rows_f32.shape[0]
    return (np.ascontiguousarray(rows_f32, "<f4").tobytes() + np.ascontiguousarray(norms_f32, "<f4").tobytes()
            + (np.arange(n) + id_base).astype("<i4").tobytes())
