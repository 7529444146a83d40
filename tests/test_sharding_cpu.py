"""The row-sharded path's host logic on a 2-rank gloo group (CPU).

Each rank takes its rows with ``sharding.row_range``, ranks them with the
oracle under global ids, and exchanges its [Q][k] lists with
``sharding.gather_topk``; merging the gathered lists by (distance, id) must
give the single-shard oracle result exactly.  The GPU merge kernel
(mdh_merge_topk_device) is tested against the same rule in
test_gpu_capi.py.
"""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest

import cases
import oracle


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, nq, k, out):
    import torch
    import torch.distributed as dist

    from winnex_madhava.sharding import gather_topk, row_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        C = cases.gmm_u8(n, 32, 8, seed=61)
        Q = cases.gmm_u8_queries(nq, 32, 8, seed_means=61, seed_q=62)
        s, e = row_range(n, rank, world)
        ids, d = oracle.l2_exact_u8_int(C[s:e], Q, k)
        ids = np.where(ids >= 0, ids + s, -1).astype(np.int32)
        d = np.where(ids >= 0, d, -1).astype(np.int32)
        all_d, all_i = gather_topk(torch.from_numpy(d), torch.from_numpy(ids))
        if rank == 0:
            np.savez(out, d=all_d.numpy(), i=all_i.numpy())
    finally:
        dist.destroy_process_group()


def _merge(all_d, all_i, k):
    world, nq, kk = all_d.shape
    out_i = np.full((nq, k), -1, np.int32)
    out_d = np.full((nq, k), -1, np.int64)
    for q in range(nq):
        pairs = [(int(all_d[r, q, j]), int(all_i[r, q, j])) for r in range(world) for j in range(kk)
                 if all_i[r, q, j] >= 0]
        pairs.sort()
        for j, (dd, ii) in enumerate(pairs[:k]):
            out_d[q, j], out_i[q, j] = dd, ii
    return out_d, out_i


@pytest.mark.parametrize("n,k", [(3001, 10), (7, 10)])
def test_two_rank_shards_merge_to_single_shard(n, k):
    mp = pytest.importorskip("torch.multiprocessing")
    nq, world = 24, 2
    with tempfile.TemporaryDirectory() as tmp:
        out = os.path.join(tmp, "gathered.npz")
        mp.spawn(_worker, args=(world, _free_port(), n, nq, k, out), nprocs=world, join=True)
        g = np.load(out)
        assert g["d"].shape == (world, nq, k) and g["i"].shape == (world, nq, k)
        # rank-major: rank r's ids lie in its own row range
        from winnex_madhava.sharding import row_range
        for r in range(world):
            s, e = row_range(n, r, world)
            v = g["i"][r][g["i"][r] >= 0]
            assert ((v >= s) & (v < e)).all()
        got_d, got_i = _merge(g["d"], g["i"], k)
    C = cases.gmm_u8(n, 32, 8, seed=61)
    Q = cases.gmm_u8_queries(nq, 32, 8, seed_means=61, seed_q=62)
    want_i, want_d = oracle.l2_exact_u8_int(C, Q, k)
    np.testing.assert_array_equal(got_i, want_i)
    np.testing.assert_array_equal(got_d[want_i >= 0], want_d[want_i >= 0])


def test_row_range_partitions():
    from winnex_madhava.sharding import row_range
    for n in (0, 1, 7, 100_000_000):
        for world in (1, 2, 4, 8):
            spans = [row_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(e - s for s, e in spans) - min(e - s for s, e in spans) <= 1
    with pytest.raises(ValueError):
        row_range(10, 2, 2)


def _coop_worker(rank, world, port, n, nq, k, frac, out):
    import torch
    import torch.distributed as dist

    from winnex_madhava.sharding import cooperative_topk, row_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        C = cases.gmm_u8(n, 32, 8, seed=65)
        Q = cases.gmm_u8_queries(nq, 32, 8, seed_means=65, seed_q=66)
        s, e = row_range(n, rank, world)
        gid = np.arange(s, e)
        D = ((C[s:e].astype(np.int64)[None, :, :] - Q.astype(np.int64)[:, None, :]) ** 2).sum(-1)  # [nq][rows]
        in_sample = (gid * 2654435761 % 1000) < frac * 1000  # a fixed subset of this shard

        def topk(mask_rows):
            di = np.full((nq, k), -1, np.int32)
            ii = np.full((nq, k), -1, np.int32)
            for q in range(nq):
                rows = np.flatnonzero(mask_rows[q])
                o = np.lexsort((gid[rows], D[q, rows]))[:k]
                di[q, :len(o)], ii[q, :len(o)] = D[q, rows[o]], gid[rows[o]]
            return torch.from_numpy(di), torch.from_numpy(ii)

        def sample(_q, _k):
            return topk(np.broadcast_to(in_sample, D.shape))

        def bounded(_q, _k, thr_d, thr_i):
            td, ti = thr_d[:, k - 1].numpy().astype(np.int64), thr_i[:, k - 1].numpy()
            inf = ti < 0
            ok = (D < td[:, None]) | ((D == td[:, None]) & (gid[None, :] <= ti[:, None])) | inf[:, None]
            return topk(ok)

        def merge(all_d, all_i):
            md, mi = _merge(all_d.numpy(), all_i.numpy(), k)
            return torch.from_numpy(md.astype(np.int32)), torch.from_numpy(mi)

        d, i = cooperative_topk(sample, bounded, merge, None, k)
        np.savez(out + f".{rank}.npz", d=d.numpy(), i=i.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("frac", [0.05, 0.0])
def test_two_rank_cooperative_thresholds(frac):
    """Thresholds from the merged sample lists of both ranks keep the result
    exact: every rank returns the single-shard oracle's top-k (an empty sample
    gives no threshold, and the bounded phase then keeps every row)."""
    mp = pytest.importorskip("torch.multiprocessing")
    n, nq, k, world = 4001, 12, 10, 2
    with tempfile.TemporaryDirectory() as tmp:
        out = os.path.join(tmp, "coop")
        mp.spawn(_coop_worker, args=(world, _free_port(), n, nq, k, frac, out), nprocs=world, join=True)
        got = [np.load(out + f".{r}.npz") for r in range(world)]
    C = cases.gmm_u8(n, 32, 8, seed=65)
    Q = cases.gmm_u8_queries(nq, 32, 8, seed_means=65, seed_q=66)
    want_i, want_d = oracle.l2_exact_u8_int(C, Q, k)
    for g in got:
        np.testing.assert_array_equal(g["i"], want_i)
        np.testing.assert_array_equal(g["d"], want_d)


def _failing_rank_worker(rank, world, port, out):
    import time

    import torch
    import torch.distributed as dist

    from winnex_madhava.sharding import cooperative_topk

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    k, nq = 4, 3
    lists = (torch.zeros((nq, k), dtype=torch.int32), torch.arange(nq * k, dtype=torch.int32).reshape(nq, k))

    def sample(_q, _k):
        if rank == 1:
            raise RuntimeError("sample phase failed on this rank")
        return lists

    t0 = time.monotonic()
    try:
        cooperative_topk(sample, lambda *a: lists, lambda d, i: (d[0], i[0]), None, k)
        outcome = "completed"
    except Exception as exc:  # noqa: BLE001 - the outcome is what the test checks
        outcome = f"{type(exc).__name__}: {exc}"
    with open(f"{out}.{rank}", "w") as f:
        f.write(f"{time.monotonic() - t0:.1f}\n{outcome}\n")
    if rank == 0:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001 - the group may already be broken
            pass


def test_failing_rank_ends_the_exchange_with_an_error():
    """A rank whose sample phase raises never joins the exchange; the other
    rank's all_gather ends with an error once the group's timeout (5 s)
    passes, instead of waiting forever, and no rank reports a result."""
    mp = pytest.importorskip("torch.multiprocessing")
    with tempfile.TemporaryDirectory() as tmp:
        out = os.path.join(tmp, "outcome")
        mp.spawn(_failing_rank_worker, args=(2, _free_port(), out), nprocs=2, join=True)
        r0 = open(out + ".0").read().split("\n", 1)
        r1 = open(out + ".1").read().split("\n", 1)
    assert "sample phase failed" in r1[1]
    assert not r0[1].startswith("completed") and float(r0[0]) < 60
