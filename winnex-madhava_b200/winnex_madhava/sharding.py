"""Row sharding of one corpus over the ranks of a process group (one process
per GPU) and the exchange step of the sharded exact scan.

Rank r of G owns the contiguous rows [r*N//G, (r+1)*N//G) and builds its
index with ``id_offset`` = its first row, so its top-k lists carry global
ids.  After the local search every rank all-gathers the ``[Q][k]`` (distance,
id) lists -- the only collective of the path, 8*Q*k bytes per rank -- and
merges them with ``mdh_merge_topk_device``, which orders by (distance,
global id).  The merged lists therefore do not depend on G.

The reference has no multi-GPU path; its single-device GPU search is
``SpeedEngine::scores_gpu_topk`` (src/speed_gpu.cu:170-233).
"""
from __future__ import annotations

import ctypes


def row_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [start, end) owned by ``rank`` of ``world``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if n < 0:
        raise ValueError("n must be >= 0")
    return n * rank // world, n * (rank + 1) // world


def gather_topk(dist, ids, group=None):
    """All-gather this rank's ``[Q][k]`` int32 (distance, id) tensors.

    Returns ``(all_dist, all_ids)`` shaped ``[world][Q][k]``, rank-major,
    on the inputs' device.  The pair travels as one ``[Q][k][2]`` tensor, so
    the exchange is a single collective (8*Q*k bytes per rank).  Works with
    any backend that implements ``all_gather`` (NCCL on GPUs, gloo on CPU).
    """
    import torch
    import torch.distributed as tdist

    if dist.shape != ids.shape or dist.dtype != torch.int32 or ids.dtype != torch.int32:
        raise ValueError("dist and ids must be int32 tensors of the same shape")
    world = tdist.get_world_size(group)
    pair = torch.stack((dist, ids), dim=-1).contiguous()
    out = torch.empty((world,) + tuple(pair.shape), dtype=torch.int32, device=dist.device)
    if tdist.get_backend(group) == "nccl":
        tdist.all_gather_into_tensor(out, pair, group=group)
    else:
        tdist.all_gather(list(out.unbind(0)), pair, group=group)
    return out[..., 0].contiguous(), out[..., 1].contiguous()


def merge_topk_device(lib, all_dist, all_ids, stream=None):
    """Merge gathered lists on the GPU (``mdh_merge_topk_device``).

    ``lib`` is the loaded ``libwinnex_madhava_b200.so`` (ctypes); inputs are
    CUDA tensors ``[world][Q][k]``.  Returns ``(dist, ids)`` ``[Q][k]``.
    """
    import torch

    world, nq, k = all_dist.shape
    out_d = torch.empty((nq, k), dtype=torch.int32, device=all_dist.device)
    out_i = torch.empty_like(out_d)
    # Default: torch's current stream on the inputs' device, the stream that
    # produced the gathered lists and the output buffers.
    if stream is None:
        stream = torch.cuda.current_stream(all_dist.device)
    sp = ctypes.c_void_p(stream.cuda_stream)
    st = lib.mdh_merge_topk_device(ctypes.c_void_p(all_dist.data_ptr()), ctypes.c_void_p(all_ids.data_ptr()),
                                   world, nq, k, ctypes.c_void_p(out_d.data_ptr()), ctypes.c_void_p(out_i.data_ptr()),
                                   sp)
    if st != 0:
        raise RuntimeError(lib.mdh_last_error().decode() if lib.mdh_last_error() else f"merge failed ({st})")
    return out_d, out_i


def cooperative_topk(sample, bounded, merge, queries, k, group=None):
    """Row-sharded exact top-k with thresholds shared across the ranks.

    ``sample(queries, k)`` -> this rank's ``(dist, ids)`` top-k over its sample
    rows; ``bounded(queries, k, thr_dist, thr_ids)`` -> its exact top-k among
    its rows at or under each query's threshold, the k-th entry of the merged
    ``[Q][k]`` lists given; ``merge(all_dist, all_ids)`` -> the k smallest
    ``(dist, global id)`` of ``[world][Q][k]`` lists.  Two exchanges
    (``gather_topk``): the sample lists, whose merged k-th entry is the k-th
    best of the union of every rank's sample and so a threshold valid for the
    whole corpus, then the final lists.  Returns the merged ``(dist, ids)``,
    the same on every rank and for every rank count.
    """
    d1, i1 = sample(queries, k)
    thr_d, thr_i = merge(*gather_topk(d1, i1, group))
    d2, i2 = bounded(queries, k, thr_d, thr_i)
    return merge(*gather_topk(d2, i2, group))


def device_phases(lib, index, dev_queries, stream=None, stats=None):
    """The (sample, bounded) callables of :func:`cooperative_topk` for one
    rank's index through the C ABI (``mdh_search_u8_device_sample`` /
    ``mdh_search_u8_device_bounded``), on CUDA tensors."""
    import torch

    def _stream(t):
        s = stream if stream is not None else torch.cuda.current_stream(t.device)
        return ctypes.c_void_p(s.cuda_stream)

    def _check(st):
        if st != 0:
            raise RuntimeError(lib.mdh_last_error().decode())

    def sample(q, k):
        ids = torch.empty((q.shape[0], k), dtype=torch.int32, device=q.device)
        dist = torch.empty_like(ids)
        _check(lib.mdh_search_u8_device_sample(index, ctypes.c_void_p(q.data_ptr()), q.shape[0], k,
                                               ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(dist.data_ptr()),
                                               _stream(q), stats))
        return dist, ids

    def bounded(q, k, thr_d, thr_i):
        ids = torch.empty((q.shape[0], k), dtype=torch.int32, device=q.device)
        dist = torch.empty_like(ids)
        _check(lib.mdh_search_u8_device_bounded(index, ctypes.c_void_p(q.data_ptr()), q.shape[0], k,
                                                ctypes.c_void_p(thr_d.data_ptr()), ctypes.c_void_p(thr_i.data_ptr()),
                                                ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(dist.data_ptr()),
                                                _stream(q), stats))
        return dist, ids

    return sample, bounded
