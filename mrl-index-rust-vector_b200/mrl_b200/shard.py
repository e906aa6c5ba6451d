"""Sharded scan across ranks (one process per GPU).

Pages shard naturally: each rank holds a contiguous range of a corpus's pages (its segment's
`block_id_base` is the range start, so ids are global) and scans only its own HBM. The single
exchange step is the merge of the per-rank top-k lists. It replaces the merge of per-shard
shortlists at the end of `scan_blocks_stats` (src/scan.rs:866-870) at GPU granularity:
  * on the device: each rank's scan writes its top-k into an exchange record; `ShardExchange`
    all-gathers the records with torch.distributed (one NCCL collective over NVLink) and merges
    them with the library's `mrl_merge_topk` kernel, so every rank ends with the global top-k;
  * on the host: `merge_topk_host` merges lists that are already in host memory (for example the
    outputs of `mrl_scan`) with the same order;
  * inside the scan launch: `PeerExchange` (mrl_exchange_*) has every rank's scan write its record
    into all ranks' receive areas over NVLink and merge there, one launch per query and no
    collective call on the query path.
Order everywhere: score descending, then id (VectorId::as_u64) ascending.
"""
from __future__ import annotations

import ctypes as C
from typing import Tuple

import numpy as np

from ._capi import check


def shard_range(n_pages: int, world: int, rank: int) -> Tuple[int, int]:
    """(first page, page count) of `rank`'s contiguous share of `n_pages` (sizes differ by <= 1)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, rem = divmod(int(n_pages), world)
    start = rank * base + min(rank, rem)
    return start, base + (1 if rank < rem else 0)


def merge_topk_host(ids: np.ndarray, scores: np.ndarray, counts: np.ndarray, k: int):
    """Merge per-shard top lists (rows of `ids` [n_lists, stride] u64 / `scores` f32, `counts[i]`
    valid entries each) into the global top-k: returns (ids[n], scores[n]) with n <= k."""
    ids = np.asarray(ids, np.uint64).reshape(len(counts), -1)
    scores = np.asarray(scores, np.float32).reshape(len(counts), -1)
    stride = ids.shape[1]
    take = [min(int(c), stride) for c in counts]
    all_ids = np.concatenate([ids[i, :n] for i, n in enumerate(take)]) if take else np.zeros(0, np.uint64)
    all_sc = np.concatenate([scores[i, :n] for i, n in enumerate(take)]) if take else np.zeros(0, np.float32)
    order = np.lexsort((all_ids, -all_sc.astype(np.float64)))[:k]
    return all_ids[order], all_sc[order]


def record_bytes(stride: int) -> int:
    """Size of one exchange record (MRL_MERGE_RECORD_BYTES): stride u64 ids, stride f32 scores,
    the u32 count, padded to a multiple of 16 bytes."""
    return (int(stride) * 12 + 4 + 15) // 16 * 16


def pack_records(ids: np.ndarray, scores: np.ndarray, counts: np.ndarray) -> np.ndarray:
    """Host copy of n exchange records (rows of `ids` [n, stride] / `scores`, `counts[i]` valid)."""
    ids = np.asarray(ids, np.uint64)
    n, stride = ids.shape
    rb = record_bytes(stride)
    out = np.zeros((n, rb), np.uint8)
    out[:, : 8 * stride] = ids.view(np.uint8).reshape(n, -1)
    out[:, 8 * stride: 12 * stride] = np.asarray(scores, np.float32).view(np.uint8).reshape(n, -1)
    out[:, 12 * stride: 12 * stride + 4] = np.asarray(counts, np.uint32).reshape(n, 1).view(np.uint8)
    return out


def unpack_records(records: np.ndarray, stride: int):
    """Inverse of pack_records: (ids [n, stride] u64, scores [n, stride] f32, counts [n] u32)."""
    rec = np.ascontiguousarray(records, np.uint8).reshape(-1, record_bytes(stride))
    ids = rec[:, : 8 * stride].copy().view(np.uint64)
    scores = rec[:, 8 * stride: 12 * stride].copy().view(np.float32)
    counts = rec[:, 12 * stride: 12 * stride + 4].copy().view(np.uint32).reshape(-1)
    return ids, scores, counts


class ShardExchange:
    """Device-side exchange of per-rank top-k lists. The scan writes its output straight into this
    rank's exchange record (`ids`, `scores`, `count` views); one all-gather of records (NCCL over
    NVLink) and the merge kernel then leave the global top-k in `top_ids`, `top_scores`,
    `top_count` on every rank. Buffers are allocated once (torch device tensors)."""

    def __init__(self, dev, k: int, group=None):
        import torch
        import torch.distributed as dist

        self.dev, self.k, self.group = dev, int(k), group
        self.world = dist.get_world_size(group)
        cuda = torch.device("cuda", torch.cuda.current_device())
        rb = record_bytes(self.k)
        self.record = torch.zeros(rb, dtype=torch.uint8, device=cuda)
        self.gathered = torch.zeros(self.world * rb, dtype=torch.uint8, device=cuda)
        k8, k12 = 8 * self.k, 12 * self.k
        self.ids = self.record[:k8].view(torch.int64)
        self.scores = self.record[k8:k12].view(torch.float32)
        self.count = self.record[k12:k12 + 4].view(torch.int32)
        self.top_ids = torch.empty(self.k, dtype=torch.int64, device=cuda)
        self.top_scores = torch.empty(self.k, dtype=torch.float32, device=cuda)
        self.top_count = torch.empty(1, dtype=torch.int32, device=cuda)

    def __call__(self):
        """All-gather the records and merge. The collective runs on torch's current stream, which
        must be the context's stream so it orders after the scan and before the merge."""
        import torch.distributed as dist

        dist.all_gather_into_tensor(self.gathered, self.record, group=self.group)
        lib = self.dev.lib
        check(self.dev.ptr, lib.mrl_merge_topk(self.dev.ptr, C.c_void_p(self.gathered.data_ptr()), self.world,
                                               self.k, self.k, C.c_void_p(self.top_ids.data_ptr()),
                                               C.c_void_p(self.top_scores.data_ptr()),
                                               C.c_void_p(self.top_count.data_ptr())))
        return self.top_ids, self.top_scores, self.top_count


class BatchShardExchange:
    """The exchange step of the sharded batched scan: each rank's batched scan
    results for n_q queries (`d_ids` / `d_scores` rows of k, `d_counts`) are packed into n_q
    records, all-gathered (one NCCL collective over NVLink for the whole batch) and merged per
    query on the device (mrl_merge_topk_batch), leaving every query's global top-k in `top_ids`,
    `top_scores` (rows of k) and `top_counts` on every rank."""

    def __init__(self, dev, n_q: int, k: int, group=None):
        import torch
        import torch.distributed as dist

        self.dev, self.n_q, self.k, self.group = dev, int(n_q), int(k), group
        self.world = dist.get_world_size(group)
        cuda = torch.device("cuda", torch.cuda.current_device())
        rb = record_bytes(self.k)
        self.records = torch.zeros(self.n_q * rb, dtype=torch.uint8, device=cuda)
        self.gathered = torch.zeros(self.world * self.n_q * rb, dtype=torch.uint8, device=cuda)
        self.top_ids = torch.empty(self.n_q * self.k, dtype=torch.int64, device=cuda)
        self.top_scores = torch.empty(self.n_q * self.k, dtype=torch.float32, device=cuda)
        self.top_counts = torch.empty(self.n_q, dtype=torch.int32, device=cuda)

    def __call__(self, d_ids: int, d_scores: int, d_counts: int):
        """Pack, all-gather and merge. The collective runs on torch's current stream, which must be
        the context's stream."""
        import torch.distributed as dist

        lib = self.dev.lib
        check(self.dev.ptr, lib.mrl_pack_records(self.dev.ptr, C.c_void_p(d_ids), C.c_void_p(d_scores),
                                                 C.c_void_p(d_counts), self.n_q, self.k,
                                                 C.c_void_p(self.records.data_ptr())))
        dist.all_gather_into_tensor(self.gathered, self.records, group=self.group)
        check(self.dev.ptr, lib.mrl_merge_topk_batch(self.dev.ptr, C.c_void_p(self.gathered.data_ptr()), self.world,
                                                     self.n_q, self.k, self.k, C.c_void_p(self.top_ids.data_ptr()),
                                                     C.c_void_p(self.top_scores.data_ptr()),
                                                     C.c_void_p(self.top_counts.data_ptr())))
        return self.top_ids, self.top_scores, self.top_counts


class PeerExchange:
    """NVLink exchange (mrl_exchange_*): after set-up, `scan(...)` runs the fused plan + scan +
    global merge of one query in a single launch on every rank. Set-up exchanges the receive
    areas' IPC handles with torch.distributed (any backend); all ranks must then scan the same
    sequence of queries. `close()` barriers before freeing, since peers write into this area."""

    def __init__(self, dev, k: int, group=None):
        import torch.distributed as dist

        self.dev, self.k, self.group = dev, int(k), group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        lib = dev.lib
        handle = (C.c_ubyte * 64)()
        self.ptr = C.c_void_p()
        check(dev.ptr, lib.mrl_exchange_create(dev.ptr, self.world, self.rank, self.k, C.cast(handle, C.c_void_p),
                                               C.byref(self.ptr)))
        gathered = [None] * self.world
        dist.all_gather_object(gathered, bytes(handle), group=group)
        allh = (C.c_ubyte * (64 * self.world)).from_buffer_copy(b"".join(gathered))
        check(dev.ptr, lib.mrl_exchange_open(dev.ptr, self.ptr, C.cast(allh, C.c_void_p)))

    def scan(self, segment, d_query: int, dims: int, desc, plans, cfg_c, d_ids: int, d_scores: int, d_count: int,
             d_status: int = 0, time_lo=None, time_hi=None):
        """Fused plan + scan of the device query at `d_query`; the device outputs receive the
        global top-k over all ranks' segments (asynchronous on the context stream)."""
        lo = None if time_lo is None else C.byref(C.c_uint32(int(time_lo)))
        hi = None if time_hi is None else C.byref(C.c_uint32(int(time_hi)))
        check(self.dev.ptr, self.dev.lib.mrl_query_scan_exchange(
            self.dev.ptr, segment.ptr, C.c_void_p(d_query), dims, C.byref(desc), plans, C.byref(cfg_c), lo, hi,
            self.ptr, C.c_void_p(d_ids), C.c_void_p(d_scores), C.c_void_p(d_count),
            C.c_void_p(d_status) if d_status else None))

    def submit(self, segment, query, desc, cfg_c, slot: int, time_lo=None, time_hi=None):
        """Pipelined host query (mrl_query_submit_exchange): launches the fused plan + scan + merge
        of the host query `query` into the context's result slot `slot` and returns at once; every
        rank submits the same sequence. `collect(slot)` returns the global top-k."""
        q = np.ascontiguousarray(query, np.float32).reshape(-1)
        lo = None if time_lo is None else C.byref(C.c_uint32(int(time_lo)))
        hi = None if time_hi is None else C.byref(C.c_uint32(int(time_hi)))
        check(self.dev.ptr, self.dev.lib.mrl_query_submit_exchange(
            self.dev.ptr, segment.ptr, q.ctypes.data_as(C.c_void_p), q.shape[0], C.byref(desc), C.byref(cfg_c), lo, hi,
            self.ptr, slot))

    def collect(self, slot: int):
        """(ids [count] u64, scores [count] f32): the global top-k of the query in `slot`."""
        if not hasattr(self, "_out"):  # result buffers kept across calls
            self._out = (np.zeros(self.k, np.uint64), np.zeros(self.k, np.float32), np.zeros(1, np.uint32))
            self._out_p = tuple(a.ctypes.data_as(C.c_void_p) for a in self._out)
        ids, sc, n = self._out
        check(self.dev.ptr, self.dev.lib.mrl_query_collect(self.dev.ptr, slot, *self._out_p))
        return ids[:int(n[0])].copy(), sc[:int(n[0])].copy()

    def close(self):
        import torch.distributed as dist

        if self.ptr:
            dist.barrier(group=self.group)
            self.dev.lib.mrl_exchange_destroy(self.dev.ptr, self.ptr)
            self.ptr = C.c_void_p()
