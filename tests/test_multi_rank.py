"""The sharded (N > 1) scan path on CPU: world-size-2 `gloo` process groups.

Each rank scans its own contiguous page range (`shard_range`) with the oracle as the stand-in
for its GPU, offsets its block ids by its range start, packs its top-k into an exchange record
(the layout the GPU scan writes), all-gathers the records and merges them with
`merge_topk_host`. The merged result must equal the oracle's scan of the whole
corpus (ids identical, scores bit-identical). This covers the host logic of the exchange step:
page split, id offsets, gather, merge order and short lists. The device merge kernel has its own
GPU test (test_gpu_merge.py).
"""
import os
import socket
import struct

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _corpus(ora):
    n, dims = 64 * 40 + 17, 384
    docs = ora.synth_docs(5, n, dims)
    mean = ora.eden_fit_prefix(docs)
    blocks = ora.encode_corpus(docs, eden_mean=mean).reshape(-1, 4096).copy()
    # tombstone a few slots in both halves so the per-rank counts differ
    for b, slot in ((3, 7), (3, 8), (30, 0), (40, 1)):
        t = struct.unpack_from("<Q", blocks[b], 16)[0] | (1 << slot)
        struct.pack_into("<Q", blocks[b], 16, t)
    q, _ = ora.synth_queries(5, n, 9, 1, dims)
    return blocks, mean, q[0]


def _rank_worker(rank, world, port, k):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch
    import torch.distributed as dist

    import ora
    from mrl_b200.shard import merge_topk_host, pack_records, shard_range, unpack_records

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        blocks, mean, q = _corpus(ora)
        plan = ora.plan_build(q, eden_mean=mean)
        cfg = ora.scan_cfg(k=k)
        start, count = shard_range(blocks.shape[0], world, rank)
        ids, sc = ora.scan_blocks(blocks[start:start + count].reshape(-1), plan, cfg, threads=2)
        gids = ((ids >> np.uint64(16)) + np.uint64(start)) << np.uint64(16) | (ids & np.uint64(0xFFFF))
        # this rank's exchange record (the layout the GPU scan writes), gathered from every rank
        pad_ids = np.zeros((1, k), np.uint64)
        pad_sc = np.zeros((1, k), np.float32)
        pad_ids[0, : len(gids)] = gids
        pad_sc[0, : len(sc)] = sc
        rec = torch.from_numpy(pack_records(pad_ids, pad_sc, np.array([len(gids)])).reshape(-1))
        recs = [torch.zeros_like(rec) for _ in range(world)]
        dist.all_gather(recs, rec)
        g_ids, g_sc, g_cnt = unpack_records(torch.stack(recs).numpy(), k)
        m_ids, m_sc = merge_topk_host(g_ids, g_sc, g_cnt, k)
        r_ids, r_sc = ora.scan_blocks(blocks.reshape(-1), plan, cfg, threads=2)
        assert np.array_equal(m_ids, r_ids.astype(np.uint64)), rank
        assert np.array_equal(m_sc.view(np.uint32), r_sc.view(np.uint32)), rank
        # every rank holds the same merged list
        chk = [torch.zeros(len(m_ids), dtype=torch.int64) for _ in range(world)]
        dist.all_gather(chk, torch.from_numpy(m_ids.astype(np.int64)))
        assert all(torch.equal(c, chk[0]) for c in chk)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("k", [64, 3000])
def test_two_rank_sharded_scan_matches_single_scan(ora, k):
    import torch.multiprocessing as tmp

    tmp.spawn(_rank_worker, args=(2, _free_port(), k), nprocs=2, join=True)


def _batch_rank_worker(rank, world, port, k):
    """Configs 4 and 5 on CPU: a batch of queries, each rank scanning its page range and searching
    its own pending ring rows (sentinel slots rank x 4096 + position, as mrl_ring_search_batch
    writes them with slot_base = rank x 4096), merging the two per query, packing one record per
    query, one all-gather, and a per-query merge across ranks. Every rank must end with, for every
    query, the top-k of the whole corpus plus every rank's ring, with every ring hit naming its
    rank and row."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch
    import torch.distributed as dist

    import ora
    from mrl_b200.shard import merge_topk_host, pack_records, shard_range, unpack_records

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        blocks, mean, _ = _corpus(ora)
        n_docs, dims = 64 * 40 + 17, 384
        qs, _ = ora.synth_queries(5, n_docs, 21, 3, dims)
        rings = [ora.synth_docs(60 + r, 10 + 13 * r, dims) for r in range(world)]
        qs[1] = rings[1 % world][4]  # a pending row of another rank must lead query 1
        cfg = ora.scan_cfg(k=k)
        start, count = shard_range(blocks.shape[0], world, rank)
        sentinel = np.uint64(0xFFFFFFFF) << np.uint64(16)
        recs = []
        for q in qs:
            plan = ora.plan_build(q, eden_mean=mean)
            ids, sc = ora.scan_blocks(blocks[start:start + count].reshape(-1), plan, cfg, threads=2)
            gids = ((ids >> np.uint64(16)) + np.uint64(start)) << np.uint64(16) | (ids & np.uint64(0xFFFF))
            pos, rsc = ora.ring_search(rings[rank], q, k)
            rids = sentinel | (np.uint64(rank * 4096) + pos.astype(np.uint64))
            pad_i = np.zeros((2, k), np.uint64)
            pad_s = np.zeros((2, k), np.float32)
            pad_i[0, :len(gids)], pad_s[0, :len(sc)] = gids, sc
            pad_i[1, :len(rids)], pad_s[1, :len(rsc)] = rids, rsc
            m_i, m_s = merge_topk_host(pad_i, pad_s, np.array([len(gids), len(rids)]), k)
            pi = np.zeros((1, k), np.uint64)
            ps = np.zeros((1, k), np.float32)
            pi[0, :len(m_i)], ps[0, :len(m_s)] = m_i, m_s
            recs.append(pack_records(pi, ps, np.array([len(m_i)]))[0])
        rec = torch.from_numpy(np.stack(recs).reshape(-1))  # this rank's batch: one record per query
        gathered = [torch.zeros_like(rec) for _ in range(world)]
        dist.all_gather(gathered, rec)
        g_ids, g_sc, g_cnt = unpack_records(torch.stack(gathered).numpy(), k)  # [world x n_q] records
        n_q = len(qs)
        for qi, q in enumerate(qs):
            sel = [r * n_q + qi for r in range(world)]
            m_ids, m_sc = merge_topk_host(g_ids[sel], g_sc[sel], g_cnt[sel], k)
            # the whole corpus and every rank's ring, in one list
            r_ids, r_sc = ora.scan_blocks(blocks.reshape(-1), ora.plan_build(q, eden_mean=mean), cfg, threads=2)
            all_i, all_s = [r_ids.astype(np.uint64)], [r_sc]
            for r in range(world):
                pos, rsc = ora.ring_search(rings[r], q, k)
                all_i.append(sentinel | (np.uint64(r * 4096) + pos.astype(np.uint64)))
                all_s.append(rsc)
            cat_i, cat_s = np.concatenate(all_i), np.concatenate(all_s)
            order = np.lexsort((cat_i, -cat_s.astype(np.float64)))[:k]
            assert np.array_equal(m_ids, cat_i[order]), (rank, qi)
            assert np.array_equal(m_sc.view(np.uint32), cat_s[order].view(np.uint32)), (rank, qi)
            if qi == 1:  # the planted pending row: rank 1's ring, row 4
                assert m_ids[0] == sentinel | np.uint64((1 % world) * 4096 + 4)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("k", [16, 256])
def test_two_rank_sharded_batch_with_rings(ora, k):
    import torch.multiprocessing as tmp

    tmp.spawn(_batch_rank_worker, args=(2, _free_port(), k), nprocs=2, join=True)


def test_shard_range_covers_pages_once():
    from mrl_b200.shard import shard_range

    for n in (0, 1, 7, 64, 15625, 137500):
        for world in (1, 2, 3, 4, 8):
            parts = [shard_range(n, world, r) for r in range(world)]
            assert parts[0][0] == 0
            assert all(a[0] + a[1] == b[0] for a, b in zip(parts, parts[1:]))
            assert sum(c for _, c in parts) == n
            assert max(c for _, c in parts) - min(c for _, c in parts) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def test_merge_topk_host_order_and_short_lists():
    from mrl_b200.shard import merge_topk_host

    ids = np.array([[5, 9, 0, 0], [2, 7, 8, 0], [0, 0, 0, 0]], np.uint64)
    sc = np.array([[0.9, 0.5, 0, 0], [0.9, 0.5, 0.1, 0], [0, 0, 0, 0]], np.float32)
    got_ids, got_sc = merge_topk_host(ids, sc, np.array([2, 3, 0]), 4)
    assert got_ids.tolist() == [2, 5, 7, 9]            # equal scores: lower id first
    assert got_sc.tolist() == pytest.approx([0.9, 0.9, 0.5, 0.5])
    got_ids, _ = merge_topk_host(ids, sc, np.array([2, 3, 0]), 10)
    assert got_ids.tolist() == [2, 5, 7, 9, 8]         # fewer than k live entries


def test_pack_records_layout():
    from mrl_b200.shard import pack_records, record_bytes

    assert [record_bytes(s) for s in (1, 16, 256, 4096)] == [16, 208, 3088, 49168]
    ids = np.array([[1, 2, 3]], np.uint64)
    sc = np.array([[0.5, 0.25, 0.125]], np.float32)
    rec = pack_records(ids, sc, np.array([2]))
    assert rec.shape == (1, record_bytes(3))
    assert rec[0, :24].view(np.uint64).tolist() == [1, 2, 3]
    assert rec[0, 24:36].view(np.float32).tolist() == [0.5, 0.25, 0.125]
    assert rec[0, 36:40].view(np.uint32).tolist() == [2]
