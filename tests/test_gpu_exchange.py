"""The NVLink exchange (mrl_exchange_*, mrl_query_scan_exchange): the merge of per-rank top-k
records inside the scan launch.

On one GPU an exchange of world 1 must reproduce mrl_query_scan_device exactly, across
consecutive queries (both buffer parities), through the rare re-selection path, and for host
queries submitted several at a time (mrl_query_submit_exchange). With two or more GPUs, two ranks
(one process per GPU, handles exchanged over gloo) scan one half of a corpus each, and every rank
must end with the global top-k of a single-GPU scan of the whole corpus, for device queries and
for host queries in flight.
"""
import ctypes as C
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def mb():
    import mrl_b200

    return mrl_b200


def _corpus(ora, n=64 * 40 + 17, dims=768, seed=11):
    docs = ora.synth_docs(seed, n, dims)
    mean = ora.eden_fit_prefix(docs)
    blocks = ora.encode_corpus(docs, eden_mean=mean)
    qs, _ = ora.synth_queries(seed, n, 5, 4, dims)
    return blocks, mean, qs


def _device_outputs(k):
    import torch

    return (torch.full((k,), -1, dtype=torch.int64, device="cuda"), torch.zeros(k, dtype=torch.float32, device="cuda"),
            torch.zeros(1, dtype=torch.int32, device="cuda"), torch.zeros(1, dtype=torch.int32, device="cuda"))


@pytest.mark.parametrize("mode", ["FAST", "EXACT"])
@pytest.mark.parametrize("list_len", [0, 1])
def test_exchange_world1_matches_device_scan(ora, dev, mode, list_len):
    import torch

    M = mb()
    lib = dev.lib
    blocks, mean, qs = _corpus(ora)
    seg = M.Segment.upload(blocks, dev)
    k = 256
    cfg = M.ScanConfig(shortlist_cand=k, mode=getattr(M.ScanMode, mode)).to_c()
    desc, keep = M.api._codec_desc(M.PrefixCodec.EDEN_PROD, M.MidCodec.RABITQ, M.EdenFit(64, 4, 1, mean), None)
    plans = C.c_void_p()
    M._capi.check(dev.ptr, lib.mrl_plans_alloc(dev.ptr, 1, 768, C.byref(plans)))
    ex = C.c_void_p()
    M._capi.check(dev.ptr, lib.mrl_exchange_create(dev.ptr, 1, 0, k, None, C.byref(ex)))
    dq = torch.from_numpy(np.ascontiguousarray(qs, np.float32)).cuda()
    dev.set_list_len(list_len)
    try:
        for qi in range(len(qs)):  # consecutive queries alternate buffer parities
            a = _device_outputs(k)
            b = _device_outputs(k)
            torch.cuda.synchronize()
            qp = C.c_void_p(dq.data_ptr() + qi * 768 * 4)
            M._capi.check(dev.ptr, lib.mrl_query_scan_device(dev.ptr, seg.ptr, qp, 1, 768, C.byref(desc), plans,
                                                             C.byref(cfg), None, None, *[C.c_void_p(t.data_ptr()) for t in a]))
            M._capi.check(dev.ptr, lib.mrl_query_scan_exchange(dev.ptr, seg.ptr, qp, 768, C.byref(desc), plans,
                                                               C.byref(cfg), None, None, ex,
                                                               *[C.c_void_p(t.data_ptr()) for t in b]))
            # outputs in pinned host memory (device-accessible under unified addressing): the launch
            # stores the merged top-k straight there
            h = [t.cpu().pin_memory() for t in _device_outputs(k)]
            M._capi.check(dev.ptr, lib.mrl_query_scan_exchange(dev.ptr, seg.ptr, qp, 768, C.byref(desc), plans,
                                                               C.byref(cfg), None, None, ex,
                                                               *[C.c_void_p(t.data_ptr()) for t in h]))
            torch.cuda.synchronize()
            n = int(a[2].item())
            assert int(b[2].item()) == n == k == int(h[2][0])
            assert int(b[3].item()) & 6 == 0 and int(h[3][0]) & 6 == 0  # no barrier or exchange timeout
            assert torch.equal(a[0][:n], b[0][:n]) and torch.equal(a[0][:n].cpu(), h[0][:n])
            assert np.array_equal(a[1][:n].cpu().numpy().view(np.uint32), b[1][:n].cpu().numpy().view(np.uint32))
            assert np.array_equal(h[1][:n].numpy().view(np.uint32), b[1][:n].cpu().numpy().view(np.uint32))
            if list_len == 1:
                assert int(b[3].item()) & 1 == 1  # the re-selection ran
    finally:
        dev.set_list_len(0)
        lib.mrl_exchange_destroy(dev.ptr, ex)
        lib.mrl_plans_free(dev.ptr, plans)
        seg.free()
    del keep


@pytest.mark.parametrize("mode", ["FAST", "EXACT"])
def test_exchange_world1_submit_pipelined(ora, dev, mode):
    """mrl_query_submit_exchange with world 1: host queries submitted several at a time (slots,
    scratch sets and buffer parities reused) end in the same top-k as mrl_query_scan_device."""
    import torch

    M = mb()
    lib = dev.lib
    blocks, mean, qs = _corpus(ora)
    qs = np.concatenate([qs, qs[::-1] * 0.5])  # 8 queries
    seg = M.Segment.upload(blocks, dev)
    k = 256
    cfg = M.ScanConfig(shortlist_cand=k, mode=getattr(M.ScanMode, mode)).to_c()
    desc, keep = M.api._codec_desc(M.PrefixCodec.EDEN_PROD, M.MidCodec.RABITQ, M.EdenFit(64, 4, 1, mean), None)
    plans = C.c_void_p()
    M._capi.check(dev.ptr, lib.mrl_plans_alloc(dev.ptr, 1, 768, C.byref(plans)))
    ex = C.c_void_p()
    M._capi.check(dev.ptr, lib.mrl_exchange_create(dev.ptr, 1, 0, k, None, C.byref(ex)))
    dq = torch.from_numpy(np.ascontiguousarray(qs, np.float32)).cuda()
    try:
        want = []
        for qi in range(len(qs)):
            a = _device_outputs(k)
            M._capi.check(dev.ptr, lib.mrl_query_scan_device(dev.ptr, seg.ptr, C.c_void_p(dq.data_ptr() + qi * 768 * 4),
                                                             1, 768, C.byref(desc), plans, C.byref(cfg), None, None,
                                                             *[C.c_void_p(t.data_ptr()) for t in a]))
            torch.cuda.synchronize()
            n = int(a[2].item())
            want.append((a[0][:n].cpu().numpy().view(np.uint64).copy(), a[1][:n].cpu().numpy().view(np.uint32).copy()))
        ids = np.zeros(k, np.uint64)
        sc = np.zeros(k, np.float32)
        cnt = np.zeros(1, np.uint32)
        order = list(range(len(qs))) * 3  # 24 queries over 8 slots, 8 in flight at a time
        for i0 in range(0, len(order), 8):
            batch = order[i0:i0 + 8]
            for slot, qi in enumerate(batch):
                q = np.ascontiguousarray(qs[qi], np.float32)
                M._capi.check(dev.ptr, lib.mrl_query_submit_exchange(dev.ptr, seg.ptr, q.ctypes.data_as(C.c_void_p), 768,
                                                                     C.byref(desc), C.byref(cfg), None, None, ex, slot))
            for slot, qi in enumerate(batch):
                M._capi.check(dev.ptr, lib.mrl_query_collect(dev.ptr, slot, ids.ctypes.data_as(C.c_void_p),
                                                             sc.ctypes.data_as(C.c_void_p), cnt.ctypes.data_as(C.c_void_p)))
                n = int(cnt[0])
                assert n == len(want[qi][0]), (i0, slot)
                assert np.array_equal(ids[:n], want[qi][0]), (i0, slot)
                assert np.array_equal(sc[:n].view(np.uint32), want[qi][1]), (i0, slot)
        # misuse: a different k than the exchange's is refused
        bad = M.ScanConfig(shortlist_cand=16, mode=getattr(M.ScanMode, mode)).to_c()
        q = np.ascontiguousarray(qs[0], np.float32)
        assert lib.mrl_query_submit_exchange(dev.ptr, seg.ptr, q.ctypes.data_as(C.c_void_p), 768, C.byref(desc),
                                             C.byref(bad), None, None, ex, 0) != 0
    finally:
        lib.mrl_exchange_destroy(dev.ptr, ex)
        lib.mrl_plans_free(dev.ptr, plans)
        seg.free()
    del keep


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, k, mode, list_len):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch
    import torch.distributed as dist

    import mrl_b200 as M
    import ora

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    dev = M.Device(rank)
    try:
        blocks, mean, qs = _corpus(ora)
        pages = blocks.reshape(-1, 4096)
        start, count = M.shard_range(pages.shape[0], world, rank)
        seg = M.Segment.upload(pages[start:start + count].reshape(-1), dev, block_id_base=start)
        whole = M.Segment.upload(blocks, dev)
        cfg = M.ScanConfig(shortlist_cand=k, mode=getattr(M.ScanMode, mode)).to_c()
        desc, keep = M.api._codec_desc(M.PrefixCodec.EDEN_PROD, M.MidCodec.RABITQ, M.EdenFit(64, 4, 1, mean), None)
        plans = C.c_void_p()
        M._capi.check(dev.ptr, dev.lib.mrl_plans_alloc(dev.ptr, 1, 768, C.byref(plans)))
        px = M.PeerExchange(dev, k)
        dq = torch.from_numpy(np.ascontiguousarray(qs, np.float32)).cuda()
        dev.set_list_len(list_len)
        want = []
        for qi in range(len(qs)):
            a = _device_outputs(k)
            b = _device_outputs(k)
            torch.cuda.synchronize()
            qp = dq.data_ptr() + qi * 768 * 4
            px.scan(seg, qp, 768, desc, plans, cfg, *[t.data_ptr() for t in b])
            M._capi.check(dev.ptr, dev.lib.mrl_query_scan_device(dev.ptr, whole.ptr, C.c_void_p(qp), 1, 768,
                                                                 C.byref(desc), plans, C.byref(cfg), None, None,
                                                                 *[C.c_void_p(t.data_ptr()) for t in a]))
            torch.cuda.synchronize()
            n = int(a[2].item())
            assert int(b[2].item()) == n, (rank, qi)
            assert int(b[3].item()) & 6 == 0, (rank, qi, int(b[3].item()))
            assert torch.equal(a[0][:n], b[0][:n]), (rank, qi)
            assert np.array_equal(a[1][:n].cpu().numpy().view(np.uint32), b[1][:n].cpu().numpy().view(np.uint32))
            want.append((a[0][:n].cpu().numpy().view(np.uint64).copy(), a[1][:n].cpu().numpy().view(np.uint32).copy()))
        # pipelined host queries over the exchange: every query submitted before the first collect
        # (all in flight together), twice over so slots, scratch sets and parities are reused
        for rnd in range(2):
            for qi in range(len(qs)):
                px.submit(seg, qs[qi], desc, cfg, qi)
            for qi in range(len(qs)):
                ids, sc = px.collect(qi)
                assert np.array_equal(ids, want[qi][0]), (rank, rnd, qi)
                assert np.array_equal(sc.view(np.uint32), want[qi][1]), (rank, rnd, qi)
        dev.set_list_len(0)
        px.close()
        del keep
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode,list_len", [("FAST", 0), ("EXACT", 0), ("FAST", 1)])
def test_exchange_two_ranks_global_topk(mode, list_len):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as tmp

    tmp.spawn(_rank_main, args=(2, _free_port(), 256, mode, list_len), nprocs=2, join=True)


def _rank_skip_main(rank, world, port, k):
    """Rank 1 stays alive but skips one query: rank 0's wait for its flag must run out and report
    status bit 2 without a result; both contexts stay usable and shut down cleanly."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import time

    import torch
    import torch.distributed as dist

    import mrl_b200 as M
    import ora

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    dev = M.Device(rank)
    try:
        blocks, mean, qs = _corpus(ora)
        pages = blocks.reshape(-1, 4096)
        start, count = M.shard_range(pages.shape[0], world, rank)
        seg = M.Segment.upload(pages[start:start + count].reshape(-1), dev, block_id_base=start)
        cfg = M.ScanConfig(shortlist_cand=k).to_c()
        desc, keep = M.api._codec_desc(M.PrefixCodec.EDEN_PROD, M.MidCodec.RABITQ, M.EdenFit(64, 4, 1, mean), None)
        plans = C.c_void_p()
        M._capi.check(dev.ptr, dev.lib.mrl_plans_alloc(dev.ptr, 1, 768, C.byref(plans)))
        px = M.PeerExchange(dev, k)
        dq = torch.from_numpy(np.ascontiguousarray(qs, np.float32)).cuda()
        out = _device_outputs(k)
        torch.cuda.synchronize()
        px.scan(seg, dq.data_ptr(), 768, desc, plans, cfg, *[t.data_ptr() for t in out])  # both ranks
        torch.cuda.synchronize()
        assert int(out[3].item()) & 6 == 0
        dist.barrier()
        if rank == 0:  # rank 1 does not take part in this query
            t0 = time.perf_counter()
            px.scan(seg, dq.data_ptr() + 768 * 4, 768, desc, plans, cfg, *[t.data_ptr() for t in out])
            torch.cuda.synchronize()
            assert int(out[3].item()) & 4, int(out[3].item())  # the wait ran out
            assert time.perf_counter() - t0 < 30
            x = torch.ones(4, device="cuda") * 2  # the context still works
            assert float(x.sum().item()) == 8.0
        dist.barrier()
        px.close()
        del keep
    finally:
        dist.destroy_process_group()


def test_exchange_missing_rank_times_out():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as tmp

    tmp.spawn(_rank_skip_main, args=(2, _free_port(), 256), nprocs=2, join=True)
