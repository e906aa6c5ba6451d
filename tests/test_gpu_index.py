"""The exact paths and the index directory on the device, against the oracle.

  * ring search (mrl_ring_search) and exact rerank (mrl_rerank_exact): bit-identical scores and
    the reference's order (stable sort, score descending) at 768 dims (dot_768) and other dims;
  * the segment loader (mrl_segment_load): the same device pages as an upload, the reference's
    CorruptSize error, a missing file as an empty segment;
  * mrl_engine_scan: scan + ring merged into one shortlist, equal to the oracle's scan and ring
    search merged with Shortlist semantics;
  * IndexDir: create, ingest with online EDEN fit and live appends, search, reopen.
"""
import ctypes as C
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def mb():
    import mrl_b200

    return mrl_b200


def _rows(seed, n, dims):
    r = np.random.default_rng(seed).standard_normal((n, dims)).astype(np.float32)
    return r / np.linalg.norm(r, axis=1, keepdims=True)


@pytest.mark.parametrize("dims", [768, 384, 100])
@pytest.mark.parametrize("n,k", [(0, 8), (1, 8), (63, 256), (63, 10), (4096, 300)])
def test_ring_search_bit_identical(ora, dev, dims, n, k):
    import torch

    M = mb()
    pend = _rows(n + dims, n, dims)
    if n > 8:
        pend[5] = pend[2]  # equal scores: push order decides
        pend[6] = -0.0 * pend[6]
    q = _rows(7, 1, dims)[0]
    rp, rs = ora.ring_search(pend, q, k)
    dq = torch.from_numpy(q).cuda()
    dp = torch.from_numpy(pend).cuda() if n else torch.zeros(1, dims, device="cuda")
    rec = torch.zeros(M.record_bytes(k), dtype=torch.uint8, device="cuda")
    M._capi.check(dev.ptr, dev.lib.mrl_ring_search(dev.ptr, C.c_void_p(dq.data_ptr()), C.c_void_p(dp.data_ptr()), n,
                                                   dims, k, C.c_void_p(rec.data_ptr())))
    torch.cuda.synchronize()
    h = rec.cpu().numpy()
    m = int(h[12 * k:12 * k + 4].view(np.uint32)[0])
    ids = h[:8 * k].view(np.uint64)[:m]
    sc = h[8 * k:12 * k].view(np.float32)[:m]
    assert m == min(n, k)
    assert np.all(ids >> np.uint64(16) == np.uint64(0xFFFFFFFF))  # VectorId(u32::MAX, i)
    assert np.array_equal((ids & np.uint64(0xFFFF)).astype(np.uint32), rp)
    assert np.array_equal(sc.view(np.uint32), rs.view(np.uint32))


@pytest.mark.parametrize("dims", [768, 384, 33])
def test_rerank_exact_bit_identical(ora, dev, dims):
    M = mb()
    rows = _rows(dims, 5000, dims)
    rows[11] = rows[10]
    q = _rows(3, 1, dims)[0]
    rng = np.random.default_rng(dims)
    for cand in (rng.choice(5000, 4096, replace=False), np.array([10, 11, 10, 4999, 0]), rng.choice(5000, 1)):
        cand = cand.astype(np.uint64)
        rr, rs = ora.rerank_rows(rows, q, cand)
        got = M.rerank_exact_rows(q, cand, rows, dev=dev)
        assert [r for r, _ in got] == [int(x) for x in rr]
        assert np.array_equal(np.array([s for _, s in got], np.float32).view(np.uint32), rs.view(np.uint32))
    assert M.rerank_exact_rows(q, [], rows, dev=dev) == []


def test_rerank_rejects_bad_rows(dev):
    import torch

    M = mb()
    rows = torch.zeros(10, 64, device="cuda")
    with pytest.raises(M.MrlError, match="out of range"):
        M.rerank_exact_rows(np.zeros(64, np.float32), [3, 10], rows, dev=dev)
    with pytest.raises(M.MrlError, match="at most 4096"):
        M.rerank_exact_rows(np.zeros(64, np.float32), np.zeros(4097, np.uint64), rows, dev=dev)
    assert M.rerank_exact_rows(np.zeros(64, np.float32), [9], rows, dev=dev)[0][0] == 9  # context usable


def test_segment_load_matches_upload(ora, dev, tmp_path):
    M = mb()
    docs = ora.synth_docs(5, 64 * 37 + 9, 768)
    blocks = ora.encode_corpus(docs, eden_mean=ora.eden_fit_prefix(docs))
    p = str(tmp_path / "000001.pax")
    blocks.tofile(p)
    a = M.load_segment(p, dev, block_id_base=3)
    b = M.Segment.upload(blocks, dev, block_id_base=3)
    pa, ta = a.read_layout()
    pb, tb = b.read_layout()
    assert a.block_count() == 38 and np.array_equal(pa, pb) and np.array_equal(ta, tb)
    q = M.QueryPlan.from_query_eden(ora.synth_queries(5, docs.shape[0], 1, 1, 768)[0][0], 768,
                                    M.EdenFit(64, 4, 1, ora.eden_fit_prefix(docs)), dev=dev)
    ha = M.scan_blocks(a, q, M.ScanConfig(shortlist_cand=64))
    hb = M.scan_blocks(b, q, M.ScanConfig(shortlist_cand=64))
    assert ha == hb and all(h.id.block >= 3 for h in ha)
    with open(p, "ab") as f:
        f.write(b"\0" * 100)
    with pytest.raises(M.SegmentError, match=r"corrupt segment size 155748 \(not multiple of 4096\)"):
        M.load_segment(p, dev)
    e = M.load_segment(str(tmp_path / "missing.pax"), dev)
    assert e.block_count() == 0
    for s in (a, b, e):
        s.free()


def _merged_reference(ora, blocks, q, mean, pend, k):
    """Oracle scan (exact mode) + ring search, pushed into one Shortlist as the engine does, then
    sorted: equal to a merge by (score desc, id asc) because ring ids exceed every block id."""
    op = ora.plan_build(q, eden_mean=mean)
    rid, rsc = ora.scan_blocks(blocks, op, ora.scan_cfg(k=k), threads=4)
    pos, ps = ora.ring_search(pend, q, k)
    ids = np.concatenate([rid, (np.uint64(0xFFFFFFFF) << np.uint64(16)) | pos.astype(np.uint64)])
    sc = np.concatenate([rsc, ps])
    order = np.lexsort((ids, -sc.astype(np.float64)))[:k]
    return ids[order], sc[order]


@pytest.mark.parametrize("n_pending", [0, 1, 40])
def test_engine_scan_merges_ring(ora, dev, n_pending):
    import torch

    M = mb()
    docs = ora.synth_docs(9, 64 * 30, 768)
    mean = ora.eden_fit_prefix(docs)
    blocks = ora.encode_corpus(docs, eden_mean=mean)
    seg = M.Segment.upload(blocks, dev)
    qs, picks = ora.synth_queries(9, docs.shape[0], 3, 3, 768)
    extra = ora.synth_docs(10, max(n_pending, 1), 768)[:n_pending]
    if n_pending:
        extra[0] = qs[0]  # a ring vector that wins outright
    ring = M.DeviceRing(768, 1024, dev)
    for i, e in enumerate(extra):
        assert ring.push(M.PendingVector(i, e, 0, 0)) is None
    k = 128
    desc, keep = M.api._codec_desc(M.PrefixCodec.EDEN_PROD, M.MidCodec.RABITQ, M.EdenFit(64, 4, 1, mean), None)
    cfg = M.ScanConfig(shortlist_cand=k, mode=M.ScanMode.EXACT).to_c()
    plans = C.c_void_p()
    M._capi.check(dev.ptr, dev.lib.mrl_plans_alloc(dev.ptr, 1, 768, C.byref(plans)))
    for qi, q in enumerate(qs):
        dq = torch.from_numpy(np.ascontiguousarray(q)).cuda()
        ids = torch.zeros(k, dtype=torch.int64, device="cuda")
        sc = torch.zeros(k, dtype=torch.float32, device="cuda")
        cs = torch.zeros(2, dtype=torch.int32, device="cuda")
        M._capi.check(dev.ptr, dev.lib.mrl_engine_scan(dev.ptr, seg.ptr, C.c_void_p(dq.data_ptr()), 768, C.byref(desc),
                                                       plans, C.byref(cfg), None, None, ring.ptr if n_pending else None,
                                                       C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                                                       C.c_void_p(cs.data_ptr()), C.c_void_p(cs.data_ptr() + 4)))
        torch.cuda.synchronize()
        n = int(cs[0].item())
        ri, rs = _merged_reference(ora, blocks, q, mean, extra, k)
        assert n == len(ri) == k
        assert np.array_equal(ids[:n].cpu().numpy().view(np.uint64), ri)
        assert np.array_equal(sc[:n].cpu().numpy().view(np.uint32), rs.view(np.uint32))
        if n_pending and qi == 0:  # the ring copy of the query is the best hit
            assert int(ids[:1].cpu().numpy().view(np.uint64)[0]) == 0xFFFFFFFF << 16
    dev.lib.mrl_plans_free(dev.ptr, plans)
    ring.close()
    seg.free()
    del keep


def test_ring_drain_keeps_order(ora, dev):
    M = mb()
    rows = _rows(4, 100, 384)
    ring = M.DeviceRing(384, 128, dev)
    for i in range(50):
        ring.push(M.PendingVector(i, rows[i], 0, 0))
    M._capi.check(dev.ptr, dev.lib.mrl_ring_drain(dev.ptr, ring.ptr, 20))
    del ring.pending[:20]
    q = rows[77]
    got = ring.search_exact(q, 30)
    rp, rs = ora.ring_search(rows[20:50], q, 30)
    assert [i for i, _ in got] == list(rp)
    assert np.array_equal(np.array([s for _, s in got], np.float32).view(np.uint32), rs.view(np.uint32))
    ring.close()


def test_index_dir_lifecycle(ora, dev, tmp_path):
    """IndexEngine create -> ingest (ring, online EDEN fit, flush every 64, live append) -> search
    -> reopen: the resident segment equals the oracle's encode of the same vectors under the fit of
    each flush, searches equal the oracle's merged shortlist, and a reopened index finds the same
    pages, id map and fit."""
    M = mb()
    d = str(tmp_path / "ix")
    cfg = M.EngineConfig(embed_dims=768, shortlist_cand=64, scan_mode=M.ScanMode.EXACT, temporal_filter_enable=False)
    ix = M.IndexDir.create(d, cfg, dev)
    vecs = ora.synth_docs(21, 64 * 3 + 17, 768)
    fits = []
    for i, v in enumerate(vecs):
        assert ix.ingest_vector(v, timestamp=1000 + i) == i
        if (i + 1) % 64 == 0:
            fits.append(ix.eden.mean.copy())
    assert ix.block_count() == 3 and len(ix.ring) == 17
    # oracle pages: each block encoded with the fit as it stood at its flush (online mean)
    ref = np.concatenate([ora.encode_block(vecs[b * 64:(b + 1) * 64], ts=np.arange(b * 64, b * 64 + 64) + 1000,
                                           eden_mean=fits[b]) for b in range(3)])
    on_disk = np.fromfile(os.path.join(d, "segments", "000001.pax"), np.uint8)
    assert np.array_equal(on_disk, ref)
    pages, _ = ix.segment.read_layout()
    assert np.array_equal(pages, M.load_segment(os.path.join(d, "segments", "000001.pax"), dev).read_layout()[0])
    qs, _ = ora.synth_queries(21, vecs.shape[0], 4, 3, 768)
    for q in qs:
        hits = ix.search(q)
        ri, rs = _merged_reference(ora, ref, q, ix.eden.mean, vecs[192:], 64)
        assert [h.id.as_u64() for h in hits] == [int(x) for x in ri]
        assert np.array_equal(np.array([h.score for h in hits], np.float32).view(np.uint32), rs.view(np.uint32))
        pids = ix.passage_ids(hits)
        for (pid, s), h in zip(pids, hits):
            if h.id.block == 0xFFFFFFFF:
                assert pid == 192 + h.id.slot
            else:
                assert pid == h.id.block * 64 + h.id.slot
    m = json.load(open(os.path.join(d, "manifest.json")))
    assert m["blocks_written"] == 3 and m["version"] == "3.5.0" and m["config"]["embed_dims"] == 768
    ix.flush()  # the 17 pending vectors into a tombstone-padded page
    assert ix.block_count() == 4 and len(ix.ring) == 0
    mean = ix.eden.mean.copy()
    ix.close()
    ix2 = M.IndexDir.open(d, dev)
    assert ix2.block_count() == 4 and ix2.next_passage_id == vecs.shape[0]
    assert np.array_equal(ix2.eden.mean, mean)
    assert np.array_equal(ix2.id_map[192:209], np.arange(192, 209)) and np.all(ix2.id_map[209:] == np.iinfo(np.uint64).max)
    ix2.cfg.scan_mode = M.ScanMode.EXACT
    hits = ix2.search(qs[0])
    pages2 = np.fromfile(os.path.join(d, "segments", "000001.pax"), np.uint8)
    ri, rs = _merged_reference(ora, pages2, qs[0], mean, np.zeros((0, 768), np.float32), 64)
    assert [h.id.as_u64() for h in hits] == [int(x) for x in ri]
    ix2.close()


def _dev_rows(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


@pytest.mark.parametrize("n", [0, 1, 63, 200])
def test_ring_search_batch_matches_single(ora, dev, n):
    """mrl_ring_search_batch (one record per query, rows pushed from device memory) equals
    mrl_ring_search of each query, bit for bit; a slot_base only moves the sentinel slots."""
    import torch

    M = mb()
    lib = dev.lib
    dims, n_q, k = 768, 5, 40
    rows = _rows(n + 3, n, dims)
    if n > 8:
        rows[7] = rows[3]
    qs = _rows(11, n_q, dims)
    ring = M.DeviceRing(dims, 1024, dev)
    d_rows = _dev_rows(rows) if n else torch.zeros(1, dims, device="cuda")
    M._capi.check(dev.ptr, lib.mrl_ring_push_device(dev.ptr, ring.ptr, C.c_void_p(d_rows.data_ptr()), n))
    dq = _dev_rows(qs)
    rb = M.record_bytes(k)
    recs = torch.zeros(n_q * rb, dtype=torch.uint8, device="cuda")
    M._capi.check(dev.ptr, lib.mrl_ring_search_batch(dev.ptr, C.c_void_p(dq.data_ptr()), n_q, dims,
                                                     ring.ptr if n else None, 0, k, C.c_void_p(recs.data_ptr())))
    based = torch.zeros_like(recs)  # rank 3's records in a sharded batch
    M._capi.check(dev.ptr, lib.mrl_ring_search_batch(dev.ptr, C.c_void_p(dq.data_ptr()), n_q, dims,
                                                     ring.ptr if n else None, 3 * 4096, k,
                                                     C.c_void_p(based.data_ptr())))
    if n:
        with pytest.raises(M.MrlError, match="slot_base"):
            M._capi.check(dev.ptr, lib.mrl_ring_search_batch(dev.ptr, C.c_void_p(dq.data_ptr()), n_q, dims, ring.ptr,
                                                             65536 - n + 1, k, C.c_void_p(based.data_ptr())))
    one = torch.zeros(rb, dtype=torch.uint8, device="cuda")
    rp = C.c_void_p()
    M._capi.check(dev.ptr, lib.mrl_ring_rows(ring.ptr, C.byref(rp)))
    for q in range(n_q):
        M._capi.check(dev.ptr, lib.mrl_ring_search(dev.ptr, C.c_void_p(dq.data_ptr() + q * dims * 4), rp, n, dims, k,
                                                   C.c_void_p(one.data_ptr())))
        torch.cuda.synchronize()
        a = one.cpu().numpy()
        b = recs[q * rb:(q + 1) * rb].cpu().numpy()
        m = int(a[12 * k:12 * k + 4].view(np.uint32)[0])
        assert m == min(n, k) == int(b[12 * k:12 * k + 4].view(np.uint32)[0])
        assert np.array_equal(a[:8 * m], b[:8 * m]) and np.array_equal(a[8 * k:8 * k + 4 * m], b[8 * k:8 * k + 4 * m])
        pos, sc = ora.ring_search(rows, qs[q], k)
        assert np.array_equal(a[:8 * m].view(np.uint64) & np.uint64(0xFFFF), pos.astype(np.uint64))
        c = based[q * rb:(q + 1) * rb].cpu().numpy()
        assert np.array_equal(c[:8 * m].view(np.uint64), b[:8 * m].view(np.uint64) + np.uint64(3 * 4096))
        assert np.array_equal(c[8 * k:], b[8 * k:])
    ring.close()


def test_live_ingest_on_device(ora, dev):
    """Device-side live ingest: rows pushed from device memory, 64 of them encoded on the device and
    appended (mrl_segment_append_device), the ring drained; the segment equals an upload of the
    oracle's pages, and a batch's merged shortlist (batched scan records + batched ring records,
    mrl_merge_topk_batch) equals mrl_engine_scan of every query."""
    import torch

    M = mb()
    lib = dev.lib
    dims = 768
    docs = ora.synth_docs(51, 64 * 40, dims)
    mean = ora.eden_fit_prefix(docs)
    base = ora.encode_corpus(docs, eden_mean=mean)
    seg = M.Segment.upload(base, dev)
    desc, keep = M.api._codec_desc(M.PrefixCodec.EDEN_PROD, M.MidCodec.RABITQ, M.EdenFit(64, 4, 1, mean), None)
    live = ora.synth_docs(52, 64 + 17, dims)
    ring = M.DeviceRing(dims, 1024, dev)
    d_live = _dev_rows(live)
    M._capi.check(dev.ptr, lib.mrl_ring_push_device(dev.ptr, ring.ptr, C.c_void_p(d_live.data_ptr()), 64 + 17))
    rp = C.c_void_p()
    M._capi.check(dev.ptr, lib.mrl_ring_rows(ring.ptr, C.byref(rp)))
    pax = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    M._capi.check(dev.ptr, lib.mrl_encode_device(dev.ptr, rp, 64, dims, 8, C.byref(desc), C.c_void_p(pax.data_ptr()),
                                                 0, None))
    M._capi.check(dev.ptr, lib.mrl_segment_append_device(dev.ptr, seg.ptr, C.c_void_p(pax.data_ptr()), 1))
    M._capi.check(dev.ptr, lib.mrl_ring_drain(dev.ptr, ring.ptr, 64))
    torch.cuda.synchronize()
    assert seg.block_count() == 41 and dev.lib.mrl_ring_len(ring.ptr) == 17
    ref_pages = np.concatenate([base, ora.encode_block(live[:64], ts=np.arange(64), eden_mean=mean)])
    full = M.Segment.upload(ref_pages, dev)
    assert np.array_equal(seg.read_layout()[0], full.read_layout()[0])
    full.free()
    # a batch against segment + ring, merged per query, against the single-query engine scan
    n_q, k = 9, 64
    qs, _ = ora.synth_queries(51, docs.shape[0], 3, n_q, dims)
    qs[0] = live[70]  # a pending row that must come first
    dq = _dev_rows(qs)
    plans = C.c_void_p()
    M._capi.check(dev.ptr, lib.mrl_plans_alloc(dev.ptr, n_q, dims, C.byref(plans)))
    M._capi.check(dev.ptr, lib.mrl_plan_build_device(dev.ptr, C.c_void_p(dq.data_ptr()), n_q, dims, C.byref(desc),
                                                     plans))
    cfg = M.ScanConfig(shortlist_cand=k).to_c()
    ids = torch.zeros(n_q * k, dtype=torch.int64, device="cuda")
    sc = torch.zeros(n_q * k, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(n_q, dtype=torch.int32, device="cuda")
    st = torch.zeros(n_q, dtype=torch.int32, device="cuda")
    M._capi.check(dev.ptr, lib.mrl_scan_batch_device(dev.ptr, seg.ptr, plans, 0, n_q, C.byref(cfg), None, None,
                                                     C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                                                     C.c_void_p(cnt.data_ptr()), C.c_void_p(st.data_ptr())))
    rb = M.record_bytes(k)
    lists = torch.zeros(2 * n_q * rb, dtype=torch.uint8, device="cuda")
    M._capi.check(dev.ptr, lib.mrl_pack_records(dev.ptr, C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                                                C.c_void_p(cnt.data_ptr()), n_q, k, C.c_void_p(lists.data_ptr())))
    M._capi.check(dev.ptr, lib.mrl_ring_search_batch(dev.ptr, C.c_void_p(dq.data_ptr()), n_q, dims, ring.ptr, 0, k,
                                                     C.c_void_p(lists.data_ptr() + n_q * rb)))
    out_i = torch.zeros(n_q * k, dtype=torch.int64, device="cuda")
    out_s = torch.zeros(n_q * k, dtype=torch.float32, device="cuda")
    out_c = torch.zeros(n_q, dtype=torch.int32, device="cuda")
    M._capi.check(dev.ptr, lib.mrl_merge_topk_batch(dev.ptr, C.c_void_p(lists.data_ptr()), 2, n_q, k, k,
                                                    C.c_void_p(out_i.data_ptr()), C.c_void_p(out_s.data_ptr()),
                                                    C.c_void_p(out_c.data_ptr())))
    torch.cuda.synchronize()
    assert not np.any(st.cpu().numpy() & 8)
    eplans = C.c_void_p()
    M._capi.check(dev.ptr, lib.mrl_plans_alloc(dev.ptr, 1, dims, C.byref(eplans)))
    gi = out_i.cpu().numpy().view(np.uint64).reshape(n_q, k)
    gs = out_s.cpu().numpy().reshape(n_q, k)
    for q in range(n_q):
        e_i = torch.zeros(k, dtype=torch.int64, device="cuda")
        e_s = torch.zeros(k, dtype=torch.float32, device="cuda")
        e_c = torch.zeros(2, dtype=torch.int32, device="cuda")
        M._capi.check(dev.ptr, lib.mrl_engine_scan(dev.ptr, seg.ptr, C.c_void_p(dq.data_ptr() + q * dims * 4), dims,
                                                   C.byref(desc), eplans, C.byref(cfg), None, None, ring.ptr,
                                                   C.c_void_p(e_i.data_ptr()), C.c_void_p(e_s.data_ptr()),
                                                   C.c_void_p(e_c.data_ptr()), C.c_void_p(e_c.data_ptr() + 4)))
        torch.cuda.synchronize()
        n = int(e_c[0].item())
        assert int(out_c[q].item()) == n == k
        assert np.array_equal(gi[q], e_i.cpu().numpy().view(np.uint64))
        assert np.array_equal(gs[q].view(np.uint32), e_s.cpu().numpy().view(np.uint32))
    assert gi[0][0] == (0xFFFFFFFF << 16) | 6  # live[70] is pending row 6 after the drain
    lib.mrl_plans_free(dev.ptr, plans)
    lib.mrl_plans_free(dev.ptr, eplans)
    ring.close()
    seg.free()
    del keep
