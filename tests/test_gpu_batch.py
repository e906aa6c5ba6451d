"""The batched fast-mode scan (mrl_scan_batch_device, and mrl_scan from 8 plans on), with each of
its engines (tcgen05 kind::i8 tensor cores, CUDA-core tables), against the single-query scan
(mrl_scan_device): identical ids and bit-identical scores for every query that is not reported
uncertified, across codecs, depths, tile remainders, k, tombstones and the temporal filter;
uncertified queries are rerun by mrl_scan, so its results always match. Both end in the exact-mode
scores of the reference's f32 arithmetic (the integer sums only choose the candidates), checked
against the oracle."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def mb():
    import mrl_b200

    return mrl_b200


def _corpus(ora, n, dims=768, seed=31, codec="eden"):
    docs = ora.synth_docs(seed, n, dims)
    mean = ora.eden_fit_prefix(docs)
    if codec == "minmax":
        blocks = ora.encode_corpus(docs, prefix_codec=ora.MINMAX4)
    elif codec == "eden_b1":
        mid = ora.eden_fit_band(docs, 64, 128)
        blocks = ora.encode_corpus(docs, eden_mean=mean, mid_mean=mid)
        return docs, blocks, mean, mid
    else:
        blocks = ora.encode_corpus(docs, eden_mean=mean)
    return docs, blocks, mean, None


def _plans(M, dev, qs, codec, mean, mid):
    if codec == "minmax":
        return M.QueryPlan.from_queries(qs, M.PrefixCodec.MIN_MAX4, dev=dev)
    if codec == "eden_b1":
        return M.QueryPlan.from_queries(qs, M.PrefixCodec.EDEN_PROD, M.MidCodec.EDEN_B1,
                                        eden=M.EdenFit(64, 4, 1, mean), eden_mid=M.EdenFit(128, 1, 1, mid), dev=dev)
    return M.QueryPlan.from_queries(qs, M.PrefixCodec.EDEN_PROD, eden=M.EdenFit(64, 4, 1, mean), dev=dev)


def _run(dev, fn, seg, plans, n_q, cfg_c, k, lo=None, hi=None):
    import torch

    M = mb()
    ids = torch.zeros(n_q * k, dtype=torch.int64, device="cuda")
    sc = torch.zeros(n_q * k, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(n_q, dtype=torch.int32, device="cuda")
    st = torch.zeros(n_q, dtype=torch.int32, device="cuda")
    lo_p = None if lo is None else C.byref(C.c_uint32(lo))
    hi_p = None if hi is None else C.byref(C.c_uint32(hi))
    torch.cuda.synchronize()
    M._capi.check(dev.ptr, fn(dev.ptr, seg.ptr, plans.ptr, 0, n_q, C.byref(cfg_c), lo_p, hi_p, C.c_void_p(ids.data_ptr()),
                              C.c_void_p(sc.data_ptr()), C.c_void_p(cnt.data_ptr()), C.c_void_p(st.data_ptr())))
    torch.cuda.synchronize()
    return (ids.cpu().numpy().view(np.uint64).reshape(n_q, k), sc.cpu().numpy().reshape(n_q, k),
            cnt.cpu().numpy().astype(np.int64), st.cpu().numpy().astype(np.int64))


@pytest.fixture(params=["tensor", "cuda_core"])
def engine(request, dev):
    """Runs a test with each batched-scan engine (tcgen05 kind::i8, CUDA-core tables)."""
    mb()._capi.check(dev.ptr, dev.lib.mrl_set_batch_engine(dev.ptr, 0 if request.param == "tensor" else 1))
    yield request.param
    dev.lib.mrl_set_batch_engine(dev.ptr, 0)


def _compare(single, batch, allow_uncertified=True):
    si, ss, sn, _ = single
    bi, bs, bn, bst = batch
    certified = 0
    for q in range(len(sn)):
        if bst[q] & 8:
            assert allow_uncertified
            continue
        certified += 1
        n = int(sn[q])
        assert int(bn[q]) == n, q
        assert np.array_equal(bi[q, :n], si[q, :n]), q
        assert np.array_equal(bs[q, :n].view(np.uint32), ss[q, :n].view(np.uint32)), q
    return certified


@pytest.mark.parametrize("codec", ["eden", "minmax", "eden_b1"])
@pytest.mark.parametrize("depth", ["FULL_64B", "L1_RABITQ"])
def test_batch_matches_single_query(ora, dev, engine, codec, depth):
    M = mb()
    docs, blocks, mean, mid = _corpus(ora, 64 * 300 + 13, codec=codec)
    seg = M.Segment.upload(blocks, dev)
    n_q = 19  # two full tiles and a remainder of 3 (odd)
    qs, _ = ora.synth_queries(31, docs.shape[0], 5, n_q, 768)
    plans = _plans(M, dev, qs, codec, mean, mid)
    k = 256
    cfg = M.ScanConfig(shortlist_cand=k, strata_depth=getattr(M.StrataDepth, depth)).to_c()
    a = _run(dev, dev.lib.mrl_scan_device, seg, plans, n_q, cfg, k)
    b = _run(dev, dev.lib.mrl_scan_batch_device, seg, plans, n_q, cfg, k)
    assert _compare(a, b) == n_q  # nothing uncertified at this k
    seg.free()
    plans.free()


@pytest.mark.parametrize("n_q", [1, 2, 8, 9, 40])
@pytest.mark.parametrize("k", [1, 16, 1000])
def test_batch_sizes_and_k(ora, dev, engine, n_q, k):
    M = mb()
    docs, blocks, mean, _ = _corpus(ora, 64 * 400, seed=7)
    seg = M.Segment.upload(blocks, dev)
    qs, _ = ora.synth_queries(7, docs.shape[0], 9, n_q, 768)
    plans = _plans(M, dev, qs, "eden", mean, None)
    cfg = M.ScanConfig(shortlist_cand=k).to_c()
    a = _run(dev, dev.lib.mrl_scan_device, seg, plans, n_q, cfg, k)
    b = _run(dev, dev.lib.mrl_scan_batch_device, seg, plans, n_q, cfg, k)
    _compare(a, b)
    seg.free()
    plans.free()


def test_batch_uncertified_rerun_by_mrl_scan(ora, dev, engine):
    """k = 4096 over 200 pages: most SMs' shares hold more than 32 of the top k, so queries are
    reported uncertified; mrl_scan (host entry) reruns them and matches the single-query scan."""
    M = mb()
    docs, blocks, mean, _ = _corpus(ora, 64 * 200, seed=3)
    seg = M.Segment.upload(blocks, dev)
    n_q = 12
    qs, _ = ora.synth_queries(3, docs.shape[0], 4, n_q, 768)
    plans = _plans(M, dev, qs, "eden", mean, None)
    k = 4096
    cfg = M.ScanConfig(shortlist_cand=k)
    a = _run(dev, dev.lib.mrl_scan_device, seg, plans, n_q, cfg.to_c(), k)
    b = _run(dev, dev.lib.mrl_scan_batch_device, seg, plans, n_q, cfg.to_c(), k)
    assert np.all(b[3] & 8)  # every query uncertified at this k
    ids, scores, counts = M.scan_blocks_batch(seg, plans, cfg)  # host entry: batched + reruns
    for q in range(n_q):
        n = int(a[2][q])
        assert int(counts[q]) == n
        assert np.array_equal(ids[q, :n], a[0][q, :n])
        assert np.array_equal(scores[q, :n].view(np.uint32), a[1][q, :n].view(np.uint32))
    seg.free()
    plans.free()


def test_batch_tombstones_and_time_filter(ora, dev, engine):
    M = mb()
    rng = np.random.default_rng(5)
    docs = ora.synth_docs(12, 64 * 60, 768)
    mean = ora.eden_fit_prefix(docs)
    pages = []
    for b in range(60):  # ragged pages (tombstoned tails) with increasing timestamps
        n = int(rng.integers(1, 65))
        ts = np.arange(n, dtype=np.uint32) + 100 * b
        pages.append(ora.encode_block(docs[b * 64:b * 64 + n], ts=ts, eden_mean=mean))
    blocks = np.concatenate(pages)
    seg = M.Segment.upload(blocks, dev, block_id_base=5)
    n_q = 10
    qs, _ = ora.synth_queries(12, docs.shape[0], 2, n_q, 768)
    plans = _plans(M, dev, qs, "eden", mean, None)
    k = 64
    for tf, lo, hi in [(False, None, None), (True, 1000, 4000), (True, None, 2500), (True, 9000, None)]:
        cfg = M.ScanConfig(shortlist_cand=k, temporal_filter_enable=tf).to_c()
        a = _run(dev, dev.lib.mrl_scan_device, seg, plans, n_q, cfg, k, lo, hi)
        b = _run(dev, dev.lib.mrl_scan_batch_device, seg, plans, n_q, cfg, k, lo, hi)
        assert _compare(a, b, allow_uncertified=False) == n_q
        for q in range(n_q):  # ids carry the segment's block_id_base
            assert np.all((b[0][q, :int(b[2][q])] >> np.uint64(16)) >= 5)
    seg.free()
    plans.free()


def test_batch_exact_mode_and_l0_fall_back(ora, dev):
    """Exact mode and L0Only are not batched: the batch entry runs the single-query scan."""
    M = mb()
    docs, blocks, mean, _ = _corpus(ora, 64 * 50, seed=2)
    seg = M.Segment.upload(blocks, dev)
    qs, _ = ora.synth_queries(2, docs.shape[0], 1, 9, 768)
    plans = _plans(M, dev, qs, "eden", mean, None)
    for cfg in (M.ScanConfig(shortlist_cand=32, mode=M.ScanMode.EXACT),
                M.ScanConfig(shortlist_cand=32, strata_depth=M.StrataDepth.L0_ONLY)):
        a = _run(dev, dev.lib.mrl_scan_device, seg, plans, 9, cfg.to_c(), 32)
        b = _run(dev, dev.lib.mrl_scan_batch_device, seg, plans, 9, cfg.to_c(), 32)
        assert _compare(a, b, allow_uncertified=False) == 9
    seg.free()
    plans.free()


def test_batch_against_oracle_exact_topk(ora, dev, engine):
    """The batched top-k equals the oracle's exact-mode top-k (the reference's f32 scores, bit for
    bit) and the oracle's scan_blocks; the fast-mode integer scores only choose the candidates."""
    M = mb()
    docs, blocks, mean, _ = _corpus(ora, 64 * 120 + 5, seed=17)
    seg = M.Segment.upload(blocks, dev)
    n_q = 8
    qs, _ = ora.synth_queries(17, docs.shape[0], 3, n_q, 768)
    plans = _plans(M, dev, qs, "eden", mean, None)
    k = 100
    cfg = M.ScanConfig(shortlist_cand=k)
    b = _run(dev, dev.lib.mrl_scan_batch_device, seg, plans, n_q, cfg.to_c(), k)
    for q in range(n_q):
        op = ora.plan_build(qs[q], eden_mean=mean)
        ocfg = ora.scan_cfg(k=k)
        fs, act = ora.full_scores(blocks, op, ocfg)
        ti, ts = ora.topk_by_key(fs, act, k)
        rid, rsc = ora.scan_blocks(blocks, op, ocfg, threads=4)
        n = int(b[2][q])
        assert n == k and not b[3][q] & 8
        assert np.array_equal(b[0][q, :n], ti)
        assert np.array_equal(b[1][q, :n].view(np.uint32), ts.view(np.uint32))
        assert np.array_equal(b[0][q, :n], rid.astype(np.uint64))
        assert np.array_equal(b[1][q, :n].view(np.uint32), rsc.view(np.uint32))
    seg.free()
    plans.free()


@pytest.mark.parametrize("n_q", [16, 40])
def test_batch_many_pages_per_sm(dev, engine, n_q):
    """A segment of 4,000 pages (27 or 28 per SM, so some CTAs end on a half slot tile): every warp
    scores several pages per tile, so the candidate queues fill and flush repeatedly; 40 queries
    take a group of two query tiles (the second tile's MMAs overlapping the first's scores, the
    next slot tile's overlapping the second's) and a group of one. Results stay identical to the
    single-query scan."""
    import torch

    M = mb()
    lib = dev.lib
    n, dims = 64 * 4000, 768
    x = torch.empty((n, dims), dtype=torch.float32, device="cuda")
    M._capi.check(dev.ptr, lib.mrl_synth_docs_device(dev.ptr, 77, 0, n, dims, C.c_void_p(x.data_ptr())))
    mean = np.zeros(64, np.float32)
    M._capi.check(dev.ptr, lib.mrl_eden_fit_device(dev.ptr, C.c_void_p(x.data_ptr()), n, dims, 0, 64,
                                                   mean.ctypes.data_as(C.c_void_p)))
    desc, keep = M.api._codec_desc(M.PrefixCodec.EDEN_PROD, M.MidCodec.RABITQ, M.EdenFit(64, 4, 1, mean), None)
    sp = C.c_void_p()
    M._capi.check(dev.ptr, lib.mrl_encode_device(dev.ptr, C.c_void_p(x.data_ptr()), n, dims, 8, C.byref(desc), None,
                                                 0, C.byref(sp)))
    seg = M.Segment(sp, dev)
    qd = torch.empty((n_q, dims), dtype=torch.float32, device="cuda")
    M._capi.check(dev.ptr, lib.mrl_synth_queries_device(dev.ptr, 77, n, 5, n_q, dims, C.c_float(0.1),
                                                        C.c_void_p(qd.data_ptr()), None))
    plans = C.c_void_p()
    M._capi.check(dev.ptr, lib.mrl_plans_alloc(dev.ptr, n_q, dims, C.byref(plans)))
    M._capi.check(dev.ptr, lib.mrl_plan_build_device(dev.ptr, C.c_void_p(qd.data_ptr()), n_q, dims, C.byref(desc),
                                                     plans))
    torch.cuda.synchronize()
    del x

    class _P:  # the plans handle in the shape _run expects
        ptr = plans

    for k in (64, 256):
        cfg = M.ScanConfig(shortlist_cand=k).to_c()
        a = _run(dev, lib.mrl_scan_device, seg, _P, n_q, cfg, k)
        b = _run(dev, lib.mrl_scan_batch_device, seg, _P, n_q, cfg, k)
        assert _compare(a, b, allow_uncertified=False) == n_q
    lib.mrl_plans_free(dev.ptr, plans)
    seg.free()
    del keep


def test_batch_records_merge_equals_whole_corpus(ora, dev):
    """Config 4's exchange step on one GPU: three page ranges scanned as separate segments (each
    with its block_id_base), their batched results packed as records (mrl_pack_records), laid out
    rank-major and merged per query (mrl_merge_topk_batch): identical to the batched scan of the
    whole corpus."""
    import torch

    M = mb()
    lib = dev.lib
    docs, blocks, mean, _ = _corpus(ora, 64 * 150, seed=41)
    n_q, k = 20, 64
    qs, _ = ora.synth_queries(41, docs.shape[0], 8, n_q, 768)
    plans = _plans(M, dev, qs, "eden", mean, None)
    cfg = M.ScanConfig(shortlist_cand=k).to_c()
    whole = M.Segment.upload(blocks, dev)
    ref = _run(dev, lib.mrl_scan_batch_device, whole, plans, n_q, cfg, k)
    rb = M.record_bytes(k)
    gathered = torch.zeros(3 * n_q * rb, dtype=torch.uint8, device="cuda")
    pages = blocks.reshape(-1, 4096)
    for r in range(3):
        p0, npg = M.shard_range(pages.shape[0], 3, r)
        seg = M.Segment.upload(pages[p0:p0 + npg].reshape(-1), dev, block_id_base=p0)
        ids = torch.zeros(n_q * k, dtype=torch.int64, device="cuda")
        sc = torch.zeros(n_q * k, dtype=torch.float32, device="cuda")
        cnt = torch.zeros(n_q, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        M._capi.check(dev.ptr, lib.mrl_scan_batch_device(dev.ptr, seg.ptr, plans.ptr, 0, n_q, C.byref(cfg), None, None,
                                                         C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                                                         C.c_void_p(cnt.data_ptr()), None))
        M._capi.check(dev.ptr, lib.mrl_pack_records(dev.ptr, C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                                                    C.c_void_p(cnt.data_ptr()), n_q, k,
                                                    C.c_void_p(gathered.data_ptr() + r * n_q * rb)))
        torch.cuda.synchronize()
        seg.free()
    out_i = torch.zeros(n_q * k, dtype=torch.int64, device="cuda")
    out_s = torch.zeros(n_q * k, dtype=torch.float32, device="cuda")
    out_c = torch.zeros(n_q, dtype=torch.int32, device="cuda")
    M._capi.check(dev.ptr, lib.mrl_merge_topk_batch(dev.ptr, C.c_void_p(gathered.data_ptr()), 3, n_q, k, k,
                                                    C.c_void_p(out_i.data_ptr()), C.c_void_p(out_s.data_ptr()),
                                                    C.c_void_p(out_c.data_ptr())))
    torch.cuda.synchronize()
    got = (out_i.cpu().numpy().view(np.uint64).reshape(n_q, k), out_s.cpu().numpy().reshape(n_q, k),
           out_c.cpu().numpy().astype(np.int64), np.zeros(n_q, np.int64))
    assert _compare(ref, got, allow_uncertified=False) == n_q
    whole.free()
    plans.free()
