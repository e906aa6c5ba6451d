"""mrl_scan_device_static (scan scratch in the library's static device region, no allocation) against
mrl_scan_device (scratch in the context) and against the CPU oracle's scan on the same inputs, and
the property the entry point exists for: once its first call on a device has looked the region up,
its calls leave the device's free memory unchanged.

The file name sorts last so the static region is exercised after every other GPU test has run;
each test also stands alone. The two static calls of a test are issued back to back on the context
stream with no host synchronisation between them.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-6  # same kernel and inputs on both entry points: scores are expected bit-identical


def mb():
    import mrl_b200

    return mrl_b200


@pytest.fixture(scope="module")
def case(ora, dev):
    n = 64 * 300 + 5  # ragged last page
    docs = ora.synth_docs(7, n, 768)
    mean = ora.eden_fit_prefix(docs)
    blocks = ora.encode_corpus(docs, eden_mean=mean)
    seg = mb().Segment.upload(blocks, dev)
    qs, _ = ora.synth_queries(7, n, 3, 3, 768)
    plan = mb().QueryPlan.from_queries(qs, mb().PrefixCodec.EDEN_PROD, mb().MidCodec.RABITQ,
                                       eden=mb().EdenFit(64, 4, 1, mean), dev=dev)
    yield dict(seg=seg, plan=plan, n_q=qs.shape[0], blocks=blocks, qs=qs, mean=mean)
    seg.free()
    plan.free()


def _outputs(n_q, k):
    """Device output buffers filled with sentinels (filled and synchronised before any scan)."""
    import torch

    out = (torch.full((n_q, k), -1, dtype=torch.int64, device="cuda"),
           torch.full((n_q, k), float("nan"), dtype=torch.float32, device="cuda"),
           torch.full((n_q,), 0xFFFF, dtype=torch.int32, device="cuda"),
           torch.full((n_q,), 0xFFFF, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    return out


def _call(dev, fn, seg, plan, n_q, cfg, out):
    ids, sc, cnt, st = out
    c = cfg.to_c()
    mb()._capi.check(dev.ptr, fn(dev.ptr, seg.ptr, plan.ptr, 0, n_q, C.byref(c), None, None,
                                 C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                                 C.c_void_p(cnt.data_ptr()), C.c_void_p(st.data_ptr())))
    return out


def _run(dev, fn, seg, plan, n_q, cfg):
    return _call(dev, fn, seg, plan, n_q, cfg, _outputs(n_q, cfg.shortlist_cand))


def _twice(dev, fn, seg, plan, n_q, cfg):
    """Two calls in a row into separate buffers, no synchronisation between them."""
    o1, o2 = _outputs(n_q, cfg.shortlist_cand), _outputs(n_q, cfg.shortlist_cand)
    _call(dev, fn, seg, plan, n_q, cfg, o1)
    _call(dev, fn, seg, plan, n_q, cfg, o2)
    return _host(o1), _host(o2)


def _host(t):
    import torch

    torch.cuda.synchronize()
    return [x.cpu().numpy() for x in t]


def _compare(ref, got):
    r_ids, r_sc, r_cnt, r_st = ref
    g_ids, g_sc, g_cnt, g_st = got
    np.testing.assert_array_equal(g_cnt, r_cnt)
    # Status bit 0 (the rescan ran) depends on which CTA happened to score which page, so it may
    # differ between any two launches; bit 1 (barrier timeout) must be clear on both.
    assert ((r_st & 2) == 0).all() and ((g_st & 2) == 0).all()
    for q in range(len(r_cnt)):
        n = int(r_cnt[q])
        np.testing.assert_array_equal(g_ids[q, :n], r_ids[q, :n])
        np.testing.assert_allclose(g_sc[q, :n], r_sc[q, :n], rtol=RTOL, atol=0.0)


@pytest.mark.parametrize("mode", ["FAST", "EXACT"])
@pytest.mark.parametrize("k", [16, 256, 1000])
def test_static_matches_context_scratch_twice(dev, case, mode, k):
    cfg = mb().ScanConfig(shortlist_cand=k, mode=getattr(mb().ScanMode, mode))
    lib = dev.lib
    ref = _host(_run(dev, lib.mrl_scan_device, case["seg"], case["plan"], case["n_q"], cfg))
    first, second = _twice(dev, lib.mrl_scan_device_static, case["seg"], case["plan"], case["n_q"], cfg)
    assert (ref[2] == min(k, 64 * 300 + 5)).all()
    assert ((ref[3] & 2) == 0).all()
    _compare(ref, first)
    _compare(ref, second)


@pytest.mark.parametrize("list_len", [1, 4])
def test_static_rescan_path_matches(dev, case, list_len):
    """Short per-CTA lists force the flagged-CTA rescan, which reads the owner bytes and flags."""
    cfg = mb().ScanConfig(shortlist_cand=256, mode=mb().ScanMode.FAST)
    lib = dev.lib
    dev.set_list_len(list_len)
    try:
        ref = _host(_run(dev, lib.mrl_scan_device, case["seg"], case["plan"], case["n_q"], cfg))
        a, b = _twice(dev, lib.mrl_scan_device_static, case["seg"], case["plan"], case["n_q"], cfg)
    finally:
        dev.set_list_len(0)
    assert ((ref[3] & 1) == 1).all()  # the rescan ran
    _compare(ref, a)
    _compare(ref, b)


def test_static_empty_segment(dev, case):
    seg = mb().Segment.upload(np.zeros((0, 4096), np.uint8), dev)
    try:
        cfg = mb().ScanConfig(shortlist_cand=8)
        got = _host(_run(dev, dev.lib.mrl_scan_device_static, seg, case["plan"], case["n_q"], cfg))
        assert (got[2] == 0).all() and (got[3] == 0).all()
    finally:
        seg.free()


def test_static_rejects_segment_over_limit(dev, case):
    """One page over MRL_STATIC_MAX_BLOCKS (2^20): refused with a message naming the limit, and the
    context still scans afterwards. The zero pages are never scanned."""
    big = np.zeros(((1 << 20) + 1, 4096), np.uint8)
    seg = mb().Segment.upload(big, dev)
    del big
    try:
        cfg = mb().ScanConfig(shortlist_cand=8)
        with pytest.raises(mb().MrlError) as ei:
            _run(dev, dev.lib.mrl_scan_device_static, seg, case["plan"], case["n_q"], cfg)
        assert ei.value.code == mb()._capi.MRL_ERR_INVALID
        assert "at most 1048576" in str(ei.value)
    finally:
        seg.free()
    got = _host(_run(dev, dev.lib.mrl_scan_device_static, case["seg"], case["plan"], case["n_q"],
                     mb().ScanConfig(shortlist_cand=8)))
    assert (got[2] == 8).all()


@pytest.mark.parametrize("mode", ["FAST", "EXACT"])
def test_static_matches_oracle_scan(ora, dev, case, mode):
    """Two static calls in a row against the oracle's scan_blocks (the reference's algorithm) of
    every query: ids identical and f32 scores bit-identical."""
    k = 256
    cfg = mb().ScanConfig(shortlist_cand=k, mode=getattr(mb().ScanMode, mode))
    for got in _twice(dev, dev.lib.mrl_scan_device_static, case["seg"], case["plan"], case["n_q"], cfg):
        for q in range(case["n_q"]):
            op = ora.plan_build(case["qs"][q], eden_mean=case["mean"])
            rid, rsc = ora.scan_blocks(case["blocks"], op, ora.scan_cfg(k=k), threads=4)
            n = int(got[2][q])
            assert n == len(rid)
            np.testing.assert_array_equal(got[0][q, :n].view(np.uint64), rid.astype(np.uint64))
            np.testing.assert_array_equal(got[1][q, :n].view(np.uint32), rsc.view(np.uint32))


def test_static_calls_allocate_no_device_memory(ora, dev, case):
    """A fresh context that has never scanned: after its first static call (which looks the region
    up and may load the module), further static calls over segments of growing size, in both modes,
    leave the device's free memory exactly unchanged. A call that allocated (a context scratch
    buffer, or any cudaMalloc) would lower it by at least one allocation granule."""
    import torch

    M = mb()
    fresh = M.Device(0)
    try:
        segs = [M.Segment.upload(case["blocks"][: p * 4096], fresh) for p in (1, 40, 301)]
        plan = M.QueryPlan.from_queries(case["qs"], M.PrefixCodec.EDEN_PROD, M.MidCodec.RABITQ,
                                        eden=M.EdenFit(64, 4, 1, case["mean"]), dev=fresh)
        outs = [_outputs(case["n_q"], 256) for _ in range(7)]
        cfgs = [M.ScanConfig(shortlist_cand=256, mode=m) for m in (M.ScanMode.FAST, M.ScanMode.EXACT)]
        fn = fresh.lib.mrl_scan_device_static
        _call(fresh, fn, segs[0], plan, case["n_q"], cfgs[0], outs[0])
        torch.cuda.synchronize()
        free0, _ = torch.cuda.mem_get_info()
        i = 1
        for sg in segs:
            for c in cfgs:
                _call(fresh, fn, sg, plan, case["n_q"], c, outs[min(i, 6)])
                i += 1
        torch.cuda.synchronize()
        free1, _ = torch.cuda.mem_get_info()
        assert free1 == free0, (free0, free1)
        got = _host(outs[6])
        assert (got[2] == 256).all() and ((got[3] & 2) == 0).all()
        for sg in segs:
            sg.free()
        plan.free()
    finally:
        fresh.close()
