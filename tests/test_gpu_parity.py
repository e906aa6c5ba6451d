"""Parity of the CUDA product path (libmrl_b200 through its C ABI) with the CPU oracle.

Bars (tightened): integer stage sums bit-exact; per-slot fast-mode scores
within 1e-5 relative of the reference's f32 scores; every returned top-k, in both modes,
bit-identical to the reference's f32 scores with id lists identical except at exactly tied scores
(the fast mode rescores its candidates in the reference's exact f32 order before the final
ranking).
"""
import ctypes as C
import os
import struct

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-5
ATOL = 1e-6


def mb():
    import mrl_b200

    return mrl_b200


@pytest.fixture(scope="module")
def corpus768(ora):
    n = 64 * 37 + 17  # ragged last block
    docs = ora.synth_docs(42, n, 768)
    mean = ora.eden_fit_prefix(docs)
    eden = ora.encode_corpus(docs, eden_mean=mean)
    minmax = ora.encode_corpus(docs, prefix_codec=ora.MINMAX4)
    qs, picks = ora.synth_queries(42, n, 7, 4, 768)
    return dict(n=n, docs=docs, mean=mean, eden=eden, minmax=minmax, qs=qs, picks=picks)


def fit(mean, dim=64, bits=4):
    return mb().EdenFit(dim, bits, 1, np.asarray(mean, np.float32))


def ids_to_ord(ids):
    return np.array([(int(i) >> 16) * 64 + (int(i) & 0xFFFF) for i in ids], np.int64)


def assert_same_topk(got_ids, got_sc, ref_ids, ref_sc, tol):
    """Equal id lists except where the reference's scores tie within `tol` of each other."""
    assert len(got_ids) == len(ref_ids)
    if tol == 0:
        np.testing.assert_array_equal(np.sort(got_sc)[::-1].view(np.uint32), np.asarray(ref_sc).view(np.uint32))
    else:
        np.testing.assert_allclose(got_sc, ref_sc, rtol=RTOL, atol=ATOL)
    if len(ref_sc) == 0:
        return
    kth = ref_sc[-1]
    diff = set(map(int, got_ids)) ^ set(map(int, ref_ids))
    ref_map = dict(zip(map(int, ref_ids), ref_sc))
    got_map = dict(zip(map(int, got_ids), got_sc))
    for vid in diff:
        s = ref_map.get(vid, got_map.get(vid))
        assert abs(float(s) - float(kth)) <= tol * abs(float(kth)) + (ATOL if tol else 0.0), (vid, s, kth)


# ---- layout and plans ------------------------------------------------------------------------

def test_transcode_matches_oracle(ora, dev, corpus768):
    seg = mb().Segment.upload(corpus768["eden"], dev)
    pages, ts = seg.read_layout()
    nb = corpus768["eden"].size // 4096
    assert seg.block_count() == nb
    for b in range(nb):
        exp, exp_ts = ora.device_layout(corpus768["eden"][b * 4096:(b + 1) * 4096])
        assert np.array_equal(pages[b * 4096:(b + 1) * 4096], exp), b
        assert np.array_equal(ts[2 * b:2 * b + 2], exp_ts)


PLAN_FIELDS = ["prefix", "bit_weights", "rabitq_q", "rabitq_scale", "rabitq_weights2", "rabitq_base", "rabitq_lut",
               "tail_fold_q", "tail_fold_weights2", "tail_fold_base", "q_tail_norm", "q_mid_norm", "q_after_prefix",
               "q_after_s1", "s4_abs_budget", "prefix_l1", "prefix_sum", "eden_q_rot", "eden_mean_ip",
               "eden_inv_sqrt_d", "eden_codebook", "eden_mid_q_rot", "eden_mid_mean_ip", "eden_mid_inv_sqrt_d",
               "eden_mid_codebook", "dims", "prefix_codec", "mid_codec", "has_tail_fold"]


@pytest.mark.parametrize("dims", [192, 200, 384, 768, 1000])
@pytest.mark.parametrize("codec", ["minmax", "eden", "eden_b1"])
def test_plan_fields_bit_identical(ora, dev, dims, codec):
    rng = np.random.default_rng(dims)
    q = rng.standard_normal(dims).astype(np.float32)
    q /= np.linalg.norm(q)
    mean = (rng.standard_normal(64) * 0.05).astype(np.float32)
    mid_mean = (rng.standard_normal(128) * 0.05).astype(np.float32)
    M = mb()
    if codec == "minmax":
        gp = M.QueryPlan.from_query(q, dims, dev=dev)
        op = ora.plan_build(q, prefix_codec=ora.MINMAX4)
    elif codec == "eden":
        gp = M.QueryPlan.from_query_eden(q, dims, fit(mean), dev=dev)
        op = ora.plan_build(q, prefix_codec=ora.EDEN_PROD, eden_mean=mean)
    else:
        gp = M.QueryPlan.from_query_eden_dual(q, dims, fit(mean), fit(mid_mean, 128, 1), dev=dev)
        op = ora.plan_build(q, prefix_codec=ora.EDEN_PROD, mid_codec=ora.EDEN_B1, eden_mean=mean, mid_mean=mid_mean)
    g = gp.fields(0)
    for f in PLAN_FIELDS:
        a = np.ctypeslib.as_array(getattr(g, f)) if not isinstance(getattr(g, f), (int, float)) else np.array(getattr(g, f))
        b = np.ctypeslib.as_array(getattr(op, f)) if not isinstance(getattr(op, f), (int, float)) else np.array(getattr(op, f))
        assert np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32)), f


def test_plan_rejects_contract_violations(dev):
    M = mb()
    with pytest.raises(ValueError):
        M.QueryPlan.from_query(np.zeros(100, np.float32), 100, dev=dev)  # dims < 192
    with pytest.raises(ValueError):
        M.QueryPlan.from_queries(np.zeros((1, 768), np.float32), M.PrefixCodec.EDEN_PROD, dev=dev)  # no fit
    q = np.zeros(768, np.float32)
    q[5] = np.nan
    with pytest.raises(M.MrlError):
        M.QueryPlan.from_query(q, 768, dev=dev)


# ---- per-slot scores ---------------------------------------------------------------------------

@pytest.mark.parametrize("depth", [0, 1, 2])
@pytest.mark.parametrize("codec", ["eden", "minmax"])
def test_exact_mode_scores_bit_identical(ora, dev, corpus768, depth, codec):
    M = mb()
    blocks = corpus768[codec]
    seg = M.Segment.upload(blocks, dev)
    for q in corpus768["qs"][:2]:
        if codec == "eden":
            gp = M.QueryPlan.from_query_eden(q, 768, fit(corpus768["mean"]), dev=dev)
            op = ora.plan_build(q, prefix_codec=ora.EDEN_PROD, eden_mean=corpus768["mean"])
        else:
            gp = M.QueryPlan.from_query(q, 768, dev=dev)
            op = ora.plan_build(q, prefix_codec=ora.MINMAX4)
        cfg = M.ScanConfig(shortlist_cand=64, strata_depth=M.StrataDepth(depth), mode=M.ScanMode.EXACT)
        sc, act, _ = M.vector_scores(seg, gp, cfg)
        rsc, ract = ora.full_scores(blocks, op, ora.scan_cfg(k=64, strata_depth=depth))
        assert np.array_equal(act, ract)
        assert np.array_equal(sc[act == 1].view(np.uint32), rsc[act == 1].view(np.uint32))


@pytest.mark.parametrize("depth", [0, 1, 2])
@pytest.mark.parametrize("codec", ["eden", "minmax"])
def test_fast_mode_integer_sums_bit_exact(ora, dev, corpus768, depth, codec):
    M = mb()
    blocks = corpus768[codec]
    seg = M.Segment.upload(blocks, dev)
    for q in corpus768["qs"][:2]:
        if codec == "eden":
            gp = M.QueryPlan.from_query_eden(q, 768, fit(corpus768["mean"]), dev=dev)
            op = ora.plan_build(q, prefix_codec=ora.EDEN_PROD, eden_mean=corpus768["mean"])
        else:
            gp = M.QueryPlan.from_query(q, 768, dev=dev)
            op = ora.plan_build(q, prefix_codec=ora.MINMAX4)
        cfg = M.ScanConfig(shortlist_cand=64, strata_depth=M.StrataDepth(depth), mode=M.ScanMode.FAST)
        ocfg = ora.scan_cfg(k=64, strata_depth=depth)
        sc, act, parts = M.vector_scores(seg, gp, cfg)
        fp = ora.fixed_plan_build(op, ocfg)
        oparts, osc, oact = ora.fixed_scores(blocks, op, fp, ocfg)
        assert np.array_equal(act, oact)
        a = act == 1
        assert np.array_equal(parts[a], oparts[a])                                 # integer sums: bit-exact
        assert np.array_equal(sc[a].view(np.uint32), osc[a].view(np.uint32))       # same f32 assembly
        rsc, _ = ora.full_scores(blocks, op, ocfg)
        np.testing.assert_allclose(sc[a], rsc[a], rtol=RTOL, atol=ATOL)            # vs reference f32
        # the bound the fast mode's final ranking relies on holds for every slot, and is tight
        # enough to leave only near-ties for the exact rescoring
        E = M.score_bound(seg, gp, cfg)
        dev_max = float(np.max(np.abs(sc[a].astype(np.float64) - rsc[a].astype(np.float64))))
        assert dev_max <= E, (dev_max, E)
        assert E < 1e-3 * float(np.max(np.abs(rsc[a]))), E


def test_eden_b1_mid_codec(ora, dev):
    """EdenB1 mid band (src/scan.rs:521-551, src/quantize.rs:265-295) end to end."""
    M = mb()
    docs = ora.synth_docs(8, 64 * 6, 768)
    mean = ora.eden_fit_prefix(docs)
    mid_mean = ora.eden_fit_band(docs, 64, 128)
    blocks = ora.encode_corpus(docs, eden_mean=mean, mid_mean=mid_mean)
    gb = M.encode_blocks(docs, 768, eden=fit(mean), eden_mid=fit(mid_mean, 128, 1), dev=dev)
    assert np.array_equal(gb, blocks)
    seg = M.Segment.upload(blocks, dev)
    q, _ = ora.synth_queries(8, docs.shape[0], 1, 1, 768)
    gp = M.QueryPlan.from_query_eden_dual(q[0], 768, fit(mean), fit(mid_mean, 128, 1), dev=dev)
    op = ora.plan_build(q[0], prefix_codec=ora.EDEN_PROD, mid_codec=ora.EDEN_B1, eden_mean=mean, mid_mean=mid_mean)
    ex, act, _ = M.vector_scores(seg, gp, M.ScanConfig(shortlist_cand=32, mode=M.ScanMode.EXACT))
    rsc, ract = ora.full_scores(blocks, op, ora.scan_cfg(k=32))
    assert np.array_equal(ex[act == 1].view(np.uint32), rsc[ract == 1].view(np.uint32))
    fa, act2, _ = M.vector_scores(seg, gp, M.ScanConfig(shortlist_cand=32, mode=M.ScanMode.FAST))
    np.testing.assert_allclose(fa[act2 == 1], rsc[ract == 1], rtol=RTOL, atol=ATOL)
    rid, rs = ora.scan_blocks(blocks, op, ora.scan_cfg(k=32))
    for mode in (M.ScanMode.EXACT, M.ScanMode.FAST):
        hits = M.scan_blocks(seg, gp, M.ScanConfig(shortlist_cand=32, mode=mode))
        assert [h.id.as_u64() for h in hits] == [int(i) for i in rid]
        assert np.array_equal(np.array([h.score for h in hits], np.float32).view(np.uint32), rs.view(np.uint32))


# ---- top-k --------------------------------------------------------------------------------------

@pytest.mark.parametrize("k", [1, 16, 64, 256, 1000])
@pytest.mark.parametrize("mode", ["exact", "fast"])
def test_scan_topk_matches_reference_scan(ora, dev, corpus768, k, mode):
    M = mb()
    seg = M.Segment.upload(corpus768["eden"], dev)
    qs = corpus768["qs"]
    plans = M.QueryPlan.from_queries(qs, M.PrefixCodec.EDEN_PROD, eden=fit(corpus768["mean"]), dev=dev)
    cfg = M.ScanConfig(shortlist_cand=k, mode=M.ScanMode.EXACT if mode == "exact" else M.ScanMode.FAST)
    ids, scores, counts = M.scan_blocks_batch(seg, plans, cfg)
    for qi, q in enumerate(qs):
        op = ora.plan_build(q, eden_mean=corpus768["mean"])
        ocfg = ora.scan_cfg(k=k)
        rid, rsc = ora.scan_blocks(corpus768["eden"], op, ocfg, threads=4)   # the reference's scan
        n = int(counts[qi])
        gi, gs = ids[qi, :n], scores[qi, :n]
        assert np.all(np.diff(gs) <= 0)                                       # sorted, descending
        assert_same_topk(gi, gs, rid, rsc, 0)                                # tolerance 0, both modes
        fs, act = ora.full_scores(corpus768["eden"], op, ocfg)
        ti, ts = ora.topk_by_key(fs, act, k)                                  # exact top-k, ties to lower ids
        assert np.array_equal(gi, ti) and np.array_equal(gs.view(np.uint32), ts.view(np.uint32))


@pytest.mark.parametrize("k", [16, 256])
@pytest.mark.parametrize("mode", ["exact", "fast"])
@pytest.mark.parametrize("codec", ["minmax", "eden", "eden_b1"])
def test_fused_query_scan_matches_plan_then_scan(ora, dev, corpus768, codec, mode, k):
    """mrl_query_scan (plan built inside the scan launch) against mrl_plan_build + mrl_scan: the
    stored plans are bit-identical to the plan kernel's and the results are identical."""
    M = mb()
    qs = corpus768["qs"]
    mean = corpus768["mean"]
    mid_mean = (np.random.default_rng(3).standard_normal(128) * 0.05).astype(np.float32)
    if codec == "minmax":
        seg = M.Segment.upload(corpus768["minmax"], dev)
        kw = dict(prefix_codec=M.PrefixCodec.MIN_MAX4, mid_codec=M.MidCodec.RABITQ)
    elif codec == "eden":
        seg = M.Segment.upload(corpus768["eden"], dev)
        kw = dict(prefix_codec=M.PrefixCodec.EDEN_PROD, mid_codec=M.MidCodec.RABITQ, eden=fit(mean))
    else:
        seg = M.Segment.upload(corpus768["eden"], dev)
        kw = dict(prefix_codec=M.PrefixCodec.EDEN_PROD, mid_codec=M.MidCodec.EDEN_B1, eden=fit(mean),
                  eden_mid=fit(mid_mean, 128, 1))
    cfg = M.ScanConfig(shortlist_cand=k, mode=M.ScanMode.EXACT if mode == "exact" else M.ScanMode.FAST)
    ref_plans = M.QueryPlan.from_queries(qs, dev=dev, **kw)
    r_ids, r_sc, r_cnt = M.scan_blocks_batch(seg, ref_plans, cfg)
    f_ids, f_sc, f_cnt, f_plans = M.query_scan(seg, qs, cfg, **kw)
    assert np.array_equal(f_cnt, r_cnt)
    for qi in range(len(qs)):
        n = int(r_cnt[qi])
        assert np.array_equal(f_ids[qi, :n], r_ids[qi, :n])
        assert np.array_equal(f_sc[qi, :n].view(np.uint32), r_sc[qi, :n].view(np.uint32))
        a, b = f_plans.fields(qi), ref_plans.fields(qi)
        for f in PLAN_FIELDS:
            x, y = getattr(a, f), getattr(b, f)
            x = np.array(x) if isinstance(x, (int, float)) else np.ctypeslib.as_array(x)
            y = np.array(y) if isinstance(y, (int, float)) else np.ctypeslib.as_array(y)
            assert np.array_equal(np.asarray(x, np.float32).view(np.uint32), np.asarray(y, np.float32).view(np.uint32)), f
    f_plans.free()
    ref_plans.free()
    seg.free()


def test_fused_query_scan_edge_cases(ora, dev, corpus768):
    """Empty segment (plans still built), temporal filter, QueryPipeline.search."""
    M = mb()
    q = corpus768["qs"][:2]
    kw = dict(prefix_codec=M.PrefixCodec.EDEN_PROD, eden=fit(corpus768["mean"]))
    empty = M.Segment.upload(np.zeros(0, np.uint8), dev)
    ids, sc, cnt, plans = M.query_scan(empty, q, M.ScanConfig(shortlist_cand=16), **kw)
    assert cnt.tolist() == [0, 0]
    ref = M.QueryPlan.from_queries(q, dev=dev, **kw)
    assert np.array_equal(np.ctypeslib.as_array(plans.fields(1).eden_q_rot),
                          np.ctypeslib.as_array(ref.fields(1).eden_q_rot))
    seg = M.Segment.upload(corpus768["eden"], dev)
    cfg = M.ScanConfig(shortlist_cand=64, temporal_filter_enable=True)
    ids, sc, cnt, _ = M.query_scan(seg, q, cfg, time_lo=64 * 30, **kw)
    assert all(int(i) >> 16 >= 30 for i in ids[0, : cnt[0]])  # ts = row index: pages 0-29 end before 1920
    r_ids, r_sc, r_cnt = M.scan_blocks_batch(seg, ref, cfg, time_lo=64 * 30)
    assert np.array_equal(ids, r_ids) and np.array_equal(cnt, r_cnt)
    pipe = M.QueryPipeline.with_eden(M.EngineConfig(embed_dims=768, shortlist_cand=64), fit(corpus768["mean"]), dev=dev)
    hits = pipe.search(q[0], seg)
    plan = pipe.build_plan(q[0])
    assert hits == M.scan_blocks(seg, plan, pipe.cfg)


def test_forced_reselection_is_exact(ora, dev, corpus768):
    """A per-CTA list of 1, 2 or 4 entries forces the verification to fail and CTA 0 to rescan the
    flagged CTAs' pages and reselect by exact key: the result must still be the exact top-k, in
    both modes (fast mode rescores the rescanned slots in the exact f32 order)."""
    M = mb()
    seg = M.Segment.upload(corpus768["eden"], dev)
    q = corpus768["qs"][0]
    gp = M.QueryPlan.from_query_eden(q, 768, fit(corpus768["mean"]), dev=dev)
    op = ora.plan_build(q, eden_mean=corpus768["mean"])
    fs, act = ora.full_scores(corpus768["eden"], op, ora.scan_cfg(k=256))
    ti, ts = ora.topk_by_key(fs, act, 256)
    try:
        for mode in (M.ScanMode.EXACT, M.ScanMode.FAST):
            for ll in (1, 2, 4):
                dev.set_list_len(ll)
                hits = M.scan_blocks(seg, gp, M.ScanConfig(shortlist_cand=256, mode=mode))
                assert [h.id.as_u64() for h in hits] == [int(i) for i in ti], (mode, ll)
                assert np.array_equal(np.array([h.score for h in hits], np.float32).view(np.uint32),
                                      ts.view(np.uint32)), (mode, ll)
    finally:
        dev.set_list_len(0)


def test_ties_resolve_to_lower_slot(ora, dev):
    """Identical vectors tie exactly; the result keeps the lowest (block, slot) ids, and the
    heavy concentration of tied winners in the first pages exercises the exact re-selection."""
    M = mb()
    row = ora.synth_docs(3, 1, 768)
    docs = np.repeat(row, 64 * 20, axis=0)
    blocks = ora.encode_corpus(docs, prefix_codec=ora.MINMAX4)
    seg = M.Segment.upload(blocks, dev)
    gp = M.QueryPlan.from_query(row[0], 768, dev=dev)
    for mode in (M.ScanMode.EXACT, M.ScanMode.FAST):
        hits = M.scan_blocks(seg, gp, M.ScanConfig(shortlist_cand=100, mode=mode))
        assert [h.id.block * 64 + h.id.slot for h in hits] == list(range(100))
        assert len(set(h.score for h in hits)) == 1


def test_order_dependent_configs_refused(ora, dev, corpus768):
    """cs_tolerance / stratum4_weight outside the region where the reference's pruning bounds are
    never below a full score make its result depend on the block scan order: such scans fail with
    MRL_ERR_INVALID naming the condition. Inside the region (e.g. cs_tolerance 0.9 at L1Rabitq,
    cs_tolerance 1.2 with stratum4_weight 0.5 at 768 dims) the results equal the oracle's scan."""
    M = mb()
    seg = M.Segment.upload(corpus768["eden"], dev)
    q = corpus768["qs"][1]
    gp = M.QueryPlan.from_query_eden(q, 768, fit(corpus768["mean"]), dev=dev)
    op = ora.plan_build(q, eden_mean=corpus768["mean"])
    for alpha, w, depth, msg in ((0.9, 0.2, 2, "cs_tolerance < 1"), (1.0, 1.0, 2, "stratum4_weight"),
                                 (1.2, 0.6, 2, "stratum4_weight"), (0.75, 0.2, 1, "sqrt(2/pi)")):
        cfg = M.ScanConfig(shortlist_cand=64, cs_tolerance=alpha, stratum4_weight=w, strata_depth=M.StrataDepth(depth))
        with pytest.raises(M.MrlError, match=msg.replace("(", r"\(").replace(")", r"\)")):
            M.scan_blocks(seg, gp, cfg)
    for alpha, w, depth in ((0.9, 0.2, 1), (0.8, 1.5, 1), (1.2, 0.5, 2), (0.8, 0.2, 0)):
        for mode in (M.ScanMode.EXACT, M.ScanMode.FAST):
            cfg = M.ScanConfig(shortlist_cand=64, cs_tolerance=alpha, stratum4_weight=w,
                               strata_depth=M.StrataDepth(depth), mode=mode)
            hits = M.scan_blocks(seg, gp, cfg)
            rid, rsc = ora.scan_blocks(corpus768["eden"], op, ora.scan_cfg(k=64, cs_tolerance=alpha, stratum4_weight=w,
                                                                            strata_depth=depth))
            assert [h.id.as_u64() for h in hits] == [int(i) for i in rid], (alpha, w, depth, mode)
            assert np.array_equal(np.array([h.score for h in hits], np.float32).view(np.uint32), rsc.view(np.uint32))
    gp.free()
    seg.free()


def test_control_words_left_zero(ora, dev, corpus768):
    """Every launch's last CTA to exit zeroes its scratch set's control words, on the clean path,
    the re-selection path and the fused path alike, so a launch never inherits a page counter or
    ticket count from the launch that used the set before."""
    M = mb()
    seg = M.Segment.upload(corpus768["eden"], dev)
    qs = corpus768["qs"]
    gp = M.QueryPlan.from_queries(qs, M.PrefixCodec.EDEN_PROD, eden=fit(corpus768["mean"]), dev=dev)
    try:
        for ll in (0, 1):
            dev.set_list_len(ll)
            for mode in (M.ScanMode.EXACT, M.ScanMode.FAST):
                M.scan_blocks_batch(seg, gp, M.ScanConfig(shortlist_cand=256, mode=mode))
                w = M.control_words(dev)
                assert list(w) == [0] * 128, (ll, mode, w)
        M.query_scan(seg, qs, M.ScanConfig(shortlist_cand=64), prefix_codec=M.PrefixCodec.EDEN_PROD,
                     eden=fit(corpus768["mean"]))
        w = M.control_words(dev)
        assert list(w) == [0] * 128, w
    finally:
        dev.set_list_len(0)
    gp.free()
    seg.free()


def _oracle_stage_counts(ora, blocks, op, ocfg, tau, depth, time_lo=None):
    """ScanStats from the oracle's per-block stage functions (src/scan.rs:453-634) at one tau."""
    exp = [0] * 6
    for b in range(blocks.size // 4096):
        blk = blocks[b * 4096:(b + 1) * 4096]
        if time_lo is not None and struct.unpack_from("<I", blk, 4)[0] < time_lo:
            continue  # temporal skip (src/scan.rs:719-730)
        act = 64 - bin(struct.unpack_from("<Q", blk, 16)[0]).count("1")
        if act == 0:
            continue
        masks, _ = ora.block_stages(blk, op, ocfg, tau)
        m = [bin(int(x)).count("1") for x in masks]
        exp[0] += 1
        exp[1] += act
        exp[2] += m[0]
        exp[3] += m[1]
        exp[4] += m[2] if depth == 2 else m[1]
        exp[5] += m[2] if depth == 2 else m[1]
    return exp


@pytest.mark.parametrize("k", [16, 256])
@pytest.mark.parametrize("depth,alpha", [(2, 1.0), (2, 1.2), (1, 0.9)])
def test_scan_stats_match_oracle_stages(ora, dev, corpus768, depth, alpha, k):
    """mrl_scan_blocks_stats (scan_blocks_stats): the hits equal the oracle's scan and the ScanStats
    counters equal the sums of the oracle's per-block stage masks (the reference's stage functions
    and Cauchy-Schwarz bounds) evaluated at the final shortlist threshold, with and without the
    temporal filter."""
    M = mb()
    blocks = corpus768["eden"]
    mean = corpus768["mean"]
    seg = M.Segment.upload(blocks, dev)
    for qi, q in enumerate(corpus768["qs"][:2]):
        gp = M.QueryPlan.from_query_eden(q, 768, fit(mean), dev=dev)
        op = ora.plan_build(q, eden_mean=mean)
        lo = None if qi == 0 else 64 * 9
        cfg = M.ScanConfig(shortlist_cand=k, strata_depth=M.StrataDepth(depth), cs_tolerance=alpha)
        hits, st = M.scan_blocks_stats(seg, gp, cfg, time_lo=lo)
        ocfg = ora.scan_cfg(k=k, strata_depth=depth, cs_tolerance=alpha, temporal_filter_enable=True)
        rid, rsc = ora.scan_blocks(blocks, op, ocfg, time_lo=lo, threads=4)
        assert [h.id.as_u64() for h in hits] == [int(i) for i in rid]
        tau = float(rsc[-1]) if len(rsc) == k else float("-inf")
        exp = _oracle_stage_counts(ora, blocks, op, ocfg, tau, depth, time_lo=lo)
        got = [st.blocks, st.active_vecs, st.after_prefix, st.after_s1, st.after_s4_budget, st.pushed]
        assert got == exp, (got, exp)
        assert st.pushed >= len(hits)  # every hit survived every bound
        gp.free()
    # L0Only: one bound, every counter equal; an empty segment counts nothing
    gp = M.QueryPlan.from_query_eden(corpus768["qs"][0], 768, fit(mean), dev=dev)
    _, st0 = M.scan_blocks_stats(seg, gp, M.ScanConfig(shortlist_cand=k, strata_depth=M.StrataDepth.L0_ONLY))
    assert st0.after_prefix == st0.after_s1 == st0.after_s4_budget == st0.pushed <= st0.active_vecs
    empty = M.Segment.upload(np.zeros(0, np.uint8), dev)
    hits_e, st_e = M.scan_blocks_stats(empty, gp, M.ScanConfig(shortlist_cand=k))
    assert hits_e == [] and st_e == M.ScanStats()
    gp.free()
    seg.free()


def test_edge_cases(ora, dev):
    M = mb()
    docs = ora.synth_docs(4, 64 * 3, 384)
    blocks = ora.encode_corpus(docs, prefix_codec=ora.MINMAX4)
    # tombstone everything in block 1 and flip one slot of block 2
    b = blocks.copy().reshape(3, 4096)
    b[1, 16:24] = 0xFF
    t = struct.unpack_from("<Q", b[2], 16)[0] | (1 << 5)
    struct.pack_into("<Q", b[2], 16, t)
    blocks2 = b.reshape(-1)
    seg = M.Segment.upload(blocks2, dev, block_id_base=1000)
    gp = M.QueryPlan.from_query(docs[0], 384, dev=dev)
    op = ora.plan_build(docs[0], prefix_codec=ora.MINMAX4)
    for mode in (M.ScanMode.EXACT, M.ScanMode.FAST):
        hits = M.scan_blocks(seg, gp, M.ScanConfig(shortlist_cand=4096, mode=mode))
        assert len(hits) == 64 + 63                                   # K > live slots
        assert all(h.id.block in (1000, 1002) for h in hits)
        assert all(not (h.id.block == 1002 and h.id.slot == 5) for h in hits)
        rid, rsc = ora.scan_blocks(blocks2, op, ora.scan_cfg(k=4096))
        exp = sorted(((int(i) >> 16) + 1000) << 16 | (int(i) & 0xFFFF) for i in rid)
        assert sorted(h.id.as_u64() for h in hits) == exp
    # empty segment
    empty = M.Segment.upload(np.zeros(0, np.uint8), dev)
    assert M.scan_blocks(empty, gp, M.ScanConfig(shortlist_cand=10)) == []
    # temporal filter (src/scan.rs:719-730): ts = row index, keep block 2 only
    seg_t = M.Segment.upload(blocks, dev)
    hits = M.scan_blocks(seg_t, gp, M.ScanConfig(shortlist_cand=500, temporal_filter_enable=True), time_lo=128)
    assert len(hits) == 64 and all(h.id.block == 2 for h in hits)
    hits = M.scan_blocks(seg_t, gp, M.ScanConfig(shortlist_cand=500, temporal_filter_enable=False), time_lo=128)
    assert len(hits) == 192


def test_append_live(ora, dev):
    M = mb()
    docs = ora.synth_docs(6, 64 * 5, 768)
    mean = ora.eden_fit_prefix(docs)
    blocks = ora.encode_corpus(docs, eden_mean=mean)
    seg = M.Segment.upload(blocks[: 2 * 4096], dev)
    for b in range(2, 5):
        seg.append_live(blocks[b * 4096:(b + 1) * 4096])
    assert seg.block_count() == 5
    full = M.Segment.upload(blocks, dev)
    gp = M.QueryPlan.from_query_eden(docs[7], 768, fit(mean), dev=dev)
    cfg = M.ScanConfig(shortlist_cand=64)
    assert M.scan_blocks(seg, gp, cfg) == M.scan_blocks(full, gp, cfg)
    assert np.array_equal(seg.read_layout()[0], full.read_layout()[0])


# ---- encode + synthetic inputs ------------------------------------------------------------------

@pytest.mark.parametrize("dims", [384, 768])
@pytest.mark.parametrize("codec", ["eden", "minmax"])
def test_encode_blocks_byte_identical(ora, dev, dims, codec):
    M = mb()
    n = 64 * 5 + 9
    docs = ora.synth_docs(13, n, dims)
    mean = ora.eden_fit_prefix(docs)
    ts = (np.arange(n) * 7 + 100).astype(np.uint32)
    src = (1 << (np.arange(n) % 4)).astype(np.uint32)
    if codec == "eden":
        got = M.encode_blocks(docs, dims, eden=fit(mean), timestamps=ts, sources=src, dev=dev)
    else:
        got = M.encode_blocks(docs, dims, timestamps=ts, sources=src, dev=dev)
    exp = np.concatenate([ora.encode_block(docs[b:b + 64], ts=ts[b:b + 64], src=src[b:b + 64],
                                           prefix_codec=ora.EDEN_PROD if codec == "eden" else ora.MINMAX4,
                                           eden_mean=mean) for b in range(0, n, 64)])
    assert np.array_equal(got, exp)
    for b in range(got.size // 4096):
        assert ora.verify_crc(got[b * 4096:(b + 1) * 4096])


def test_synth_fit_encode_device_match_oracle(ora, dev):
    torch = pytest.importorskip("torch")
    M = mb()
    lib = M.load()
    n, dims = 64 * 9 + 3, 768
    x = torch.empty((n, dims), dtype=torch.float32, device="cuda")
    assert lib.mrl_synth_docs_device(dev.ptr, 42, 0, n, dims, C.c_void_p(x.data_ptr())) == 0
    docs = ora.synth_docs(42, n, dims)
    assert np.array_equal(x.cpu().numpy(), docs)
    qd = torch.empty((5, dims), dtype=torch.float32, device="cuda")
    pk = torch.empty(5, dtype=torch.int64, device="cuda")
    assert lib.mrl_synth_queries_device(dev.ptr, 42, n, 7, 5, dims, C.c_float(0.1), C.c_void_p(qd.data_ptr()),
                                        C.c_void_p(pk.data_ptr())) == 0
    oq, opk = ora.synth_queries(42, n, 7, 5, dims)
    assert np.array_equal(qd.cpu().numpy(), oq) and np.array_equal(pk.cpu().numpy().astype(np.uint64), opk)
    mean = np.zeros(64, np.float32)
    assert lib.mrl_eden_fit_device(dev.ptr, C.c_void_p(x.data_ptr()), n, dims, 0, 64,
                                   mean.ctypes.data_as(C.c_void_p)) == 0
    assert np.array_equal(mean, ora.eden_fit_prefix(docs))
    pax = torch.empty(((n + 63) // 64) * 4096, dtype=torch.uint8, device="cuda")
    desc, keep = M.api._codec_desc(M.PrefixCodec.EDEN_PROD, M.MidCodec.RABITQ, fit(mean), None)
    segp = C.c_void_p()
    assert lib.mrl_encode_device(dev.ptr, C.c_void_p(x.data_ptr()), n, dims, 8, C.byref(desc),
                                 C.c_void_p(pax.data_ptr()), 0, C.byref(segp)) == 0
    blocks = ora.encode_corpus(docs, eden_mean=mean)
    assert np.array_equal(pax.cpu().numpy(), blocks)
    seg = M.Segment(segp, dev)
    ref = M.Segment.upload(blocks, dev)
    assert np.array_equal(seg.read_layout()[0], ref.read_layout()[0])
    assert np.array_equal(seg.read_layout()[1], ref.read_layout()[1])


# ---- full size (BASELINE config 2 shapes): size-independent properties ---------------------------

def test_full_size_1m_properties(ora, dev):
    """1,000,000 x 768 docs synthesised, fitted and encoded on the device:
    the device blocks of sampled pages equal the oracle's encode of the same rows; exact-mode
    per-slot scores of sampled pages equal the oracle's bit for bit; exact mode returns the exact
    top-256 of its per-slot scores; fast mode returns the same hits bit for bit; and for several
    queries both modes' top-256 equal the oracle's scan_blocks over the same 1M-vector corpus
    (ids and f32 score bits, tolerance 0)."""
    torch = pytest.importorskip("torch")
    M = mb()
    lib = M.load()
    n, dims, k = 1_000_000, 768, 256
    x = torch.empty((n, dims), dtype=torch.float32, device="cuda")
    assert lib.mrl_synth_docs_device(dev.ptr, 42, 0, n, dims, C.c_void_p(x.data_ptr())) == 0
    mean = np.zeros(64, np.float32)
    assert lib.mrl_eden_fit_device(dev.ptr, C.c_void_p(x.data_ptr()), n, dims, 0, 64,
                                   mean.ctypes.data_as(C.c_void_p)) == 0
    nb = (n + 63) // 64
    pax = torch.empty(nb * 4096, dtype=torch.uint8, device="cuda")
    desc, keep = M.api._codec_desc(M.PrefixCodec.EDEN_PROD, M.MidCodec.RABITQ, fit(mean), None)
    segp = C.c_void_p()
    assert lib.mrl_encode_device(dev.ptr, C.c_void_p(x.data_ptr()), n, dims, 8, C.byref(desc),
                                 C.c_void_p(pax.data_ptr()), 0, C.byref(segp)) == 0
    seg = M.Segment(segp, dev)
    rng = np.random.default_rng(0)
    sample = np.sort(rng.choice(nb, 24, replace=False))
    host_blocks = pax.cpu().numpy()
    for b in sample:
        rows = ora.synth_docs(42, 64, dims, row0=int(b) * 64)
        exp = ora.encode_block(rows, ts=np.arange(b * 64, b * 64 + 64), src=np.full(64, 8), eden_mean=mean)
        assert np.array_equal(host_blocks[b * 4096:(b + 1) * 4096], exp)
    del x
    q, _ = ora.synth_queries(42, n, 7, 1, dims)
    gp = M.QueryPlan.from_query_eden(q[0], dims, fit(mean), dev=dev)
    op = ora.plan_build(q[0], eden_mean=mean)
    res = {}
    for mode in (M.ScanMode.EXACT, M.ScanMode.FAST):
        cfg = M.ScanConfig(shortlist_cand=k, mode=mode)
        sc, act, _ = M.vector_scores(seg, gp, cfg)
        hits = M.scan_blocks(seg, gp, cfg)
        gi = np.array([h.id.block * 64 + h.id.slot for h in hits])
        gs = np.array([h.score for h in hits], np.float32)
        res[mode] = (gi, gs, sc)
        if mode == M.ScanMode.EXACT:
            order = np.lexsort((np.arange(sc.size), -sc.astype(np.float64)))
            order = order[act[order] == 1][:k]
            assert np.array_equal(gi, order) and np.array_equal(gs.view(np.uint32), sc[order].view(np.uint32))
            sub = np.concatenate([host_blocks[b * 4096:(b + 1) * 4096] for b in sample])
            rs, ra = ora.full_scores(sub, op, ora.scan_cfg(k=k))
            idx = np.concatenate([np.arange(b * 64, b * 64 + 64) for b in sample])
            assert np.array_equal(sc[idx][ra == 1].view(np.uint32), rs[ra == 1].view(np.uint32))
    ei, es, esc = res[M.ScanMode.EXACT]
    fi, fs, fsc = res[M.ScanMode.FAST]
    np.testing.assert_allclose(fsc, esc, rtol=RTOL, atol=ATOL)             # per-slot fast scores
    assert np.array_equal(fi, ei) and np.array_equal(fs.view(np.uint32), es.view(np.uint32))
    # the reference's scan (oracle scan_blocks, Rayon sharding rules) over the same 1M corpus
    threads = os.cpu_count() or 4
    qs, _ = ora.synth_queries(42, n, 11, 4, dims)
    for qv in qs:
        op = ora.plan_build(qv, eden_mean=mean)
        rid, rsc = ora.scan_blocks(host_blocks, op, ora.scan_cfg(k=k), threads=threads)
        gp_q = M.QueryPlan.from_query_eden(qv, dims, fit(mean), dev=dev)
        for mode in (M.ScanMode.EXACT, M.ScanMode.FAST):
            hits = M.scan_blocks(seg, gp_q, M.ScanConfig(shortlist_cand=k, mode=mode))
            gi = [h.id.as_u64() for h in hits]
            gs = np.array([h.score for h in hits], np.float32)
            assert gi == [int(i) for i in rid], mode
            assert np.array_equal(gs.view(np.uint32), rsc.view(np.uint32)), mode
        gp_q.free()


def test_query_scan_host_staging_regrows(ora, dev, corpus768):
    """mrl_query_scan's pinned, device-mapped staging (query in, results stored by the scan) across
    calls whose sizes grow and shrink: one query, then the whole set, then a shortlist of 4,096,
    then one query again; each call equals the plan + scan path, and a non-finite query is refused
    before anything is staged."""
    M = mb()
    qs = corpus768["qs"]
    kw = dict(prefix_codec=M.PrefixCodec.EDEN_PROD, eden=fit(corpus768["mean"]))
    seg = M.Segment.upload(corpus768["eden"], dev)
    ref = M.QueryPlan.from_queries(qs, dev=dev, **kw)
    for n, k in ((1, 16), (len(qs), 256), (1, 4096), (1, 16)):
        cfg = M.ScanConfig(shortlist_cand=k)
        ids, sc, cnt, plans = M.query_scan(seg, qs[:n], cfg, **kw)
        r_ids, r_sc, r_cnt = M.scan_blocks_batch(seg, ref, cfg)
        assert np.array_equal(cnt, r_cnt[:n])
        for qi in range(n):
            m = int(cnt[qi])
            assert np.array_equal(ids[qi, :m], r_ids[qi, :m])
            assert np.array_equal(sc[qi, :m].view(np.uint32), r_sc[qi, :m].view(np.uint32))
        plans.free()
    bad = qs[:1].copy()
    bad[0, 5] = np.nan
    with pytest.raises(M.MrlError, match="non-finite"):
        M.query_scan(seg, bad, M.ScanConfig(shortlist_cand=16), **kw)
    ref.free()
    seg.free()


@pytest.mark.parametrize("mode", ["fast", "exact"])
def test_query_stream_pipelined_matches_device_scan(ora, dev, corpus768, mode):
    """mrl_query_submit / mrl_query_collect with three queries in flight and the slots reused: each
    result equals the plan + scan of the same query on the device path, bit for bit, and the first
    query equals the oracle's scan_blocks. Shortlists that shrink after a larger one keep working."""
    M = mb()
    seg = M.Segment.upload(corpus768["eden"], dev)
    mean = corpus768["mean"]
    qs = np.concatenate([corpus768["qs"]] * 3)[:11]
    kw = dict(prefix_codec=M.PrefixCodec.EDEN_PROD, mid_codec=M.MidCodec.RABITQ, eden=fit(mean))
    m = M.ScanMode.EXACT if mode == "exact" else M.ScanMode.FAST
    big = M.QueryStream(seg, M.ScanConfig(shortlist_cand=256, mode=m), **kw)
    big.submit(qs[0], 0)
    big.collect(0)  # the slots now hold room for 256 hits
    for k in (96, 16):
        cfg = M.ScanConfig(shortlist_cand=k, mode=m)
        ref_plans = M.QueryPlan.from_queries(qs, dev=dev, **kw)
        r_ids, r_sc, r_cnt = M.scan_blocks_batch(seg, ref_plans, cfg)
        st = M.QueryStream(seg, cfg, **kw)
        depth, slots = 3, 4
        got = {}
        for i in range(len(qs)):
            if i >= depth:
                got[i - depth] = st.collect((i - depth) % slots)
            st.submit(qs[i], i % slots)
        for j in range(len(qs) - depth, len(qs)):
            got[j] = st.collect(j % slots)
        for qi in range(len(qs)):
            ids, sc = got[qi]
            n = int(r_cnt[qi])
            assert len(ids) == n
            assert np.array_equal(ids, r_ids[qi, :n])
            assert np.array_equal(sc.view(np.uint32), r_sc[qi, :n].view(np.uint32))
        op = ora.plan_build(qs[0], eden_mean=mean)
        rid, rsc = ora.scan_blocks(corpus768["eden"], op, ora.scan_cfg(k=k))
        assert [int(x) for x in got[0][0]] == [int(x) for x in rid]
        assert np.array_equal(got[0][1].view(np.uint32), rsc.view(np.uint32))
        ref_plans.free()
    # misuse: a free slot, a busy slot, a non-finite query, dims beyond the launch's capacity
    with pytest.raises(M.MrlError):
        st.collect(0)
    st.submit(qs[0], 5)
    with pytest.raises(M.MrlError):
        st.submit(qs[1], 5)
    st.collect(5)
    bad = qs[0].copy()
    bad[3] = np.nan
    with pytest.raises(M.MrlError):
        st.submit(bad, 6)
    with pytest.raises(M.MrlError):
        st.submit(np.zeros(1040, np.float32), 6)
    with pytest.raises(M.MrlError):
        st.submit(qs[0], M.MAX_INFLIGHT)
    seg.free()


@pytest.mark.parametrize("ctas", [1, 16, 24, 74])
def test_fewer_ctas_per_query_same_results(ora, dev, corpus768, ctas):
    """mrl_set_scan_ctas: with fewer CTAs per launch (several queries then run side by side on the
    device), the results of the fused device path and of pipelined host queries are bit-identical
    to one CTA per SM, and every scratch set's control words end at zero."""
    import torch

    M = mb()
    seg = M.Segment.upload(corpus768["eden"], dev)
    mean = corpus768["mean"]
    qs = np.concatenate([corpus768["qs"]] * 3)[:9]
    kw = dict(prefix_codec=M.PrefixCodec.EDEN_PROD, mid_codec=M.MidCodec.RABITQ, eden=fit(mean))
    cfg = M.ScanConfig(shortlist_cand=128)
    r_ids, r_sc, r_cnt, r_plans = M.query_scan(seg, qs, cfg, **kw)
    try:
        dev.set_scan_ctas(ctas)
        ids, sc, cnt, plans = M.query_scan(seg, qs, cfg, **kw)  # several launches in flight
        assert np.array_equal(cnt, r_cnt)
        for qi in range(len(qs)):
            n = int(r_cnt[qi])
            assert np.array_equal(ids[qi, :n], r_ids[qi, :n])
            assert np.array_equal(sc[qi, :n].view(np.uint32), r_sc[qi, :n].view(np.uint32))
        st = M.QueryStream(seg, cfg, **kw)
        for i in range(len(qs)):
            st.submit(qs[i], i % M.MAX_INFLIGHT)
            if i >= 5:
                j = i - 5
                gi, gs = st.collect(j % M.MAX_INFLIGHT)
                assert np.array_equal(gi, r_ids[j, : int(r_cnt[j])])
        for j in range(len(qs) - 5, len(qs)):
            gi, gs = st.collect(j % M.MAX_INFLIGHT)
            assert np.array_equal(gs.view(np.uint32), r_sc[j, : int(r_cnt[j])].view(np.uint32))
        torch.cuda.synchronize()
        assert list(M.control_words(dev)) == [0] * 128
        plans.free()
    finally:
        dev.set_scan_ctas(0)
    op = ora.plan_build(qs[0], eden_mean=mean)
    rid, rsc = ora.scan_blocks(corpus768["eden"], op, ora.scan_cfg(k=128))
    assert [int(x) for x in r_ids[0, : int(r_cnt[0])]] == [int(x) for x in rid]
    r_plans.free()
    seg.free()
