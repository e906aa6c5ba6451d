"""The fixed-point restatement (the product's fast mode) against the reference f32 arithmetic.

The fast mode replaces each stage's sequential f32 loop by an exact int32 sum of table entries
(2^shift-scaled, round-to-nearest-even products computed in double). These CPU tests pin the
formulation itself: integer sums reproduced independently in numpy, and full scores within the
north-star tolerance of 1e-5 relative of the reference's f32 scores.
"""
import numpy as np
import pytest

RTOL = 1e-5  # f32 scores within 1e-5 relative
ATOL = 1e-6


@pytest.fixture(scope="module")
def corpus(ora):
    docs = ora.synth_docs(21, 64 * 40, 768)
    mean = ora.eden_fit_prefix(docs)
    return docs, mean


def _levels(blocks, nb):
    """Per-slot 4-bit levels, 128 mid bits and 64 tail bits from PaxBlock64 pages (numpy)."""
    b = blocks.reshape(nb, 4096)
    pl = lambda off, n: b[:, off:off + 8 * n].view(np.uint64).reshape(nb, n)  # noqa: E731
    s0, s1, s2, s3, s4, s5 = pl(512, 64), pl(1024, 128), pl(2048, 64), pl(2560, 64), pl(3072, 64), pl(3584, 64)
    v = np.arange(64, dtype=np.uint64)
    bit = lambda w: ((w[:, :, None] >> v[None, None, :]) & np.uint64(1)).astype(np.int64)  # [nb, d, v]  # noqa: E731
    lv = bit(s5) | (bit(s3) << 1) | (bit(s2) << 2) | (bit(s0) << 3)
    return lv, bit(s1), bit(s4)


@pytest.mark.parametrize("codec", ["eden", "minmax"])
@pytest.mark.parametrize("depth", [0, 1, 2])
def test_fixed_scores_close_to_reference(ora, corpus, codec, depth):
    docs, mean = corpus
    pc = ora.EDEN_PROD if codec == "eden" else ora.MINMAX4
    blocks = ora.encode_corpus(docs, prefix_codec=pc, eden_mean=mean)
    qs, _ = ora.synth_queries(21, docs.shape[0], 5, 4, 768)
    cfg = ora.scan_cfg(k=64, strata_depth=depth)
    for q in qs:
        p = ora.plan_build(q, prefix_codec=pc, eden_mean=mean)
        fp = ora.fixed_plan_build(p, cfg)
        parts, fsc, fact = ora.fixed_scores(blocks, p, fp, cfg)
        rsc, ract = ora.full_scores(blocks, p, cfg)
        assert np.array_equal(fact, ract)
        a = fact == 1
        np.testing.assert_allclose(fsc[a], rsc[a], rtol=RTOL, atol=ATOL)
        # the exact top-64 by fixed-point score equals the reference top-64 up to near-ties
        ti, ts = ora.topk_by_key(fsc, fact, 64)
        ri, rs = ora.topk_by_key(rsc, ract, 64)
        kth = rs[-1]
        diff = set(ti.tolist()) ^ set(ri.tolist())
        for vid in diff:
            o = (int(vid) >> 16) * 64 + (int(vid) & 0xFFFF)
            assert abs(rsc[o] - kth) <= RTOL * abs(kth) + ATOL


def test_fixed_integer_sums_reproduced_in_numpy(ora, corpus):
    docs, mean = corpus
    blocks = ora.encode_corpus(docs[: 64 * 4], eden_mean=mean)
    q, _ = ora.synth_queries(21, docs.shape[0], 9, 1, 768)
    p = ora.plan_build(q[0], eden_mean=mean)
    cfg = ora.scan_cfg(k=16)
    fp = ora.fixed_plan_build(p, cfg)
    parts, _, act = ora.fixed_scores(blocks, p, fp, cfg)
    lv, s1, s4 = _levels(blocks, 4)
    lut_p = np.array(fp.prefix_lut, np.int64)  # [64,16]
    P = lut_p[np.arange(64)[None, :, None], lv].sum(axis=1)  # [nb, v]
    s1lut = np.array(fp.s1_lut, np.int64)
    S1 = np.zeros((4, 64), np.int64)
    for g in range(26):
        m = np.zeros((4, 64), np.int64)
        for i in range(min(5, 128 - 5 * g)):
            m |= s1[:, 5 * g + i, :] << i
        S1 += s1lut[g][m]
    s4lut = np.array(fp.s4_lut, np.int64)
    S4 = np.zeros((4, 64), np.int64)
    for g in range(13):
        m = np.zeros((4, 64), np.int64)
        for i in range(min(5, 64 - 5 * g)):
            m |= s4[:, 5 * g + i, :] << i
        S4 += s4lut[g][m]
    a = act.reshape(4, 64) == 1
    got = parts.reshape(4, 64, 3)
    assert np.array_equal(got[..., 0][a], P[a])
    assert np.array_equal(got[..., 1][a], S1[a])
    assert np.array_equal(got[..., 2][a], S4[a])
    # every table fits the int32 headroom argument: |sum| < 2^30 + 64 per stage
    assert np.abs(P).max() < 2 ** 30 + 64 and np.abs(S1).max() < 2 ** 30 + 64


def test_fixed_shift_tracks_query_scale(ora, corpus):
    """Scaling the query by 2^k shifts every stage's table scale by -k (scores scale with it)."""
    docs, mean = corpus
    q, _ = ora.synth_queries(21, docs.shape[0], 9, 1, 768)
    cfg = ora.scan_cfg(k=16)
    base = ora.fixed_plan_build(ora.plan_build(q[0], prefix_codec=ora.MINMAX4), cfg)
    big = ora.fixed_plan_build(ora.plan_build(q[0] * np.float32(1024.0), prefix_codec=ora.MINMAX4), cfg)
    assert big.prefix_shift == base.prefix_shift - 10
    assert big.s1_shift == base.s1_shift - 10 and big.s4_shift == base.s4_shift - 10
    assert np.array_equal(np.array(big.prefix_lut), np.array(base.prefix_lut))
