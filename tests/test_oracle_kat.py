"""The CPU oracle against the reference's own known-answer tests, the golden fixtures of the
independent numpy restatement, and the reference's property tests (ported).

Reference tests ported (paths relative to the reference project root):
  src/eden.rs:374-424, src/rotate.rs:204-235, src/quantize.rs:375-427, src/scan.rs:925-1037,
  src/geometry.rs:123-129, src/encoder.rs:284-323, src/pipeline.rs:204-243,
  tests/test_challenger_architecture.rs:27-322, tests/test_operator_folding.rs:53-93.
"""
import hashlib
import struct
import zlib

import numpy as np
import pytest

F = np.float32


def l2n(v):
    v = np.asarray(v, np.float32)
    n = np.float32(0)
    for x in v:
        n = np.float32(n + np.float32(x * x))
    n = max(np.sqrt(n), np.float32(1e-12))
    return (v / n).astype(np.float32)


def synth_block_rows(seed, n, dims):
    """`synth_block` fixture of src/scan.rs:901-922 (LCG-like integer hash, L2-normalised)."""
    rows = []
    for i in range(n):
        v = np.zeros(dims, np.float32)
        for d in range(dims):
            x = ((seed * 1103515245 + 12345 + i * 9973 + d * 7919) & 0xFFFFFFFF) % 10007
            v[d] = np.float32(np.float32(x) / np.float32(5003.5) - np.float32(1.0))
        rows.append(l2n(v))
    return np.array(rows, np.float32)


# ---- known-answer values ------------------------------------------------------------------

def test_lloyd_tables_match_reference_and_are_sorted_symmetric(ora, golden):
    b4 = ora.lloyd_max(4)
    assert np.array_equal(b4, golden["kat_lloyd_b4"])
    assert np.array_equal(ora.lloyd_max(1), golden["kat_lloyd_b1"])
    assert np.all(np.diff(b4) > 0)
    assert np.all(np.abs(b4 + b4[::-1]) < 1e-5)  # src/eden.rs:374-381


def test_crc32_check_value_and_zlib(ora, golden):
    assert ora.crc32(b"123456789") == int(golden["kat_crc_check"][0]) == 0xCBF43926
    rng = np.random.default_rng(3)
    for n in (0, 1, 7, 4096, 10000):
        data = rng.integers(0, 256, n, dtype=np.uint8)
        assert ora.crc32(data) == zlib.crc32(data.tobytes())


def test_f16_round_to_nearest_even(ora):
    rng = np.random.default_rng(5)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(3.0),
        rng.standard_normal(2000).astype(np.float32) * np.float32(1e-5),   # subnormal halves
        np.array([0.0, -0.0, 65504.0, 65520.0, 1e9, -1e9, 6.0e-8, 2.9e-8, 3.0e-8, 1.0 + 2 ** -11,
                  1.0 + 3 * 2 ** -11], np.float32),
    ])
    ours = np.array([ora.f32_to_f16(v) for v in vals], np.uint16)
    with np.errstate(over="ignore"):
        ref = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, ref)
    back = np.array([ora.f16_to_f32(h) for h in ref], np.float32)
    assert np.array_equal(back.view(np.uint32), ref.view(np.float16).astype(np.float32).view(np.uint32))


def test_paxblock_field_offsets(ora, golden):
    """tests/test_challenger_architecture.rs:263-322 — header 0, meta 64 (64 x 7 B), S0 512,
    S1 1024, S2 2048, S3 2560, S4 3072, S5 3584, total 4096."""
    offs = golden["kat_offsets"]
    assert list(offs) == [0, 64, 512, 1024, 2048, 2560, 3072, 3584, 4096]
    # One slot with known prefix levels lands its bits at those offsets.
    v = np.zeros(256, np.float32)
    v[:64] = np.linspace(-1, 1, 64, dtype=np.float32)
    v[64:] = 0.1
    blk = ora.encode_block(v[None, :], ts=[42], src=[4], prefix_codec=ora.MINMAX4)
    tomb = struct.unpack_from("<Q", blk, 16)[0]
    assert tomb == ~1 & 0xFFFFFFFFFFFFFFFF
    assert struct.unpack_from("<III", blk, 0) == (42, 42, 4)
    levels = []
    for d in range(64):
        q = 0
        for off, bit in ((512, 8), (2048, 4), (2560, 2), (3584, 1)):
            if struct.unpack_from("<Q", blk, off + 8 * d)[0] & 1:
                q |= bit
        levels.append(q)
    assert levels[0] == 0 and levels[-1] == 15 and levels == sorted(levels)


def test_ballot_word_order_matches_u64_planes(ora):
    """tests/test_challenger_architecture.rs:27-187: u32 word d*2+sg with sg 0 = slots 0..31 is
    the little-endian u64 plane word; checked on an oracle-encoded block."""
    rng = np.random.default_rng(9)
    rows = np.array([l2n(r) for r in rng.standard_normal((64, 384)).astype(np.float32)])
    blk = ora.encode_block(rows, prefix_codec=ora.MINMAX4)
    s1 = blk[1024:2048].view(np.uint32)
    signs =np.array([ora.rotate_mid_band(np.ascontiguousarray(r[64:192])) >= 0 for r in rows])  # [64,128]
    for d in range(128):
        lo = sum(1 << v for v in range(32) if signs[v, d])
        hi = sum(1 << (v - 32) for v in range(32, 64) if signs[v, d])
        assert s1[2 * d] == lo and s1[2 * d + 1] == hi


def test_fwht_preserves_l2(ora):
    """src/rotate.rs:204-211"""
    v = np.array([((i * 17) % 97) * 0.01 - 0.5 for i in range(128)], np.float32)
    n0 = np.linalg.norm(v)
    n1 = np.linalg.norm(ora.fwht(v))
    assert abs(n0 - n1) < 1e-4


def test_fwht_spreads_a_spike(ora):
    """src/rotate.rs:213-220"""
    mid = np.zeros(128, np.float32)
    mid[0] = 1
    assert np.any(np.abs(ora.rotate_mid_band(mid)[1:]) > 1e-6)


def test_fold_tail_768_is_nontrivial(ora):
    """src/rotate.rs:222-235"""
    v = np.array([((i * 3) % 17) * 0.01 - 0.08 if i >= 192 else 0.0 for i in range(768)], np.float32)
    rot = ora.rotate_tail_fold(v)
    assert np.sum(rot * rot) > 1e-6


def test_operator_t_reproduces_pipeline_functions(ora):
    """tests/test_operator_folding.rs:53-93: T built from basis vectors reproduces the pipeline
    rotations within 1e-6 (relative to max(1, |value|): the inputs here come from numpy's RNG
    rather than the reference's ChaCha stream, and reach magnitudes where 1e-6 is ~2 ulp)."""
    T = np.zeros((256, 768))
    for i in range(64):
        T[i, i] = 1
    for j in range(128):
        e = np.zeros(128, np.float32)
        e[j] = 1
        T[64:192, 64 + j] = ora.rotate_mid_band(e)
    for j in range(192, 768):
        e = np.zeros(768, np.float32)
        e[j] = 1
        T[192:256, j] = ora.rotate_tail_fold(e)
    rng = np.random.default_rng(42)
    for _ in range(20):
        z = rng.uniform(-2, 2, 768).astype(np.float32)
        exp = np.concatenate([z[:64], ora.rotate_mid_band(z[64:192]), ora.rotate_tail_fold(z)])
        act = (T @ z.astype(np.float64)).astype(np.float32)
        assert np.max(np.abs(act - exp) / np.maximum(1.0, np.abs(exp))) < 1e-6


def test_geometry_fold_blocks(ora):
    """src/geometry.rs:113-129: B = 9 at 768 dims, 3 at 384 (only the first B*64 tail dims fold)."""
    v = np.zeros(768, np.float32)
    v[192 + 9 * 64 - 1] = 1.0
    assert np.any(ora.rotate_tail_fold(v) != 0)
    v384 = np.zeros(384, np.float32)
    v384[383] = 1.0
    assert np.any(ora.rotate_tail_fold(v384) != 0)
    v400 = np.zeros(400, np.float32)
    v400[399] = 1.0  # dims 384..399 are beyond the 3 whole fold blocks
    assert np.all(ora.rotate_tail_fold(v400) == 0)


# ---- golden fixtures of the independent numpy restatement ---------------------------------

@pytest.mark.parametrize("tag,dims,n,nq", [("d768", 768, 130, 3), ("d384", 384, 70, 2)])
def test_oracle_matches_golden(ora, golden, tag, dims, n, nq):
    docs = ora.synth_docs(42, n, dims)
    assert hashlib.sha256(docs.tobytes()).digest() == bytes(golden[f"{tag}_docs_sha256"])
    mean = ora.eden_fit_prefix(docs)
    assert np.array_equal(mean, golden[f"{tag}_eden_mean"])
    q, pick = ora.synth_queries(42, n, 7, nq, dims)
    assert np.array_equal(q, golden[f"{tag}_queries"]) and np.array_equal(pick, golden[f"{tag}_picks"])
    for codec, cname in ((ora.EDEN_PROD, "eden"), (ora.MINMAX4, "minmax")):
        blocks = ora.encode_corpus(docs, prefix_codec=codec, eden_mean=mean)
        assert np.array_equal(blocks, golden[f"{tag}_{cname}_blocks"])
        for qi in range(nq):
            p = ora.plan_build(q[qi], prefix_codec=codec, eden_mean=mean)
            pre = f"{tag}_{cname}_q{qi}"
            assert np.array_equal(np.array(p.eden_q_rot), golden[pre + "_eden_q_rot"])
            assert np.array_equal(np.array(p.rabitq_q), golden[pre + "_rabitq_q"])
            assert np.array_equal(np.array(p.rabitq_weights2), golden[pre + "_w2"])
            assert np.array_equal(np.array(p.tail_fold_q), golden[pre + "_tfq"])
            assert np.array_equal(np.array(p.tail_fold_weights2), golden[pre + "_tw2"])
            sc = np.array([p.rabitq_base, p.tail_fold_base, p.s4_abs_budget, p.q_tail_norm, p.q_mid_norm,
                           p.q_after_prefix, p.prefix_sum, p.eden_mean_ip], np.float32)
            assert np.array_equal(sc, golden[pre + "_scalars"])
            for depth in (0, 1, 2):
                fs, act = ora.full_scores(blocks, p, ora.scan_cfg(k=16, strata_depth=depth))
                assert np.array_equal(act, golden[pre + f"_d{depth}_active"])
                assert np.array_equal(fs[act == 1].view(np.uint32),
                                      golden[pre + f"_d{depth}_scores"][act == 1].view(np.uint32))


# ---- reference property tests, ported onto the oracle -------------------------------------

def test_encode_roundtrip_bits_and_crc(ora):
    """src/quantize.rs:375-398"""
    v = np.array([((i * 0.07) % 2.0) - 1.0 for i in range(256)], np.float32)
    blk = ora.encode_block(v[None, :], ts=[42], src=[4], prefix_codec=ora.MINMAX4)
    assert ora.verify_crc(blk)
    assert struct.unpack_from("<I", blk, 0)[0] == 42
    tomb = struct.unpack_from("<Q", blk, 16)[0]
    assert bin(~tomb & (2 ** 64 - 1)).count("1") == 1 and (tomb >> 1) & 1
    scale = ora.f16_to_f32(struct.unpack_from("<H", blk, 64)[0])
    offset = ora.f16_to_f32(struct.unpack_from("<H", blk, 66)[0])
    err = 0.0
    for d in range(64):
        q = 0
        for off, bit in ((512, 8), (2048, 4), (2560, 2), (3584, 1)):
            if struct.unpack_from("<Q", blk, off + 8 * d)[0] & 1:
                q |= bit
        err += abs(q * scale + offset - v[d])
    assert err / 64 < 0.2
    bad = blk.copy()
    bad[700] ^= 1
    assert not ora.verify_crc(bad)


def test_encode_768_packs_rho_and_stratum4(ora):
    """src/quantize.rs:401-427"""
    v = l2n([((i * 0.013) % 2.0) - 1.0 for i in range(768)])
    blk = ora.encode_block(v[None, :], ts=[1], src=[8], prefix_codec=ora.MINMAX4)
    tail = ora.f16_to_f32(struct.unpack_from("<H", blk, 68)[0])
    flags = blk[70]
    assert flags > 0
    rho = np.float32(flags) / np.float32(255)
    mid = np.sqrt(max(1 - rho * rho, 0)) * tail
    high = rho * tail
    assert abs(mid * mid + high * high - tail * tail) < 1e-3
    ones = sum((struct.unpack_from("<Q", blk, 3072 + 8 * d)[0] & 1) for d in range(64))
    assert 5 < ones < 60


def test_eden_unbiased_slope_near_one(ora):
    """src/eden.rs:384-424"""
    rows = []
    for n in range(128):
        v = np.zeros(64, np.float32)
        for i in range(64):
            x = ((n * 0x9E37 + i) * 0xBF58) & 0xFFFFFFFFFFFFFFFF
            x ^= x >> 17
            xi = x - (1 << 64) if x >= (1 << 63) else x
            v[i] = np.float32(np.float32(xi) / np.float32(2 ** 64 - 1)) * np.float32(2.0) - np.float32(1.0)
        rows.append(v / max(np.linalg.norm(v), 1e-6))
    rows = np.array(rows, np.float32)
    mean = ora.eden_fit_prefix(rows)
    q = rows[0]
    import ctypes as C
    lv = np.zeros(64, np.uint8)
    num = den = 0.0
    cb = ora.lloyd_max(4)
    rot = np.array(q, np.float32)
    rot = np.array([rot[i] * ora.lib().ora_rademacher_diag(1, i) for i in range(64)], np.float32)
    rot = ora.fwht(rot)
    mean_ip = float(np.dot(q, mean))
    for r in rows:
        cn, ss = C.c_float(), C.c_float()
        ora.lib().ora_eden_encode_slice(mean, 64, 1, 4, np.ascontiguousarray(r), lv, C.byref(cn), C.byref(ss))
        dot_cw = float(np.sum(rot * cb[lv] / 8.0))
        est = mean_ip + cn.value * ss.value * dot_cw
        exact = float(np.dot(q, r))
        num += est * exact
        den += exact * exact
    assert abs(num / den - 1.0) < 0.35


def test_default_kernel_stages_narrow_monotonically(ora):
    """src/scan.rs:925-957 (MinMax plan on the synth_block fixture)."""
    rows = synth_block_rows(42, 64, 768)
    blk = ora.encode_block(rows, ts=np.arange(64), src=np.ones(64), prefix_codec=ora.MINMAX4)
    plan = ora.plan_build(rows[0], prefix_codec=ora.MINMAX4)
    masks, _ = ora.block_stages(blk, plan, ora.scan_cfg(k=64), -1.0)
    after_prefix = bin(int(masks[0])).count("1")
    assert after_prefix > 0
    assert bin(int(masks[1])).count("1") <= after_prefix
    assert int(masks[2]) & ~int(masks[1]) == 0
    assert bin(int(masks[3])).count("1") > 0


def test_scan_blocks_deterministic_and_stats_consistent(ora):
    """src/scan.rs:960-993"""
    rows = synth_block_rows(7, 32, 768)
    blk = ora.encode_block(rows, ts=np.arange(32), src=np.ones(32), prefix_codec=ora.MINMAX4)
    plan = ora.plan_build(rows[3], prefix_codec=ora.MINMAX4)
    cfg = ora.scan_cfg(k=16, numa_sharding=False, temporal_filter_enable=True)
    a = ora.scan_blocks(blk, plan, cfg)
    b = ora.scan_blocks(blk, plan, cfg)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
    ids, sc, st = ora.scan_blocks(blk, plan, cfg, stats=True)
    assert np.array_equal(ids, a[0]) and np.array_equal(sc.view(np.uint32), a[1].view(np.uint32))
    assert st.blocks == 1 and st.active_vecs >= 32
    assert st.after_prefix <= st.active_vecs and st.after_s1 <= st.after_prefix
    assert st.after_s4_budget <= st.after_s1 and st.pushed <= st.after_s4_budget
    assert len(ids) <= 16 and len(ids) <= st.pushed


def test_s4_abs_budget_positive_for_768d_query(ora):
    """src/scan.rs:996-1008"""
    q = l2n([((i * 17) % 101) * 0.01 - 0.5 for i in range(768)])
    p = ora.plan_build(q, prefix_codec=ora.MINMAX4)
    assert p.has_tail_fold and p.s4_abs_budget > 0 and p.q_mid_norm > 0 and p.q_tail_norm > 0
    assert p.q_after_s1 == p.q_tail_norm


def test_strata_depth_gates_s4_scores(ora):
    """src/scan.rs:1011-1037"""
    rows = synth_block_rows(99, 64, 768)
    blk = ora.encode_block(rows, ts=np.arange(64), src=np.ones(64), prefix_codec=ora.MINMAX4)
    plan = ora.plan_build(rows[0], prefix_codec=ora.MINMAX4)
    full = ora.scan_blocks(blk, plan, ora.scan_cfg(k=64, strata_depth=ora.FULL_64B, numa_sharding=False))
    l1 = ora.scan_blocks(blk, plan, ora.scan_cfg(k=64, strata_depth=ora.L1_RABITQ, numa_sharding=False))
    assert len(full[0]) and len(full[0]) == len(l1[0])
    assert not np.array_equal(full[1].view(np.uint32), l1[1].view(np.uint32))


def test_encoder_parallel_equals_serial(ora):
    """src/encoder.rs:303-323 (130 rows -> 3 blocks)"""
    m = np.array([((i * 17) % 101) * 0.01 - 0.5 for i in range(130 * 384)], np.float32).reshape(130, 384)
    m = np.array([l2n(r) for r in m])
    par = ora.encode_corpus(m, prefix_codec=ora.MINMAX4, threads=4)
    ser = ora.encode_corpus(m, prefix_codec=ora.MINMAX4, threads=1)
    assert par.size == 3 * 4096 and np.array_equal(par, ser)


def test_threaded_scan_equals_serial_and_exact_topk(ora):
    """Under the exactness condition (cs_tolerance >= 1, default w_s4) the sharded scan, the
    serial scan and the exact top-k by full score agree (ties aside; none occur here)."""
    docs = ora.synth_docs(11, 64 * 80, 768)
    mean = ora.eden_fit_prefix(docs)
    blocks = ora.encode_corpus(docs, eden_mean=mean)
    qs, _ = ora.synth_queries(11, 64 * 80, 3, 3, 768)
    for q in qs:
        p = ora.plan_build(q, eden_mean=mean)
        for alpha in (1.0, 1.2):
            cfg = ora.scan_cfg(k=64, cs_tolerance=alpha)
            par = ora.scan_blocks(blocks, p, cfg, threads=4)
            ser = ora.scan_blocks(blocks, p, ora.scan_cfg(k=64, cs_tolerance=alpha, numa_sharding=False))
            fs, act = ora.full_scores(blocks, p, cfg)
            top = ora.topk_by_key(fs, act, 64)
            assert np.array_equal(par[0], ser[0]) and np.array_equal(par[0], top[0])
            assert np.array_equal(par[1].view(np.uint32), top[1].view(np.uint32))


def test_scan_order_dependence_outside_exactness_region(ora):
    """Why the device scans refuse cs_tolerance < 1 with the folded-tail stage: near-duplicate
    vectors whose folded-tail bits all agree with the query (|s4| equal to the S4 budget) are pruned
    by the budget bound alpha * budget < |s4| (src/scan.rs:587-607) depending on the shortlist's
    running threshold, so the same vectors stored in the reverse block order give a different
    top-k, and neither equals the top-k by full score. At cs_tolerance 1 every order gives that
    top-k."""
    rng = np.random.default_rng(5)
    q = ora.synth_docs(21, 1, 768)[0]
    n = 64 * 40
    docs = np.repeat(q[None, :], n, axis=0).astype(np.float64)
    docs[:, :192] += rng.standard_normal((n, 192)) * 0.02  # the tail keeps the query's direction
    docs = (docs / np.linalg.norm(docs, axis=1, keepdims=True)).astype(np.float32)
    mean = ora.eden_fit_prefix(docs)
    blocks = ora.encode_corpus(docs, eden_mean=mean)
    nb = n // 64
    rev = blocks.reshape(nb, 4096)[::-1].reshape(-1).copy()
    p = ora.plan_build(q, eden_mean=mean)

    def unrev(ids):
        return {((nb - 1 - (int(i) >> 16)) << 16) | (int(i) & 0xFFFF) for i in ids}

    for alpha, differs in ((1.0, False), (0.9, True)):
        cfg = ora.scan_cfg(k=64, cs_tolerance=alpha, numa_sharding=False)
        fwd = set(map(int, ora.scan_blocks(blocks, p, cfg)[0]))
        bwd = unrev(ora.scan_blocks(rev, p, cfg)[0])
        fs, act = ora.full_scores(blocks, p, cfg)
        top = set(map(int, ora.topk_by_key(fs, act, 64)[0]))
        assert (fwd != bwd) == differs and (fwd != top) == differs and (bwd != top) == differs, alpha


def test_temporal_filter_skips_blocks(ora):
    """src/scan.rs:719-730"""
    docs = ora.synth_docs(5, 64 * 3, 384)
    blocks = ora.encode_corpus(docs, prefix_codec=ora.MINMAX4)  # ts = row index
    p = ora.plan_build(docs[0], prefix_codec=ora.MINMAX4)
    cfg = ora.scan_cfg(k=256, temporal_filter_enable=True)
    ids, _ = ora.scan_blocks(blocks, p, cfg, time_lo=64, time_hi=127)
    assert len(ids) == 64 and all((int(i) >> 16) == 1 for i in ids)
    cfg_off = ora.scan_cfg(k=256, temporal_filter_enable=False)
    ids2, _ = ora.scan_blocks(blocks, p, cfg_off, time_lo=64, time_hi=127)
    assert len(ids2) == 192
