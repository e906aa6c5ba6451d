"""Host side of the index directory (no GPU): manifest.json parsing with the reference's serde
names, the segment file writer, the id map rebuilt from tombstones, and the oracle's exact dot,
ring search and row rerank against direct restatements of the reference's loops."""
import json
import os

import numpy as np
import pytest


def M():
    import mrl_b200

    return mrl_b200


# A manifest as IndexEngine::write_manifest serialises it (serde_json pretty, src/engine.rs:218-233;
# EngineConfig fields in declaration order, src/config.rs:122-162).
REFERENCE_MANIFEST = """{
  "version": "3.5.0",
  "config": {
    "strata_depth": "l1_rabitq",
    "slab_residency": "ram_locked",
    "numa_sharding": false,
    "shortlist_cand": 256,
    "cs_tolerance": 0.9,
    "stratum4_weight": 0.3,
    "rabitq_confidence": 2.576,
    "jit_batch_size": 64,
    "io_read_workers": 4,
    "max_latency_budget_ms": 100,
    "ring_buffer_size": 2048,
    "tombstone_compact_ratio": 0.25,
    "temporal_filter_enable": false,
    "embed_dims": 768,
    "mrl_prefix": 64,
    "final_top_k": 10,
    "use_gemma2": true,
    "prefix_codec": "min_max4",
    "eden_seed": 7,
    "mid_codec": "eden_b1"
  },
  "next_passage_id": 130,
  "blocks_written": 2
}"""


def test_manifest_config_parses_reference_names():
    m = M()
    d = json.loads(REFERENCE_MANIFEST)
    cfg = m.config_from_json(d["config"])
    assert cfg.strata_depth == m.StrataDepth.L1_RABITQ
    assert cfg.prefix_codec == m.PrefixCodec.MIN_MAX4 and cfg.mid_codec == m.MidCodec.EDEN_B1
    assert cfg.shortlist_cand == 256 and cfg.embed_dims == 768 and cfg.eden_seed == 7
    assert cfg.numa_sharding is False and cfg.temporal_filter_enable is False
    assert abs(cfg.cs_tolerance - 0.9) < 1e-12 and abs(cfg.stratum4_weight - 0.3) < 1e-12
    assert cfg.ring_buffer_size == 2048
    out = m.config_to_json(cfg, d["config"])
    assert out == d["config"]  # unmodelled fields carried through, modelled ones re-serialised


def test_manifest_defaults_and_errors():
    m = M()
    cfg = m.config_from_json({"embed_dims": 384})  # serde(default) fields absent
    assert cfg.prefix_codec == m.PrefixCodec.EDEN_PROD and cfg.mid_codec == m.MidCodec.RABITQ
    assert cfg.eden_seed == 1 and cfg.strata_depth == m.StrataDepth.FULL_64B
    with pytest.raises(ValueError, match="unknown variant"):
        m.config_from_json({"strata_depth": "Full64b"})  # serde names are snake_case
    full = m.config_to_json(m.EngineConfig())
    for key in ("slab_residency", "rabitq_confidence", "jit_batch_size", "io_read_workers",
                "max_latency_budget_ms", "tombstone_compact_ratio", "use_gemma2", "strata_depth"):
        assert key in full  # every EngineConfig field, so the reference can read it back
    assert full["strata_depth"] == "full64b" and full["prefix_codec"] == "eden_prod"


def test_segment_writer_and_corrupt_size(tmp_path):
    m = M()
    p = str(tmp_path / "segments" / "000001.pax")
    w = m.SegmentWriter.create(p)
    blocks = np.random.default_rng(0).integers(0, 256, (3, 4096), dtype=np.uint8)
    assert [w.append_block(b) for b in blocks] == [0, 1, 2]
    w.close()
    assert np.array_equal(np.fromfile(p, np.uint8), blocks.reshape(-1))
    w = m.SegmentWriter.open_append(p)
    assert w.block_count() == 3
    w.append_block(blocks[0])
    w.close()
    assert os.path.getsize(p) == 4 * 4096
    with open(p, "ab") as f:
        f.write(b"x" * 10)
    with pytest.raises(m.SegmentError, match=r"corrupt segment size 16394 \(not multiple of 4096\)"):
        m.SegmentWriter.open_append(p)


def test_id_map_from_tombstones(ora):
    m = M()
    rng = np.random.default_rng(1)
    full = rng.standard_normal((64, 384)).astype(np.float32)
    part = rng.standard_normal((10, 384)).astype(np.float32)
    pages = np.concatenate([ora.encode_block(full, prefix_codec=ora.MINMAX4),
                            ora.encode_block(part, prefix_codec=ora.MINMAX4),
                            ora.encode_block(full[:64], prefix_codec=ora.MINMAX4)])
    id_map, nxt = m.id_map_from_pages(pages)
    assert nxt == 64 + 10 + 64
    mx = np.iinfo(np.uint64).max
    assert np.array_equal(id_map[:64], np.arange(64))
    assert np.array_equal(id_map[64:74], np.arange(64, 74)) and np.all(id_map[74:128] == mx)
    assert np.array_equal(id_map[128:], np.arange(74, 138))


def _dot_ref(a, b):
    """dot (src/embed.rs:115-152) restated as plain Python f32 loops."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    if a.size == 768:
        acc = [np.float32(0.0)] * 8
        for i in range(0, 768, 8):
            for j in range(8):
                acc[j] = np.float32(acc[j] + np.float32(a[i + j] * b[i + j]))
        r = acc[0]
        for j in range(1, 8):
            r = np.float32(r + acc[j])
        return r
    s = np.float32(-0.0)  # Rust's f32 Sum starts from -0.0
    for x, y in zip(a, b):
        s = np.float32(s + np.float32(x * y))
    return s


@pytest.mark.parametrize("dims", [768, 384, 100, 1])
def test_oracle_dot_order(ora, dims):
    rng = np.random.default_rng(dims)
    for _ in range(3):
        a = rng.standard_normal(dims).astype(np.float32)
        b = rng.standard_normal(dims).astype(np.float32)
        assert ora.dot(a, b).view(np.uint32) == _dot_ref(a, b).view(np.uint32)
    z = ora.dot(np.zeros(dims, np.float32), -np.ones(dims, np.float32))
    assert np.signbit(z) == (dims != 768)  # -0.0 neutral element, 0.0 accumulators at 768


def test_oracle_ring_search_and_rerank(ora):
    rng = np.random.default_rng(5)
    pend = rng.standard_normal((40, 384)).astype(np.float32)
    pend[7] = pend[3]  # a tie: equal scores keep push order (stable sort)
    q = rng.standard_normal(384).astype(np.float32)
    pos, sc = ora.ring_search(pend, q, 10)
    ref = sorted([(_dot_ref(p, q), i) for i, p in enumerate(pend)], key=lambda t: -t[0])[:10]
    assert list(pos) == [i for _, i in ref]
    assert np.array_equal(sc.view(np.uint32), np.array([s for s, _ in ref], np.float32).view(np.uint32))
    cand = np.array([3, 7, 0, 39, 3], np.uint64)
    rows, rs = ora.rerank_rows(pend, q, cand)
    ref = sorted([(_dot_ref(q, pend[c]), int(c)) for c in cand], key=lambda t: -t[0])
    assert list(rows) == [c for _, c in ref]
    assert np.array_equal(rs.view(np.uint32), np.array([s for s, _ in ref], np.float32).view(np.uint32))
    pos, sc = ora.ring_search(np.zeros((0, 384), np.float32), q, 5)
    assert pos.size == 0
