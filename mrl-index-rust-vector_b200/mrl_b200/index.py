"""The index directory and the engine's query-side state around the scan, on the device.

Mirrors of the reference crate (mrl_index 0.3.5):
  * `SegmentWriter` (src/segment.rs:21-79): the append-only segment file of 4096-byte pages;
  * `load_segment` (SegmentReader::open, src/segment.rs:88-162): the file straight into HBM through
    the library's pinned, double-buffered loader (mrl_segment_load);
  * `DeviceRing` (RingBuffer, src/ring.rs:49-119): pending embeddings mirrored in HBM, exact search
    on the device (mrl_ring_search), flush into an encoded page every 64 pushes;
  * `rerank_exact_rows` (QueryPipeline::rerank_exact_rows, src/pipeline.rs:157-169) on the device;
  * `IndexDir` (IndexEngine::{create, open}, src/engine.rs:79-194, and the scan half of
    query_filtered, :547-610): manifest.json, eden_prefix.json, segments/000001.pax, the slot ->
    passage id map, live appends, and the scan + ring merge of one query (mrl_engine_scan).
Passage text, embedders and the text rerank are not part of this package.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import json
import os
from typing import List, Optional, Sequence, Tuple

import numpy as np

from ._capi import check
from .api import (
    BLOCK_BYTES,
    VECTORS_PER_BLOCK,
    Device,
    EdenFit,
    EngineConfig,
    MidCodec,
    PrefixCodec,
    ScanMode,
    ScoredHit,
    Segment,
    StrataDepth,
    VectorId,
    _codec_desc,
    _time_ptrs,
    default_device,
    encode_blocks,
)
from .shard import record_bytes

SOURCE_DOC = 1 << 3  # block::source::DOC (src/block.rs:28)
RING_BLOCK = 0xFFFFFFFF  # VectorId.block of ring hits (src/engine.rs:588)
MANIFEST_VERSION = "3.5.0"  # IndexEngine::write_manifest (src/engine.rs:218-233)
EDEN_PREFIX_FILE = "eden_prefix.json"
SEGMENT_PATH = os.path.join("segments", "000001.pax")


class SegmentError(ValueError):
    """SegmentError::CorruptSize (src/segment.rs:13-19)."""


class SegmentWriter:
    """SegmentWriter (src/segment.rs:21-79): pages appended to one file."""

    def __init__(self, path: str, f, blocks: int):
        self.path = path
        self._f = f
        self.blocks = blocks

    @staticmethod
    def create(path: str) -> "SegmentWriter":
        d = os.path.dirname(path)
        if d:
            os.makedirs(d, exist_ok=True)
        return SegmentWriter(path, open(path, "w+b"), 0)

    @staticmethod
    def open_append(path: str) -> "SegmentWriter":
        f = open(path, "a+b")
        size = os.path.getsize(path)
        if size % BLOCK_BYTES:
            f.close()
            raise SegmentError(f"corrupt segment size {size} (not multiple of 4096)")
        return SegmentWriter(path, f, size // BLOCK_BYTES)

    def append_block(self, block) -> int:
        buf = np.ascontiguousarray(block, np.uint8).reshape(-1)
        if buf.size != BLOCK_BYTES:
            raise ValueError("a block is exactly 4096 bytes")
        idx = self.blocks
        self._f.write(buf.tobytes())
        self._f.flush()
        self.blocks += 1
        return idx

    def block_count(self) -> int:
        return self.blocks

    def close(self) -> None:
        if self._f:
            self._f.close()
            self._f = None


def load_segment(path: str, dev: Optional[Device] = None, block_id_base: int = 0) -> Segment:
    """SegmentReader::open into HBM. A missing file is an empty segment (src/segment.rs:90-97); a
    size that is not a multiple of 4096 raises the reference's CorruptSize message."""
    dev = dev or default_device()
    if not os.path.exists(path):
        return Segment.upload(np.zeros(0, np.uint8), dev, block_id_base)
    out = C.c_void_p()
    rc = dev.lib.mrl_segment_load(dev.ptr, os.fsencode(path), block_id_base, C.byref(out))
    if rc != 0:
        msg = dev.lib.mrl_last_error(dev.ptr).decode()
        if msg.startswith("corrupt segment size"):
            raise SegmentError(msg)
        check(dev.ptr, rc)
    return Segment(out, dev)


def tombstone_masks(pages: np.ndarray) -> np.ndarray:
    """BlockHeader::tombstone_mask (u64 at byte 16 of each page, src/block.rs:34-44)."""
    p = np.ascontiguousarray(pages, np.uint8).reshape(-1, BLOCK_BYTES)
    return p[:, 16:24].copy().view("<u8").reshape(-1)


def id_map_from_pages(pages: np.ndarray) -> Tuple[np.ndarray, int]:
    """IndexEngine::open's rebuild of (block, slot) -> passage id (src/engine.rs:148-162): live
    slots take consecutive passage ids in flush order, tombstoned slots u64::MAX. Returns
    (id_map, next passage id)."""
    masks = tombstone_masks(pages)
    slots = np.arange(VECTORS_PER_BLOCK, dtype=np.uint64)
    dead = ((masks[:, None] >> slots[None, :]) & np.uint64(1)).astype(bool).reshape(-1)
    out = np.full(dead.size, np.iinfo(np.uint64).max, np.uint64)
    live = ~dead
    out[live] = np.arange(int(live.sum()), dtype=np.uint64)
    return out, int(live.sum())


def _torch():
    import torch

    return torch


@dataclasses.dataclass
class PendingVector:
    """PendingVector (src/ring.rs:15-38) without the text."""

    passage_id: int
    embedding: np.ndarray
    timestamp: int
    source: int


class DeviceRing:
    """RingBuffer (src/ring.rs:49-119) whose pending embeddings live in HBM (mrl_ring_*)."""

    def __init__(self, dims: int, capacity: int = 1024, dev: Optional[Device] = None):
        self.dev = dev or default_device()
        self.dims = int(dims)
        self.capacity = max(int(capacity), VECTORS_PER_BLOCK)
        self.pending: List[PendingVector] = []
        self.ptr = C.c_void_p()
        check(self.dev.ptr, self.dev.lib.mrl_ring_create(self.dev.ptr, self.dims, self.capacity, C.byref(self.ptr)))

    def __len__(self) -> int:
        return len(self.pending)

    def push(self, item: PendingVector, eden: Optional[EdenFit] = None) -> Optional[np.ndarray]:
        """Append one vector; at 64 pending, drain them into an encoded page (returned)."""
        row = np.ascontiguousarray(item.embedding, np.float32).reshape(-1)
        if row.size != self.dims:
            raise ValueError("embedding length differs from the ring's dims")
        check(self.dev.ptr, self.dev.lib.mrl_ring_push(self.dev.ptr, self.ptr, row.ctypes.data_as(C.c_void_p)))
        self.pending.append(dataclasses.replace(item, embedding=row))
        if len(self.pending) >= VECTORS_PER_BLOCK:
            return self._flush_block(eden)
        return None

    def flush_partial(self, eden: Optional[EdenFit] = None) -> Optional[np.ndarray]:
        """Force a partial page (tombstone-padded); None when nothing is pending."""
        return self._flush_block(eden) if self.pending else None

    def _flush_block(self, eden: Optional[EdenFit]) -> np.ndarray:
        take = min(len(self.pending), VECTORS_PER_BLOCK)
        batch = self.pending[:take]
        rows = np.stack([p.embedding for p in batch])
        ts = np.array([p.timestamp for p in batch], np.uint32)
        src = np.array([p.source if p.source else SOURCE_DOC for p in batch], np.uint32)
        block = encode_blocks(rows, self.dims, eden=eden, timestamps=ts, sources=src, dev=self.dev)
        check(self.dev.ptr, self.dev.lib.mrl_ring_drain(self.dev.ptr, self.ptr, take))
        del self.pending[:take]
        return block

    def search_exact(self, query, top_k: int) -> List[Tuple[int, float]]:
        """search_exact (src/ring.rs:109-119): (pending index, exact dot), score descending."""
        torch = _torch()
        n = len(self.pending)
        if n == 0 or top_k < 1:
            return []
        k = min(int(top_k), 4096)
        q = torch.from_numpy(np.ascontiguousarray(query, np.float32).reshape(-1)).cuda(self.dev.index)
        rec = torch.zeros(record_bytes(k), dtype=torch.uint8, device=q.device)
        rows = C.c_void_p()
        check(self.dev.ptr, self.dev.lib.mrl_ring_rows(self.ptr, C.byref(rows)))
        check(self.dev.ptr, self.dev.lib.mrl_ring_search(self.dev.ptr, C.c_void_p(q.data_ptr()), rows, n, self.dims,
                                                         k, C.c_void_p(rec.data_ptr())))
        torch.cuda.synchronize(q.device)
        h = rec.cpu().numpy()
        m = int(h[12 * k: 12 * k + 4].view(np.uint32)[0])
        ids = h[: 8 * k].view(np.uint64)[:m]
        sc = h[8 * k: 12 * k].view(np.float32)[:m]
        return [(int(i) & 0xFFFF, float(s)) for i, s in zip(ids, sc)]

    def close(self) -> None:
        if self.ptr:
            self.dev.lib.mrl_ring_destroy(self.dev.ptr, self.ptr)
            self.ptr = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def rerank_exact_rows(query, candidate_ids: Sequence[int], corpus, dev: Optional[Device] = None
                      ) -> List[Tuple[int, float]]:
    """QueryPipeline::rerank_exact_rows: exact dot of the query with every candidate row of
    `corpus` (a CUDA f32 tensor [n_rows, dims], or a host array uploaded for this call), sorted by
    score descending; equal scores keep candidate order. Bit-identical to the reference's dot."""
    torch = _torch()
    dev = dev or default_device()
    cand = np.ascontiguousarray(candidate_ids, np.uint64).reshape(-1)
    if cand.size == 0:
        return []
    if not (isinstance(corpus, torch.Tensor) and corpus.is_cuda):
        corpus = torch.from_numpy(np.ascontiguousarray(corpus, np.float32)).cuda(dev.index)
    if corpus.dtype != torch.float32 or corpus.dim() != 2 or not corpus.is_contiguous():
        raise ValueError("corpus must be a contiguous [n_rows, dims] float32 tensor")
    n_rows, dims = corpus.shape
    q = torch.from_numpy(np.ascontiguousarray(query, np.float32).reshape(-1)).to(corpus.device)
    if q.numel() != dims:
        raise ValueError("query length differs from the corpus rows")
    d_cand = torch.from_numpy(cand.view(np.int64)).to(corpus.device)
    out_rows = torch.empty(cand.size, dtype=torch.int64, device=corpus.device)
    out_sc = torch.empty(cand.size, dtype=torch.float32, device=corpus.device)
    check(dev.ptr, dev.lib.mrl_rerank_exact(dev.ptr, C.c_void_p(q.data_ptr()), C.c_void_p(corpus.data_ptr()), n_rows,
                                            dims, C.c_void_p(d_cand.data_ptr()), cand.size,
                                            C.c_void_p(out_rows.data_ptr()), C.c_void_p(out_sc.data_ptr())))
    rows = out_rows.cpu().numpy().view(np.uint64)
    sc = out_sc.cpu().numpy()
    return [(int(r), float(s)) for r, s in zip(rows, sc)]


# Rust's serde snake_case of each variant (MinMax4 -> min_max4, L1Rabitq -> l1_rabitq), per enum
# (the IntEnum values overlap across enums).
_SERDE_NAMES = {
    PrefixCodec: {PrefixCodec.MIN_MAX4: "min_max4", PrefixCodec.EDEN_PROD: "eden_prod"},
    MidCodec: {MidCodec.RABITQ: "rabitq", MidCodec.EDEN_B1: "eden_b1"},
    StrataDepth: {StrataDepth.L0_ONLY: "l0_only", StrataDepth.L1_RABITQ: "l1_rabitq",
                  StrataDepth.FULL_64B: "full64b"},
}
_ENUMS = {"prefix_codec": PrefixCodec, "mid_codec": MidCodec, "strata_depth": StrataDepth}
_SCAN_KEYS = ("shortlist_cand", "cs_tolerance", "stratum4_weight", "temporal_filter_enable", "numa_sharding",
              "embed_dims", "mrl_prefix", "final_top_k", "eden_seed", "ring_buffer_size")


def config_from_json(d: dict) -> EngineConfig:
    """EngineConfig as serialised in manifest.json (serde, snake_case enums; src/config.rs:122-162).
    Keys outside the scan's subset are ignored; the defaults of #[serde(default)] fields apply."""
    cfg = EngineConfig()
    for key, enum_t in _ENUMS.items():
        if key in d:
            names = {name: v for v, name in _SERDE_NAMES[enum_t].items()}
            if d[key] not in names:
                raise ValueError(f"unknown variant `{d[key]}` for {key}")
            setattr(cfg, key, names[d[key]])
    for key in _SCAN_KEYS:
        if key in d:
            setattr(cfg, key, type(getattr(cfg, key))(d[key]))
    return cfg


# EngineConfig fields this package does not model, with the reference defaults
# (src/config.rs:172-201), so that a manifest written here deserialises in the reference.
_OTHER_DEFAULTS = {"slab_residency": "mmap_willneed", "rabitq_confidence": 2.576, "jit_batch_size": 64,
                   "io_read_workers": 4, "max_latency_budget_ms": 100, "tombstone_compact_ratio": 0.25,
                   "use_gemma2": False}


def config_to_json(cfg: EngineConfig, extra: Optional[dict] = None) -> dict:
    """EngineConfig in manifest.json form: the scan's fields from `cfg`, the others from `extra`
    (the manifest this index was opened from) or the reference defaults."""
    d = dict(_OTHER_DEFAULTS)
    d.update(extra or {})
    for key, enum_t in _ENUMS.items():
        d[key] = _SERDE_NAMES[enum_t][enum_t(getattr(cfg, key))]
    for key in _SCAN_KEYS:
        v = getattr(cfg, key)
        d[key] = bool(v) if isinstance(v, bool) else v
    return d


class IndexDir:
    """IndexEngine's on-disk index and query-side state with the segment resident in HBM."""

    def __init__(self, path: str, cfg: EngineConfig, raw_cfg: dict, eden: Optional[EdenFit], seg: Segment,
                 writer: SegmentWriter, id_map: np.ndarray, next_passage_id: int, dev: Device):
        self.path = path
        self.cfg = cfg
        self._raw_cfg = raw_cfg
        self.eden = eden
        self.segment = seg
        self.writer = writer
        self.id_map = id_map
        self.next_passage_id = next_passage_id
        self.dev = dev
        self.ring = DeviceRing(cfg.embed_dims, cfg.ring_buffer_size, dev)
        self._plans = C.c_void_p()
        check(dev.ptr, dev.lib.mrl_plans_alloc(dev.ptr, 1, cfg.embed_dims, C.byref(self._plans)))

    @staticmethod
    def create(path: str, cfg: EngineConfig, dev: Optional[Device] = None) -> "IndexDir":
        """IndexEngine::create (src/engine.rs:79-119): empty segment, manifest, default EDEN fit."""
        cfg.validate()
        dev = dev or default_device()
        os.makedirs(path, exist_ok=True)
        seg_path = os.path.join(path, SEGMENT_PATH)
        writer = SegmentWriter.create(seg_path)
        seg = load_segment(seg_path, dev)
        eden = EdenFit.default_prefix(cfg.eden_seed) if cfg.prefix_codec == PrefixCodec.EDEN_PROD else None
        ix = IndexDir(path, cfg, {}, eden, seg, writer, np.zeros(0, np.uint64), 0, dev)
        ix.write_manifest(0)
        ix.write_eden_fit()
        return ix

    @staticmethod
    def open(path: str, dev: Optional[Device] = None) -> "IndexDir":
        """IndexEngine::open (src/engine.rs:133-194): manifest.json, the segment file into HBM, the
        id map rebuilt from tombstones, eden_prefix.json (or the default fit)."""
        dev = dev or default_device()
        with open(os.path.join(path, "manifest.json")) as f:
            manifest = json.load(f)
        raw = manifest["config"]
        cfg = config_from_json(raw)
        cfg.validate()
        seg_path = os.path.join(path, SEGMENT_PATH)
        writer = SegmentWriter.open_append(seg_path)
        seg = load_segment(seg_path, dev)
        pages = np.fromfile(seg_path, np.uint8) if os.path.exists(seg_path) else np.zeros(0, np.uint8)
        id_map, next_pid = id_map_from_pages(pages)
        eden = None
        if cfg.prefix_codec == PrefixCodec.EDEN_PROD:
            ep = os.path.join(path, EDEN_PREFIX_FILE)
            eden = EdenFit.load_json(ep) if os.path.exists(ep) else EdenFit.default_prefix(cfg.eden_seed)
        return IndexDir(path, cfg, raw, eden, seg, writer, id_map, max(next_pid, int(manifest.get("next_passage_id", 0))),
                        dev)

    def write_manifest(self, blocks_written: int) -> None:
        m = {"version": MANIFEST_VERSION, "config": config_to_json(self.cfg, self._raw_cfg),
             "next_passage_id": self.next_passage_id, "blocks_written": int(blocks_written)}
        with open(os.path.join(self.path, "manifest.json"), "w") as f:
            json.dump(m, f, indent=2)

    def write_eden_fit(self) -> None:
        if self.eden is not None:
            self.eden.save_json(os.path.join(self.path, EDEN_PREFIX_FILE))

    def block_count(self) -> int:
        return self.segment.block_count()

    def ingest_vector(self, embedding, timestamp: int = 0, source_mask: int = 0) -> int:
        """The vector half of IndexEngine::ingest (src/engine.rs:240-291): a new passage id, the
        online EDEN fit update, the ring push, and at 64 pending the flush into a page that is
        written to the segment file and appended to the resident segment (append_live)."""
        pid = self.next_passage_id
        self.next_passage_id += 1
        src = source_mask if source_mask else SOURCE_DOC
        e = np.ascontiguousarray(embedding, np.float32).reshape(-1)
        if self.eden is not None:
            self.eden.observe_prefix(e)
        block = self.ring.push(PendingVector(pid, e, int(timestamp), src), self.eden)
        if block is not None:
            self._commit_block(block)
        return pid

    def flush(self) -> None:
        """IndexEngine::flush (src/engine.rs:527-541): pending vectors into a padded page."""
        block = self.ring.flush_partial(self.eden)
        if block is not None:
            self._commit_block(block)

    def _commit_block(self, block: np.ndarray) -> None:  # commit_block_inner, src/engine.rs:491-525
        masks = tombstone_masks(block)
        active = VECTORS_PER_BLOCK - bin(int(masks[0])).count("1")
        start = self.next_passage_id - active  # the last `active` passages written
        ids = np.full(VECTORS_PER_BLOCK, np.iinfo(np.uint64).max, np.uint64)
        ids[:active] = np.arange(start, start + active, dtype=np.uint64)
        self.id_map = np.concatenate([self.id_map, ids])
        n = self.writer.append_block(block)
        self.segment.append_live(block)
        self.write_manifest(n + 1)
        self.write_eden_fit()

    def search(self, query, time_lo=None, time_hi=None, mode: ScanMode = None) -> List[ScoredHit]:
        """The scan half of query_filtered (src/engine.rs:564-594): fused plan + scan of the
        resident segment and exact search of the ring, merged into one shortlist of
        cfg.shortlist_cand hits (mrl_engine_scan)."""
        torch = _torch()
        c = self.cfg
        if c.prefix_codec == PrefixCodec.EDEN_PROD and self.eden is not None:
            pc, mc, eden = PrefixCodec.EDEN_PROD, MidCodec.RABITQ, self.eden
        else:
            pc, mc, eden = PrefixCodec.MIN_MAX4, MidCodec.RABITQ, None
        desc, keep = _codec_desc(pc, mc, eden, None)
        sc = c.scan_config()
        if mode is not None:
            sc.mode = mode
        cfg_c = sc.to_c()
        k = int(sc.shortlist_cand)
        q = np.ascontiguousarray(query, np.float32).reshape(-1)
        if q.size != c.embed_dims:
            raise ValueError("assertion failed: query.len() == dims")
        dq = torch.from_numpy(q).cuda(self.dev.index)
        ids = torch.empty(k, dtype=torch.int64, device=dq.device)
        scores = torch.empty(k, dtype=torch.float32, device=dq.device)
        cs = torch.zeros(2, dtype=torch.int32, device=dq.device)
        lo, hi = _time_ptrs(time_lo, time_hi)
        ring = self.ring.ptr if len(self.ring) else None
        check(self.dev.ptr, self.dev.lib.mrl_engine_scan(
            self.dev.ptr, self.segment.ptr, C.c_void_p(dq.data_ptr()), c.embed_dims, C.byref(desc), self._plans,
            C.byref(cfg_c), lo, hi, ring, C.c_void_p(ids.data_ptr()), C.c_void_p(scores.data_ptr()),
            C.c_void_p(cs.data_ptr()), C.c_void_p(cs.data_ptr() + 4)))
        torch.cuda.synchronize(dq.device)  # the library runs on its own stream
        h = cs.cpu().numpy()
        del keep
        if int(h[1]) & 10:
            raise RuntimeError("scan: a bounded wait ran out (status bits 1/3)")
        n = int(h[0])
        hi_ids = ids[:n].cpu().numpy().view(np.uint64)
        hi_sc = scores[:n].cpu().numpy()
        return [ScoredHit(VectorId.from_u64(int(i)), float(s)) for i, s in zip(hi_ids, hi_sc)]

    def passage_ids(self, hits: Sequence[ScoredHit]) -> List[Tuple[int, float]]:
        """The fetch stage's id resolution (src/engine.rs:601-626): ring hits to the pending
        vector's passage id, scanned hits through the id map; tombstoned slots are skipped."""
        out = []
        for h in hits:
            if h.id.block == RING_BLOCK:
                if h.id.slot < len(self.ring.pending):
                    out.append((self.ring.pending[h.id.slot].passage_id, h.score))
                continue
            ordinal = h.id.block * VECTORS_PER_BLOCK + h.id.slot
            if ordinal < self.id_map.size and self.id_map[ordinal] != np.iinfo(np.uint64).max:
                out.append((int(self.id_map[ordinal]), h.score))
        return out

    def close(self) -> None:
        if self._plans:
            self.dev.lib.mrl_plans_free(self.dev.ptr, self._plans)
            self._plans = C.c_void_p()
        self.ring.close()
        self.segment.free()
        self.writer.close()
