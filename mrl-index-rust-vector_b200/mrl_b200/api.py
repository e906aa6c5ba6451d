"""Host-side mirror of the reference's scan-path interface, backed by libmrl_b200 on a B200.

Names, argument meaning and defaults follow the reference crate `mrl_index` v0.3.5 (file:line
relative to its project root) so callers of the reference's scan path find the same surface:

  * EngineConfig / ScanConfig / PrefixCodec / MidCodec / StrataDepth   (src/config.rs:8-241)
  * EdenFit (fit_prefix / fit_band / zeros / observe_prefix / save_json / load_json)
                                                                      (src/eden.rs:104-203)
  * VectorId / ScoredHit                                              (src/block.rs:200-222,
                                                                       src/scan.rs:304-308)
  * QueryPlan.from_query / from_query_eden / from_query_eden_dual / from_query_codec
                                                                      (src/scan.rs:73-124)
  * scan_blocks(segment, plan, cfg, time_lo, time_hi)                 (src/scan.rs:802-810)
  * QueryPipeline.{new, with_eden, with_eden_dual, build_plan, scan_slab} (src/pipeline.rs:34-98)
  * Segment (SegmentReader::open + as_slice + append_live, src/segment.rs:88-232) as a
    device-resident set of pages.

Contract violations that panic in the reference raise MrlError / ValueError here.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import enum
import json
import math
from typing import Iterable, List, Optional, Sequence

import numpy as np

from . import _capi
from ._capi import CodecDesc, MrlError, QueryPlanC, ScanCfgC, check, load

VECTORS_PER_BLOCK = 64
BLOCK_BYTES = 4096
MRL_PREFIX_DIMS = 64
RABITQ_DIMS = 128
TAIL_START = 192
DEFAULT_STRATUM4_WEIGHT = 0.20  # src/rotate.rs:120


class PrefixCodec(enum.IntEnum):
    MIN_MAX4 = 0
    EDEN_PROD = 1


class MidCodec(enum.IntEnum):
    RABITQ = 0
    EDEN_B1 = 1


class StrataDepth(enum.IntEnum):
    L0_ONLY = 0
    L1_RABITQ = 1
    FULL_64B = 2


class ScanMode(enum.IntEnum):
    FAST = 0   # exact int32 stage sums choose the candidates; the final top-k is rescored in the exact mode
    EXACT = 1  # bit-identical f32 arithmetic of the reference for every slot


@dataclasses.dataclass
class ScanConfig:
    """`ScanConfig` (src/config.rs:79-114) plus the device scoring mode."""

    shortlist_cand: int = 64
    cs_tolerance: float = 1.0
    stratum4_weight: float = DEFAULT_STRATUM4_WEIGHT
    strata_depth: StrataDepth = StrataDepth.FULL_64B
    temporal_filter_enable: bool = True
    numa_sharding: bool = True
    mode: ScanMode = ScanMode.FAST

    def validate(self) -> None:
        if not 16 <= self.shortlist_cand <= 4096:
            raise ValueError("shortlist_cand must be in [16, 4096]")
        if not 0.80 <= self.cs_tolerance <= 1.20:
            raise ValueError("cs_tolerance must be in [0.80, 1.20]")
        if not 0.05 <= self.stratum4_weight <= 1.50:
            raise ValueError("stratum4_weight must be in [0.05, 1.50]")

    def to_c(self) -> ScanCfgC:
        return ScanCfgC(int(self.shortlist_cand), float(self.cs_tolerance), float(self.stratum4_weight),
                        int(self.strata_depth), int(bool(self.temporal_filter_enable)),
                        int(bool(self.numa_sharding)), int(self.mode))


@dataclasses.dataclass
class EngineConfig:
    """Scan-relevant subset of `EngineConfig` with the reference defaults (src/config.rs:172-201)."""

    strata_depth: StrataDepth = StrataDepth.FULL_64B
    numa_sharding: bool = True
    shortlist_cand: int = 64
    cs_tolerance: float = 1.0
    stratum4_weight: float = DEFAULT_STRATUM4_WEIGHT
    temporal_filter_enable: bool = True
    embed_dims: int = 384
    mrl_prefix: int = 64
    final_top_k: int = 10
    prefix_codec: PrefixCodec = PrefixCodec.EDEN_PROD
    eden_seed: int = 1
    mid_codec: MidCodec = MidCodec.RABITQ
    ring_buffer_size: int = 1024
    scan_mode: ScanMode = ScanMode.FAST

    def scan_config(self) -> ScanConfig:
        return ScanConfig(self.shortlist_cand, self.cs_tolerance, self.stratum4_weight, self.strata_depth,
                          self.temporal_filter_enable, self.numa_sharding, self.scan_mode)

    def validate(self) -> None:  # src/config.rs:203-217
        self.scan_config().validate()
        if self.embed_dims < TAIL_START:
            raise ValueError(f"embed_dims ({self.embed_dims}) must be >= tail_start ({TAIL_START})")
        if self.mrl_prefix != 64:
            raise ValueError("mrl_prefix must be 64 for PaxBlock64 layout")
        if self.ring_buffer_size < 64:
            raise ValueError("ring_buffer_size must be >= 64")

    def active_strata(self) -> Sequence[int]:  # src/config.rs:234-240
        return {StrataDepth.L0_ONLY: (0,), StrataDepth.L1_RABITQ: (0, 1, 2, 3, 5),
                StrataDepth.FULL_64B: (0, 1, 2, 3, 4, 5)}[StrataDepth(self.strata_depth)]


@dataclasses.dataclass
class EdenFit:
    """`EdenFit` (src/eden.rs:104-203): fitted centre of the coded slice, persisted as
    eden_prefix.json with the same field names."""

    dim: int
    bits: int
    seed: int
    mean: np.ndarray
    n_observed: int = 0

    @staticmethod
    def fit_band(rows: np.ndarray, start: int, dim: int, bits: int, seed: int) -> "EdenFit":
        if not 1 <= bits <= 4:
            raise ValueError("bits must be in 1..=4")
        if dim <= 0 or dim & (dim - 1):
            raise ValueError(f"EDEN slice dim must be 2^k, got {dim}")
        rows = np.ascontiguousarray(rows, np.float32)
        if rows.shape[0] == 0:
            raise ValueError("empty corpus for EdenFit")
        mean = np.zeros(dim, np.float32)
        for r in rows[:, start:start + dim]:  # sequential f32 sum over rows, as the reference
            mean += r
        inv = np.float32(1.0) / np.float32(rows.shape[0])
        return EdenFit(dim, bits, seed, (mean * inv).astype(np.float32), rows.shape[0])

    @staticmethod
    def fit_prefix(rows: np.ndarray, bits: int = 4, seed: int = 1) -> "EdenFit":
        return EdenFit.fit_band(rows, 0, MRL_PREFIX_DIMS, bits, seed)

    @staticmethod
    def zeros(dim: int, bits: int, seed: int) -> "EdenFit":
        return EdenFit(dim, bits, seed, np.zeros(dim, np.float32), 0)

    @staticmethod
    def default_prefix(seed: int = 1) -> "EdenFit":
        return EdenFit.zeros(MRL_PREFIX_DIMS, 4, seed)

    def observe_prefix(self, x: np.ndarray) -> None:  # src/eden.rs:182-191
        n = self.n_observed + 1
        inv = np.float32(1.0) / np.float32(n)
        x = np.asarray(x, np.float32)[: self.dim]
        self.mean = (self.mean + (x - self.mean) * inv).astype(np.float32)
        self.n_observed = n

    def save_json(self, path: str) -> None:
        with open(path, "w") as f:
            json.dump({"dim": self.dim, "bits": self.bits, "seed": self.seed,
                       "mean": [float(v) for v in self.mean], "n_observed": self.n_observed}, f, indent=2)

    @staticmethod
    def load_json(path: str) -> "EdenFit":
        with open(path) as f:
            d = json.load(f)
        return EdenFit(d["dim"], d["bits"], d["seed"], np.asarray(d["mean"], np.float32), d.get("n_observed", 0))


@dataclasses.dataclass(frozen=True)
class VectorId:
    block: int
    slot: int

    def as_u64(self) -> int:
        return (self.block << 16) | self.slot

    @staticmethod
    def from_u64(v: int) -> "VectorId":
        v = int(v)
        return VectorId(v >> 16, v & 0xFFFF)


@dataclasses.dataclass(frozen=True)
class ScoredHit:
    id: VectorId
    score: float


class Device:
    """A libmrl_b200 context on one CUDA device (one stream)."""

    def __init__(self, index: int = 0):
        self.lib = load()
        self.ptr = C.c_void_p()
        rc = self.lib.mrl_ctx_create(int(index), C.byref(self.ptr))
        if rc != 0:
            raise MrlError(rc, f"cannot create a context on CUDA device {index} (needs an sm_100 GPU)")
        self.index = index

    def close(self) -> None:
        if self.ptr:
            self.lib.mrl_ctx_destroy(self.ptr)
            self.ptr = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return int(self.lib.mrl_ctx_stream(self.ptr) or 0)

    def set_stream(self, stream: int) -> None:
        check(self.ptr, self.lib.mrl_ctx_set_stream(self.ptr, C.c_void_p(stream)))

    def geometry(self, k: int):
        ctas, ll = C.c_uint32(), C.c_uint32()
        check(self.ptr, self.lib.mrl_scan_geometry(self.ptr, k, C.byref(ctas), C.byref(ll)))
        return ctas.value, ll.value

    def set_list_len(self, n: int) -> None:
        check(self.ptr, self.lib.mrl_set_list_len(self.ptr, n))

    def set_scan_ctas(self, n: int) -> None:
        """CTAs per single-query scan launch (mrl_set_scan_ctas): 0 = one per SM."""
        check(self.ptr, self.lib.mrl_set_scan_ctas(self.ptr, n))


_default_device: Optional[Device] = None


def default_device() -> Device:
    global _default_device
    if _default_device is None:
        _default_device = Device(0)
    return _default_device


def _f32p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(C.POINTER(C.c_float))


class Segment:
    """Device-resident slab of PaxBlock64 pages (the scan's `&[PaxBlock64]`)."""

    def __init__(self, ptr, dev: Device, keep=None):
        self.ptr = ptr
        self.dev = dev

    @staticmethod
    def upload(blocks, dev: Optional[Device] = None, block_id_base: int = 0) -> "Segment":
        dev = dev or default_device()
        buf = np.ascontiguousarray(np.frombuffer(bytes(blocks), np.uint8) if not isinstance(blocks, np.ndarray)
                                   else blocks.view(np.uint8).reshape(-1))
        if buf.size % BLOCK_BYTES:
            raise ValueError(f"corrupt segment size {buf.size} (not multiple of 4096)")  # src/segment.rs:17
        out = C.c_void_p()
        check(dev.ptr, dev.lib.mrl_segment_upload(dev.ptr, buf.ctypes.data_as(C.c_void_p), buf.size // BLOCK_BYTES,
                                                  block_id_base, C.byref(out)))
        return Segment(out, dev)

    def append_live(self, block) -> None:
        buf = np.ascontiguousarray(np.frombuffer(bytes(block), np.uint8) if not isinstance(block, np.ndarray)
                                   else block.view(np.uint8).reshape(-1))
        if buf.size != BLOCK_BYTES:
            raise ValueError("a block is exactly 4096 bytes")
        check(self.dev.ptr, self.dev.lib.mrl_segment_append(self.dev.ptr, self.ptr, buf.ctypes.data_as(C.c_void_p)))

    def block_count(self) -> int:
        return int(self.dev.lib.mrl_segment_blocks(self.ptr))

    def read_layout(self):
        n = self.block_count()
        pages = np.zeros(n * BLOCK_BYTES, np.uint8)
        ts = np.zeros(n * 2, np.uint32)
        check(self.dev.ptr, self.dev.lib.mrl_segment_read_layout(self.dev.ptr, self.ptr,
                                                                 pages.ctypes.data_as(C.c_void_p),
                                                                 ts.ctypes.data_as(C.c_void_p)))
        return pages, ts

    def device_ptrs(self):
        p, t = C.c_void_p(), C.c_void_p()
        check(self.dev.ptr, self.dev.lib.mrl_segment_device_ptrs(self.ptr, C.byref(p), C.byref(t)))
        return p.value, t.value

    def free(self) -> None:
        if self.ptr:
            self.dev.lib.mrl_segment_free(self.dev.ptr, self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _codec_desc(prefix_codec, mid_codec, eden: Optional[EdenFit], eden_mid: Optional[EdenFit]):
    keep = []
    em = mm = None
    if eden is not None:
        em = np.ascontiguousarray(eden.mean, np.float32)
        keep.append(em)
    if eden_mid is not None:
        mm = np.ascontiguousarray(eden_mid.mean, np.float32)
        keep.append(mm)
    d = CodecDesc(int(prefix_codec), int(mid_codec), _f32p(em), int(eden.seed) if eden else 1,
                  _f32p(mm), int(eden_mid.seed) if eden_mid else 1)
    return d, keep


def _check_plan_args(queries, prefix_codec, mid_codec, eden, eden_mid) -> np.ndarray:
    """The contract checks of QueryPlan::from_query_codec (src/scan.rs:113-124); returns the
    queries as a contiguous [n_q, dims] f32 array."""
    q = np.ascontiguousarray(np.atleast_2d(queries), np.float32)
    if q.shape[1] < MRL_PREFIX_DIMS + RABITQ_DIMS:
        raise ValueError("assertion failed: dims >= MRL_PREFIX_DIMS + RABITQ_DIMS")  # src/scan.rs:114
    if prefix_codec == PrefixCodec.EDEN_PROD:
        if eden is None:
            raise ValueError("EdenProd requires EdenFit")
        if eden.dim != MRL_PREFIX_DIMS or eden.bits != 4:
            raise ValueError("EdenProd fit must have dim 64 and bits 4")
    if mid_codec == MidCodec.EDEN_B1:
        if eden_mid is None:
            raise ValueError("EdenB1 mid requires EdenFit")
        if eden_mid.dim != RABITQ_DIMS or eden_mid.bits != 1:
            raise ValueError("EdenB1 mid fit must have dim 128 and bits 1")
    return q


class QueryPlan:
    """Device-resident plan(s) built by the plan kernel (QueryPlan::from_query_codec)."""

    def __init__(self, ptr, dev: Device, n_q: int, dims: int):
        self.ptr = ptr
        self.dev = dev
        self.n_q = n_q
        self.dims = dims

    @staticmethod
    def from_queries(queries: np.ndarray, prefix_codec=PrefixCodec.MIN_MAX4, mid_codec=MidCodec.RABITQ,
                     eden: Optional[EdenFit] = None, eden_mid: Optional[EdenFit] = None,
                     dev: Optional[Device] = None) -> "QueryPlan":
        dev = dev or default_device()
        q = _check_plan_args(queries, prefix_codec, mid_codec, eden, eden_mid)
        n_q, dims = q.shape
        desc, keep = _codec_desc(prefix_codec, mid_codec, eden, eden_mid)
        out = C.c_void_p()
        check(dev.ptr, dev.lib.mrl_plan_build(dev.ptr, q.ctypes.data_as(C.c_void_p), n_q, dims, C.byref(desc),
                                              C.byref(out)))
        del keep
        return QueryPlan(out, dev, n_q, dims)

    @staticmethod
    def from_query(query, dims: int, dev: Optional[Device] = None) -> "QueryPlan":
        q = np.asarray(query, np.float32)
        if q.size != dims:
            raise ValueError("assertion failed: query.len() == dims")
        return QueryPlan.from_queries(q, PrefixCodec.MIN_MAX4, MidCodec.RABITQ, dev=dev)

    @staticmethod
    def from_query_eden(query, dims: int, fit: EdenFit, dev: Optional[Device] = None) -> "QueryPlan":
        q = np.asarray(query, np.float32)
        if q.size != dims:
            raise ValueError("assertion failed: query.len() == dims")
        return QueryPlan.from_queries(q, PrefixCodec.EDEN_PROD, MidCodec.RABITQ, eden=fit, dev=dev)

    @staticmethod
    def from_query_eden_dual(query, dims: int, prefix: EdenFit, mid: EdenFit,
                             dev: Optional[Device] = None) -> "QueryPlan":
        q = np.asarray(query, np.float32)
        return QueryPlan.from_queries(q, PrefixCodec.EDEN_PROD, MidCodec.EDEN_B1, eden=prefix, eden_mid=mid, dev=dev)

    @staticmethod
    def from_query_codec(query, dims: int, prefix_codec, mid_codec, eden=None, eden_mid=None,
                         dev: Optional[Device] = None) -> "QueryPlan":
        q = np.asarray(query, np.float32)
        if q.size != dims:
            raise ValueError("assertion failed: query.len() == dims")
        return QueryPlan.from_queries(q, prefix_codec, mid_codec, eden, eden_mid, dev=dev)

    def fields(self, i: int = 0) -> QueryPlanC:
        out = QueryPlanC()
        check(self.dev.ptr, self.dev.lib.mrl_plan_read(self.dev.ptr, self.ptr, i, C.byref(out)))
        return out

    def free(self) -> None:
        if self.ptr:
            self.dev.lib.mrl_plans_free(self.dev.ptr, self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _time_ptrs(time_lo, time_hi):
    lo = None if time_lo is None else C.byref(C.c_uint32(int(time_lo)))
    hi = None if time_hi is None else C.byref(C.c_uint32(int(time_hi)))
    return lo, hi


def _cfg_of(cfg) -> ScanConfig:
    return cfg.scan_config() if isinstance(cfg, EngineConfig) else cfg


def scan_blocks_batch(segment: Segment, plan: QueryPlan, cfg, time_lo=None, time_hi=None):
    """All plans of `plan` against `segment`: returns (ids [n_q,k] u64, scores [n_q,k] f32, counts)."""
    sc = _cfg_of(cfg)
    c = sc.to_c()
    k = int(sc.shortlist_cand)
    ids = np.zeros((plan.n_q, k), np.uint64)
    scores = np.zeros((plan.n_q, k), np.float32)
    counts = np.zeros(plan.n_q, np.uint32)
    lo, hi = _time_ptrs(time_lo, time_hi)
    dev = segment.dev
    check(dev.ptr, dev.lib.mrl_scan(dev.ptr, segment.ptr, plan.ptr, C.byref(c), lo, hi,
                                    ids.ctypes.data_as(C.c_void_p), scores.ctypes.data_as(C.c_void_p),
                                    counts.ctypes.data_as(C.c_void_p)))
    return ids, scores, counts


def query_scan(segment: Segment, queries, cfg, prefix_codec=PrefixCodec.MIN_MAX4, mid_codec=MidCodec.RABITQ,
               eden: Optional[EdenFit] = None, eden_mid: Optional[EdenFit] = None, time_lo=None, time_hi=None):
    """Plan build + scan of every query in one fused launch per query (mrl_query_scan; the
    reference's QueryPipeline::build_plan followed by scan_segments_into, src/pipeline.rs:63-133).
    Returns (ids [n_q,k] u64, scores [n_q,k] f32, counts [n_q], plan) with the plans kept."""
    dev = segment.dev
    q = _check_plan_args(queries, prefix_codec, mid_codec, eden, eden_mid)
    n_q, dims = q.shape
    sc = _cfg_of(cfg)
    c = sc.to_c()
    k = int(sc.shortlist_cand)
    plans = C.c_void_p()
    check(dev.ptr, dev.lib.mrl_plans_alloc(dev.ptr, n_q, dims, C.byref(plans)))
    plan = QueryPlan(plans, dev, n_q, dims)
    desc, keep = _codec_desc(prefix_codec, mid_codec, eden, eden_mid)
    ids = np.zeros((n_q, k), np.uint64)
    scores = np.zeros((n_q, k), np.float32)
    counts = np.zeros(n_q, np.uint32)
    lo, hi = _time_ptrs(time_lo, time_hi)
    check(dev.ptr, dev.lib.mrl_query_scan(dev.ptr, segment.ptr, q.ctypes.data_as(C.c_void_p), n_q, dims,
                                          C.byref(desc), plans, C.byref(c), lo, hi, ids.ctypes.data_as(C.c_void_p),
                                          scores.ctypes.data_as(C.c_void_p), counts.ctypes.data_as(C.c_void_p)))
    del keep
    return ids, scores, counts, plan


MAX_INFLIGHT = 8  # MRL_MAX_INFLIGHT


class QueryStream:
    """Pipelined host queries over one segment (mrl_query_submit / mrl_query_collect): submit()
    launches the fused plan + scan of one query into a result slot and returns at once; collect()
    waits for that slot's top-k. Keeping two or more queries submitted lets consecutive scans
    overlap on the device. The reference's scan is a blocking call; this has no counterpart there."""

    def __init__(self, segment: Segment, cfg, prefix_codec=PrefixCodec.MIN_MAX4, mid_codec=MidCodec.RABITQ,
                 eden: Optional[EdenFit] = None, eden_mid: Optional[EdenFit] = None, time_lo=None, time_hi=None):
        self.segment = segment
        self.dev = segment.dev
        sc = _cfg_of(cfg)
        self.c = sc.to_c()
        self.k = int(sc.shortlist_cand)
        self.desc, self._keep = _codec_desc(prefix_codec, mid_codec, eden, eden_mid)
        self._tl = (np.array([time_lo], np.uint32) if time_lo is not None else None,
                    np.array([time_hi], np.uint32) if time_hi is not None else None)
        self._ids = np.zeros(self.k, np.uint64)
        self._sc = np.zeros(self.k, np.float32)
        self._n = np.zeros(1, np.uint32)

    def _time(self):
        lo, hi = self._tl
        return (lo.ctypes.data_as(C.c_void_p) if lo is not None else None,
                hi.ctypes.data_as(C.c_void_p) if hi is not None else None)

    def submit(self, query, slot: int) -> None:
        q = np.ascontiguousarray(query, np.float32).reshape(-1)
        lo, hi = self._time()
        check(self.dev.ptr, self.dev.lib.mrl_query_submit(self.dev.ptr, self.segment.ptr, q.ctypes.data_as(C.c_void_p),
                                                          q.shape[0], C.byref(self.desc), C.byref(self.c), lo, hi, slot))

    def collect(self, slot: int):
        """(ids [count] u64, scores [count] f32) of the query in `slot`."""
        check(self.dev.ptr, self.dev.lib.mrl_query_collect(self.dev.ptr, slot, self._ids.ctypes.data_as(C.c_void_p),
                                                           self._sc.ctypes.data_as(C.c_void_p),
                                                           self._n.ctypes.data_as(C.c_void_p)))
        n = int(self._n[0])
        return self._ids[:n].copy(), self._sc[:n].copy()


def scan_blocks(segment: Segment, plan: QueryPlan, cfg, time_lo=None, time_hi=None) -> List[ScoredHit]:
    """`scan_blocks` (src/scan.rs:802-810): top `shortlist_cand` hits, score descending."""
    if plan.n_q != 1:
        raise ValueError("scan_blocks takes one plan; use scan_blocks_batch for several")
    ids, scores, counts = scan_blocks_batch(segment, plan, cfg, time_lo, time_hi)
    n = int(counts[0])
    return [ScoredHit(VectorId.from_u64(int(i)), float(s)) for i, s in zip(ids[0, :n], scores[0, :n])]


class ScanStatsC(C.Structure):
    _fields_ = [("blocks", C.c_uint64), ("active_vecs", C.c_uint64), ("after_prefix", C.c_uint64),
                ("after_s1", C.c_uint64), ("after_s4_budget", C.c_uint64), ("pushed", C.c_uint64)]


@dataclasses.dataclass
class ScanStats:
    """`ScanStats` (src/scan.rs:269-302), counted by mrl_scan_blocks_stats against the final shortlist
    threshold (the counts of a fully warmed scan)."""

    blocks: int = 0
    active_vecs: int = 0
    after_prefix: int = 0
    after_s1: int = 0
    after_s4_budget: int = 0
    pushed: int = 0

    def merge(self, other: "ScanStats") -> None:  # src/scan.rs:281-288
        for f in dataclasses.fields(self):
            setattr(self, f.name, getattr(self, f.name) + getattr(other, f.name))

    def summary(self) -> str:  # ScanStats::print_summary, src/scan.rs:290-301
        a = float(max(self.active_vecs, 1))
        return (f"scan-stats: blocks={self.blocks} active={self.active_vecs}  "
                f"keep_prefix={100.0 * self.after_prefix / a:.2f}%  keep_s1={100.0 * self.after_s1 / a:.2f}%  "
                f"keep_s4bud={100.0 * self.after_s4_budget / a:.2f}%  pushed={100.0 * self.pushed / a:.2f}%")


def scan_blocks_stats(segment: Segment, plan: QueryPlan, cfg, time_lo=None, time_hi=None, q: int = 0):
    """`scan_blocks_stats` (src/scan.rs:813-886): the hits of plan q and its ScanStats
    (mrl_scan_blocks_stats)."""
    sc = _cfg_of(cfg)
    c = sc.to_c()
    k = int(sc.shortlist_cand)
    ids = np.zeros(k, np.uint64)
    scores = np.zeros(k, np.float32)
    count = C.c_uint32(0)
    st = ScanStatsC()
    lo, hi = _time_ptrs(time_lo, time_hi)
    dev = segment.dev
    check(dev.ptr, dev.lib.mrl_scan_blocks_stats(dev.ptr, segment.ptr, plan.ptr, q, C.byref(c), lo, hi,
                                          ids.ctypes.data_as(C.c_void_p), scores.ctypes.data_as(C.c_void_p),
                                          C.byref(count), C.byref(st)))
    n = int(count.value)
    hits = [ScoredHit(VectorId.from_u64(int(i)), float(s)) for i, s in zip(ids[:n], scores[:n])]
    return hits, ScanStats(*(int(getattr(st, f[0])) for f in ScanStatsC._fields_))


def vector_scores(segment: Segment, plan: QueryPlan, cfg, q: int = 0, time_lo=None, time_hi=None):
    """Per-slot scores (and fast-mode int32 stage sums) of plan q for every slot of the segment."""
    sc = _cfg_of(cfg)
    c = sc.to_c()
    n = segment.block_count() * VECTORS_PER_BLOCK
    scores = np.zeros(n, np.float32)
    active = np.zeros(n, np.uint8)
    parts = np.zeros(n * 3, np.int32)
    lo, hi = _time_ptrs(time_lo, time_hi)
    dev = segment.dev
    check(dev.ptr, dev.lib.mrl_debug_vector_scores(dev.ptr, segment.ptr, plan.ptr, q, C.byref(c), lo, hi,
                                                   scores.ctypes.data_as(C.c_void_p),
                                                   active.ctypes.data_as(C.c_void_p),
                                                   parts.ctypes.data_as(C.c_void_p)))
    return scores, active, parts.reshape(-1, 3)


def score_bound(segment: Segment, plan: QueryPlan, cfg, q: int = 0) -> float:
    """The bound E the fast mode's final ranking assumes: |fast score - exact score| <= E for every
    slot of the segment under plan q (mrl_debug_score_bound)."""
    c = _cfg_of(cfg).to_c()
    out = C.c_float(0.0)
    dev = segment.dev
    check(dev.ptr, dev.lib.mrl_debug_score_bound(dev.ptr, segment.ptr, plan.ptr, q, C.byref(c), C.byref(out)))
    return float(out.value)


def control_words(dev: "Device") -> List[int]:
    """The context's scan control words, 8 per scratch set (mrl_debug_control_words)."""
    out = (C.c_uint32 * 128)()
    check(dev.ptr, dev.lib.mrl_debug_control_words(dev.ptr, out))
    return list(out)


def encode_blocks(rows: np.ndarray, dims: int, eden: Optional[EdenFit] = None, eden_mid: Optional[EdenFit] = None,
                  timestamps=None, sources=None, dev: Optional[Device] = None) -> np.ndarray:
    """encode_block_with_fits over consecutive groups of 64 rows (src/quantize.rs:36-96)."""
    dev = dev or default_device()
    r = np.ascontiguousarray(rows, np.float32).reshape(-1, dims)
    n = r.shape[0]
    ts = None if timestamps is None else np.ascontiguousarray(timestamps, np.uint32)
    src = None if sources is None else np.ascontiguousarray(sources, np.uint32)
    pc = PrefixCodec.EDEN_PROD if eden is not None else PrefixCodec.MIN_MAX4
    mc = MidCodec.EDEN_B1 if eden_mid is not None else MidCodec.RABITQ
    desc, keep = _codec_desc(pc, mc, eden, eden_mid)
    out = np.zeros(((n + 63) // 64) * BLOCK_BYTES, np.uint8)
    check(dev.ptr, dev.lib.mrl_encode_blocks(dev.ptr, r.ctypes.data_as(C.c_void_p), n, dims,
                                             None if ts is None else ts.ctypes.data_as(C.c_void_p),
                                             None if src is None else src.ctypes.data_as(C.c_void_p),
                                             C.byref(desc), out.ctypes.data_as(C.c_void_p)))
    del keep
    return out


class QueryPipeline:
    """`QueryPipeline` (src/pipeline.rs:34-98): codec dispatch + timed scan of a slab."""

    def __init__(self, cfg: EngineConfig, eden: Optional[EdenFit] = None, eden_mid: Optional[EdenFit] = None,
                 dev: Optional[Device] = None):
        self.cfg = cfg
        self.eden = eden
        self.eden_mid = eden_mid
        self.dev = dev or default_device()

    @staticmethod
    def new(cfg: EngineConfig, dev=None) -> "QueryPipeline":
        return QueryPipeline(cfg, dev=dev)

    @staticmethod
    def with_eden(cfg: EngineConfig, fit: EdenFit, dev=None) -> "QueryPipeline":
        return QueryPipeline(cfg, fit, dev=dev)

    @staticmethod
    def with_eden_dual(cfg: EngineConfig, prefix: EdenFit, mid: EdenFit, dev=None) -> "QueryPipeline":
        return QueryPipeline(cfg, prefix, mid, dev=dev)

    def build_plan(self, query) -> QueryPlan:  # src/pipeline.rs:63-74
        c = self.cfg
        if c.prefix_codec == PrefixCodec.EDEN_PROD and c.mid_codec == MidCodec.EDEN_B1 and self.eden and self.eden_mid:
            return QueryPlan.from_query_eden_dual(query, c.embed_dims, self.eden, self.eden_mid, dev=self.dev)
        if c.prefix_codec == PrefixCodec.EDEN_PROD and self.eden is not None:
            return QueryPlan.from_query_eden(query, c.embed_dims, self.eden, dev=self.dev)
        return QueryPlan.from_query(query, c.embed_dims, dev=self.dev)

    def search(self, query, segment: Segment, time_lo=None, time_hi=None) -> List[ScoredHit]:
        """build_plan + scan of one query in a single fused launch (mrl_query_scan)."""
        c = self.cfg
        if c.prefix_codec == PrefixCodec.EDEN_PROD and c.mid_codec == MidCodec.EDEN_B1 and self.eden and self.eden_mid:
            codec = dict(prefix_codec=PrefixCodec.EDEN_PROD, mid_codec=MidCodec.EDEN_B1, eden=self.eden,
                         eden_mid=self.eden_mid)
        elif c.prefix_codec == PrefixCodec.EDEN_PROD and self.eden is not None:
            codec = dict(prefix_codec=PrefixCodec.EDEN_PROD, mid_codec=MidCodec.RABITQ, eden=self.eden)
        else:
            codec = dict(prefix_codec=PrefixCodec.MIN_MAX4, mid_codec=MidCodec.RABITQ)
        q = np.asarray(query, np.float32)
        if q.size != c.embed_dims:
            raise ValueError("assertion failed: query.len() == dims")
        ids, scores, counts, plan = query_scan(segment, q.reshape(1, -1), c, time_lo=time_lo, time_hi=time_hi,
                                               **codec)
        plan.free()
        n = int(counts[0])
        return [ScoredHit(VectorId.from_u64(int(ids[0, i])), float(scores[0, i])) for i in range(n)]

    def scan_slab(self, query, segment: Segment, time_lo=None, time_hi=None):
        import time
        plan = self.build_plan(query)
        t = time.perf_counter()
        hits = scan_blocks(segment, plan, self.cfg, time_lo, time_hi)
        return plan, hits, (time.perf_counter() - t) * 1000.0, segment.block_count()


def scored_hits_to_row_ids(hits: Iterable[ScoredHit]) -> List[int]:  # src/pipeline.rs:175-181
    return [h.id.block * VECTORS_PER_BLOCK + h.id.slot for h in hits if h.id.block != 0xFFFFFFFF]


def row_id_to_vector_id(row: int) -> VectorId:
    return VectorId(row // VECTORS_PER_BLOCK, row % VECTORS_PER_BLOCK)
