"""ctypes binding of the CPU oracle — TEST INFRASTRUCTURE ONLY.

The oracle is a CPU restatement of the reference crate's PaxBlock64 scan path (see mrl_oracle.h
for the per-function reference citations and the parity-pinning status). Only tests/,
__graft_entry__.smoke() and bench.py's CPU baseline / reference arm may import this module; the
product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")

MINMAX4, EDEN_PROD = 0, 1
RABITQ, EDEN_B1 = 0, 1
L0_ONLY, L1_RABITQ, FULL_64B = 0, 1, 2


class QueryPlan(C.Structure):
    """Field-for-field mirror of `QueryPlan` (src/scan.rs:19-71)."""

    _fields_ = [
        ("dims", C.c_uint32), ("prefix_codec", C.c_uint32), ("mid_codec", C.c_uint32),
        ("has_tail_fold", C.c_uint32),
        ("prefix", C.c_float * 64), ("bit_weights", (C.c_float * 4) * 64),
        ("rabitq_q", C.c_float * 128), ("rabitq_scale", C.c_float),
        ("rabitq_weights2", C.c_float * 128), ("rabitq_base", C.c_float),
        ("rabitq_lut", (C.c_float * 16) * 32),
        ("tail_fold_q", C.c_float * 64), ("tail_fold_weights2", C.c_float * 64),
        ("tail_fold_base", C.c_float), ("q_tail_norm", C.c_float), ("q_mid_norm", C.c_float),
        ("q_after_prefix", C.c_float), ("q_after_s1", C.c_float), ("s4_abs_budget", C.c_float),
        ("prefix_l1", C.c_float), ("prefix_sum", C.c_float),
        ("eden_q_rot", C.c_float * 64), ("eden_mean_ip", C.c_float),
        ("eden_inv_sqrt_d", C.c_float), ("eden_codebook", C.c_float * 16),
        ("eden_mid_q_rot", C.c_float * 128), ("eden_mid_mean_ip", C.c_float),
        ("eden_mid_inv_sqrt_d", C.c_float), ("eden_mid_codebook", C.c_float * 2),
    ]


class ScanCfg(C.Structure):
    """Mirror of `ScanConfig` (src/config.rs:79-88)."""

    _fields_ = [
        ("shortlist_cand", C.c_uint32), ("cs_tolerance", C.c_float),
        ("stratum4_weight", C.c_float), ("strata_depth", C.c_uint32),
        ("temporal_filter_enable", C.c_uint32), ("numa_sharding", C.c_uint32),
    ]


class ScanStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in
                ("blocks", "active_vecs", "after_prefix", "after_s1", "after_s4_budget", "pushed")]


class FixedPlan(C.Structure):
    _fields_ = [
        ("prefix_lut", (C.c_int32 * 16) * 64), ("s1_lut", (C.c_int32 * 32) * 26),
        ("s4_lut", (C.c_int32 * 32) * 13), ("prefix_shift", C.c_int32),
        ("s1_shift", C.c_int32), ("s4_shift", C.c_int32), ("pad", C.c_int32),
    ]


def build() -> str:
    """Compile the oracle library (g++) if it is missing or stale."""
    src = os.path.join(_HERE, "mrl_oracle.cpp")
    if (not os.path.exists(_LIB_PATH)) or os.path.getmtime(_LIB_PATH) < max(
            os.path.getmtime(src), os.path.getmtime(os.path.join(_HERE, "mrl_oracle.h"))):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(build())
        L = _lib
        L.ora_f32_to_f16.argtypes = [C.c_float]; L.ora_f32_to_f16.restype = C.c_uint16
        L.ora_f16_to_f32.argtypes = [C.c_uint16]; L.ora_f16_to_f32.restype = C.c_float
        L.ora_crc32.argtypes = [u8p, C.c_size_t]; L.ora_crc32.restype = C.c_uint32
        L.ora_fwht.argtypes = [f32p, C.c_int]
        L.ora_rotate_mid_band.argtypes = [f32p, f32p]
        L.ora_rotate_tail_fold.argtypes = [f32p, C.c_int, f32p]
        L.ora_tail_rademacher.argtypes = [C.c_uint64, C.c_uint64]; L.ora_tail_rademacher.restype = C.c_float
        L.ora_rademacher_diag.argtypes = [C.c_uint64, C.c_uint64]; L.ora_rademacher_diag.restype = C.c_float
        L.ora_rabitq_bit_scale.restype = C.c_float
        L.ora_tail_fold_bit_scale.restype = C.c_float
        L.ora_lloyd_max.argtypes = [C.c_int, f32p]
        L.ora_nearest_centroid.argtypes = [f32p, C.c_int, C.c_float]; L.ora_nearest_centroid.restype = C.c_int
        L.ora_eden_fit_prefix.argtypes = [f32p, C.c_uint64, C.c_int, f32p]
        L.ora_eden_fit_band.argtypes = [f32p, C.c_uint64, C.c_int, C.c_int, C.c_int, f32p]
        L.ora_eden_encode_slice.argtypes = [f32p, C.c_int, C.c_uint64, C.c_int, f32p, u8p,
                                            C.POINTER(C.c_float), C.POINTER(C.c_float)]
        L.ora_encode_block.argtypes = [f32p, C.c_int, C.c_int, u32p, u32p, C.c_int, C.c_void_p,
                                       C.c_uint64, C.c_void_p, C.c_uint64, u8p]
        L.ora_encode_block.restype = C.c_int
        L.ora_encode_corpus.argtypes = [f32p, C.c_uint64, C.c_int, C.c_uint32, C.c_int, C.c_void_p,
                                        C.c_uint64, C.c_void_p, C.c_uint64, C.c_int, u8p]
        L.ora_encode_corpus.restype = C.c_int
        L.ora_verify_crc.argtypes = [u8p]; L.ora_verify_crc.restype = C.c_int
        L.ora_plan_build.argtypes = [f32p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_uint64,
                                     C.c_void_p, C.c_uint64, C.POINTER(QueryPlan)]
        L.ora_plan_build.restype = C.c_int
        L.ora_scan_blocks.argtypes = [u8p, C.c_uint64, C.POINTER(QueryPlan), C.POINTER(ScanCfg),
                                      C.c_int, C.c_uint32, C.c_int, C.c_uint32, C.c_int,
                                      C.POINTER(ScanStats), u64p, f32p]
        L.ora_scan_blocks.restype = C.c_int
        L.ora_full_scores.argtypes = [u8p, C.c_uint64, C.POINTER(QueryPlan), C.POINTER(ScanCfg),
                                      C.c_int, C.c_uint32, C.c_int, C.c_uint32, f32p, u8p]
        L.ora_block_stages.argtypes = [u8p, C.POINTER(QueryPlan), C.POINTER(ScanCfg), C.c_float,
                                       u64p, f32p]
        L.ora_fixed_plan_build.argtypes = [C.POINTER(QueryPlan), C.POINTER(ScanCfg), C.POINTER(FixedPlan)]
        L.ora_fixed_scores.argtypes = [u8p, C.c_uint64, C.POINTER(QueryPlan), C.POINTER(FixedPlan),
                                       C.POINTER(ScanCfg), C.c_int, C.c_uint32, C.c_int, C.c_uint32,
                                       i32p, f32p, u8p]
        L.ora_device_layout.argtypes = [u8p, u8p, u32p]
        L.ora_synth_docs.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_int, C.c_int, f32p]
        L.ora_synth_queries.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_int,
                                        C.c_float, f32p, u64p]
        L.ora_topk_by_key.argtypes = [f32p, u8p, C.c_uint64, C.c_uint32, u64p, f32p]
        L.ora_topk_by_key.restype = C.c_int
        L.ora_dot.argtypes = [f32p, f32p, C.c_uint64]; L.ora_dot.restype = C.c_float
        L.ora_ring_search.argtypes = [f32p, C.c_uint64, C.c_int, f32p, C.c_uint32, u32p, f32p]
        L.ora_ring_search.restype = C.c_uint32
        L.ora_rerank_rows.argtypes = [f32p, C.c_int, f32p, u64p, C.c_uint64, u64p, f32p]
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------------------------------------
# Convenience wrappers (numpy in, numpy out)

def f32_to_f16(x: float) -> int:
    return lib().ora_f32_to_f16(float(x))


def f16_to_f32(h: int) -> float:
    return lib().ora_f16_to_f32(int(h))


def crc32(data: bytes | np.ndarray) -> int:
    a = np.frombuffer(bytes(data), dtype=np.uint8).copy() if not isinstance(data, np.ndarray) else data
    return lib().ora_crc32(np.ascontiguousarray(a, dtype=np.uint8), a.size)


def fwht(v: np.ndarray) -> np.ndarray:
    a = np.array(v, dtype=np.float32, copy=True)
    lib().ora_fwht(a, a.size)
    return a


def rotate_mid_band(mid: np.ndarray) -> np.ndarray:
    out = np.zeros(128, np.float32)
    lib().ora_rotate_mid_band(np.ascontiguousarray(mid, np.float32), out)
    return out


def rotate_tail_fold(vec: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(vec, np.float32)
    out = np.zeros(64, np.float32)
    lib().ora_rotate_tail_fold(v, v.size, out)
    return out


def lloyd_max(bits: int) -> np.ndarray:
    out = np.zeros(1 << bits, np.float32)
    lib().ora_lloyd_max(bits, out)
    return out


def eden_fit_prefix(rows: np.ndarray) -> np.ndarray:
    rows = np.ascontiguousarray(rows, np.float32)
    mean = np.zeros(64, np.float32)
    lib().ora_eden_fit_prefix(rows, rows.shape[0], rows.shape[1], mean)
    return mean


def eden_fit_band(rows: np.ndarray, start: int, width: int) -> np.ndarray:
    rows = np.ascontiguousarray(rows, np.float32)
    mean = np.zeros(width, np.float32)
    lib().ora_eden_fit_band(rows, rows.shape[0], rows.shape[1], start, width, mean)
    return mean


def encode_block(vecs, ts=None, src=None, prefix_codec=EDEN_PROD, eden_mean=None, eden_seed=1,
                 mid_mean=None, mid_seed=1) -> np.ndarray:
    vecs = np.ascontiguousarray(vecs, np.float32)
    n, dims = vecs.shape
    ts = np.ascontiguousarray(np.arange(n) if ts is None else ts, np.uint32)
    src = np.ascontiguousarray(np.full(n, 8) if src is None else src, np.uint32)
    em = None if eden_mean is None else np.ascontiguousarray(eden_mean, np.float32)
    mm = None if mid_mean is None else np.ascontiguousarray(mid_mean, np.float32)
    out = np.zeros(4096, np.uint8)
    rc = lib().ora_encode_block(vecs, n, dims, ts, src, prefix_codec, _ptr(em), eden_seed, _ptr(mm),
                                mid_seed, out)
    if rc:
        raise ValueError(f"ora_encode_block rc={rc}")
    return out


def encode_corpus(rows, prefix_codec=EDEN_PROD, eden_mean=None, eden_seed=1, mid_mean=None,
                  mid_seed=1, src=8, threads=None) -> np.ndarray:
    rows = np.ascontiguousarray(rows, np.float32)
    n, dims = rows.shape
    nb = (n + 63) // 64
    out = np.zeros(nb * 4096, np.uint8)
    em = None if eden_mean is None else np.ascontiguousarray(eden_mean, np.float32)
    mm = None if mid_mean is None else np.ascontiguousarray(mid_mean, np.float32)
    rc = lib().ora_encode_corpus(rows, n, dims, src, prefix_codec, _ptr(em), eden_seed, _ptr(mm),
                                 mid_seed, threads or os.cpu_count() or 1, out)
    if rc:
        raise ValueError(f"ora_encode_corpus rc={rc}")
    return out


def verify_crc(block: np.ndarray) -> bool:
    return bool(lib().ora_verify_crc(np.ascontiguousarray(block, np.uint8)))


def plan_build(q, prefix_codec=EDEN_PROD, mid_codec=RABITQ, eden_mean=None, eden_seed=1,
               mid_mean=None, mid_seed=1) -> QueryPlan:
    q = np.ascontiguousarray(q, np.float32)
    em = None if eden_mean is None else np.ascontiguousarray(eden_mean, np.float32)
    mm = None if mid_mean is None else np.ascontiguousarray(mid_mean, np.float32)
    p = QueryPlan()
    rc = lib().ora_plan_build(q, q.size, prefix_codec, mid_codec, _ptr(em), eden_seed, _ptr(mm),
                              mid_seed, C.byref(p))
    if rc:
        raise ValueError(f"ora_plan_build rc={rc}")
    return p


def scan_cfg(k=256, cs_tolerance=1.0, stratum4_weight=0.2, strata_depth=FULL_64B,
             temporal_filter_enable=False, numa_sharding=True) -> ScanCfg:
    return ScanCfg(k, cs_tolerance, stratum4_weight, strata_depth, int(temporal_filter_enable),
                   int(numa_sharding))


def _tr(time_lo, time_hi):
    return (0 if time_lo is None else 1, 0 if time_lo is None else time_lo,
            0 if time_hi is None else 1, 0 if time_hi is None else time_hi)


def scan_blocks(blocks: np.ndarray, plan: QueryPlan, cfg: ScanCfg, time_lo=None, time_hi=None,
                threads=None, stats: bool = False):
    blocks = np.ascontiguousarray(blocks, np.uint8)
    nb = blocks.size // 4096
    ids = np.zeros(cfg.shortlist_cand, np.uint64)
    sc = np.zeros(cfg.shortlist_cand, np.float32)
    st = ScanStats() if stats else None
    n = lib().ora_scan_blocks(blocks, nb, C.byref(plan), C.byref(cfg), *_tr(time_lo, time_hi),
                              threads or os.cpu_count() or 1, C.byref(st) if st else None, ids, sc)
    if stats:
        return ids[:n], sc[:n], st
    return ids[:n], sc[:n]


def full_scores(blocks, plan, cfg, time_lo=None, time_hi=None):
    blocks = np.ascontiguousarray(blocks, np.uint8)
    nb = blocks.size // 4096
    sc = np.zeros(nb * 64, np.float32)
    act = np.zeros(nb * 64, np.uint8)
    lib().ora_full_scores(blocks, nb, C.byref(plan), C.byref(cfg), *_tr(time_lo, time_hi), sc, act)
    return sc, act


def block_stages(block, plan, cfg, tau):
    masks = np.zeros(4, np.uint64)
    sc = np.zeros(64, np.float32)
    lib().ora_block_stages(np.ascontiguousarray(block, np.uint8), C.byref(plan), C.byref(cfg),
                           float(tau), masks, sc)
    return masks, sc


def fixed_plan_build(plan, cfg) -> FixedPlan:
    fp = FixedPlan()
    lib().ora_fixed_plan_build(C.byref(plan), C.byref(cfg), C.byref(fp))
    return fp


def fixed_scores(blocks, plan, fp, cfg, time_lo=None, time_hi=None):
    blocks = np.ascontiguousarray(blocks, np.uint8)
    nb = blocks.size // 4096
    parts = np.zeros(nb * 64 * 3, np.int32)
    sc = np.zeros(nb * 64, np.float32)
    act = np.zeros(nb * 64, np.uint8)
    lib().ora_fixed_scores(blocks, nb, C.byref(plan), C.byref(fp), C.byref(cfg),
                           *_tr(time_lo, time_hi), parts, sc, act)
    return parts.reshape(-1, 3), sc, act


def device_layout(block) -> tuple[np.ndarray, np.ndarray]:
    out = np.zeros(4096, np.uint8)
    ts2 = np.zeros(2, np.uint32)
    lib().ora_device_layout(np.ascontiguousarray(block, np.uint8), out, ts2)
    return out, ts2


def synth_docs(seed: int, n: int, dims: int, row0: int = 0, threads=None) -> np.ndarray:
    out = np.zeros((n, dims), np.float32)
    lib().ora_synth_docs(seed, row0, n, dims, threads or os.cpu_count() or 1, out)
    return out


def synth_queries(doc_seed, n_docs, q_seed, n_q, dims, sigma=0.1):
    out = np.zeros((n_q, dims), np.float32)
    pick = np.zeros(n_q, np.uint64)
    lib().ora_synth_queries(doc_seed, n_docs, q_seed, n_q, dims, sigma, out, pick)
    return out, pick


def topk_by_key(scores, active, k):
    ids = np.zeros(k, np.uint64)
    sc = np.zeros(k, np.float32)
    n = lib().ora_topk_by_key(np.ascontiguousarray(scores, np.float32),
                              np.ascontiguousarray(active, np.uint8), scores.size, k, ids, sc)
    return ids[:n], sc[:n]


def dot(a, b) -> np.float32:
    """dot / dot_768 of the reference (src/embed.rs:115-152)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return np.float32(lib().ora_dot(a, b, a.size))


def ring_search(pending, q, k):
    """RingBuffer::search_exact (src/ring.rs:109-119): (positions, scores) of the top k."""
    pending = np.ascontiguousarray(np.atleast_2d(pending), np.float32)
    q = np.ascontiguousarray(q, np.float32)
    n = pending.shape[0] if pending.size else 0
    pos = np.zeros(max(k, 1), np.uint32)
    sc = np.zeros(max(k, 1), np.float32)
    m = lib().ora_ring_search(pending, n, q.size, q, k, pos, sc)
    return pos[:m], sc[:m]


def rerank_rows(rows, q, cand):
    """QueryPipeline::rerank_exact_rows (src/pipeline.rs:157-169): (row ids, scores) sorted."""
    rows = np.ascontiguousarray(rows, np.float32)
    q = np.ascontiguousarray(q, np.float32)
    cand = np.ascontiguousarray(cand, np.uint64)
    out_r = np.zeros(max(cand.size, 1), np.uint64)
    out_s = np.zeros(max(cand.size, 1), np.float32)
    lib().ora_rerank_rows(rows, q.size, q, cand, cand.size, out_r, out_s)
    return out_r[:cand.size], out_s[:cand.size]
