"""ctypes binding of libmrl_b200.so (the C ABI declared in include/mrl_cuda.h).

The library is the only compute path: importing this module loads it and raises immediately if
it is missing or was built without sm_100a support; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmrl_b200.so")

MRL_OK = 0
MRL_ERR_INVALID = -1
MRL_ERR_CUDA = -2
MRL_ERR_NOMEM = -3


class MrlError(RuntimeError):
    """Raised for every non-zero status of the C ABI (the reference panics in these cases)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"mrl status {code}: {msg}")
        self.code = code


class QueryPlanC(C.Structure):
    """C mirror of `QueryPlan` (src/scan.rs:19-71) = struct mrl_query_plan."""

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


class CodecDesc(C.Structure):
    _fields_ = [
        ("prefix_codec", C.c_uint32), ("mid_codec", C.c_uint32),
        ("eden_mean", C.POINTER(C.c_float)), ("eden_seed", C.c_uint64),
        ("mid_mean", C.POINTER(C.c_float)), ("mid_seed", C.c_uint64),
    ]


class ScanCfgC(C.Structure):
    _fields_ = [
        ("shortlist_cand", C.c_uint32), ("cs_tolerance", C.c_float),
        ("stratum4_weight", C.c_float), ("strata_depth", C.c_uint32),
        ("temporal_filter_enable", C.c_uint32), ("numa_sharding", C.c_uint32),
        ("mode", C.c_uint32),
    ]


# Every exported symbol of include/mrl_cuda.h with its ctypes signature.
_vp = C.c_void_p
_u32 = C.c_uint32
_u64 = C.c_uint64
_i = C.c_int
SIGNATURES = {
    "mrl_ctx_create": (_i, [_i, C.POINTER(_vp)]),
    "mrl_ctx_destroy": (None, [_vp]),
    "mrl_last_error": (C.c_char_p, [_vp]),
    "mrl_ctx_stream": (_vp, [_vp]),
    "mrl_ctx_set_stream": (_i, [_vp, _vp]),
    "mrl_segment_upload": (_i, [_vp, _vp, _u64, _u32, C.POINTER(_vp)]),
    "mrl_segment_append": (_i, [_vp, _vp, _vp]),
    "mrl_segment_free": (_i, [_vp, _vp]),
    "mrl_segment_blocks": (_u64, [_vp]),
    "mrl_segment_device_ptrs": (_i, [_vp, C.POINTER(_vp), C.POINTER(_vp)]),
    "mrl_segment_read_layout": (_i, [_vp, _vp, _vp, _vp]),
    "mrl_plan_build": (_i, [_vp, _vp, _u32, _u32, C.POINTER(CodecDesc), C.POINTER(_vp)]),
    "mrl_plans_alloc": (_i, [_vp, _u32, _u32, C.POINTER(_vp)]),
    "mrl_plan_build_device": (_i, [_vp, _vp, _u32, _u32, C.POINTER(CodecDesc), _vp]),
    "mrl_plan_rebuild": (_i, [_vp, _vp, _u32, _u32, C.POINTER(CodecDesc), _vp]),
    "mrl_plans_free": (_i, [_vp, _vp]),
    "mrl_plan_read": (_i, [_vp, _vp, _u32, C.POINTER(QueryPlanC)]),
    "mrl_scan": (_i, [_vp, _vp, _vp, C.POINTER(ScanCfgC), _vp, _vp, _vp, _vp, _vp]),
    "mrl_scan_device": (_i, [_vp, _vp, _vp, _u32, _u32, C.POINTER(ScanCfgC), _vp, _vp, _vp, _vp, _vp, _vp]),
    "mrl_scan_batch_device": (_i, [_vp, _vp, _vp, _u32, _u32, C.POINTER(ScanCfgC), _vp, _vp, _vp, _vp, _vp, _vp]),
    "mrl_query_scan_device": (_i, [_vp, _vp, _vp, _u32, _u32, C.POINTER(CodecDesc), _vp, C.POINTER(ScanCfgC), _vp, _vp,
                                   _vp, _vp, _vp, _vp]),
    "mrl_query_scan": (_i, [_vp, _vp, _vp, _u32, _u32, C.POINTER(CodecDesc), _vp, C.POINTER(ScanCfgC), _vp, _vp, _vp,
                            _vp, _vp]),
    "mrl_query_submit": (_i, [_vp, _vp, _vp, _u32, C.POINTER(CodecDesc), C.POINTER(ScanCfgC), _vp, _vp, _u32]),
    "mrl_query_collect": (_i, [_vp, _u32, _vp, _vp, _vp]),
    "mrl_exchange_create": (_i, [_vp, _u32, _u32, _u32, _vp, C.POINTER(_vp)]),
    "mrl_exchange_open": (_i, [_vp, _vp, _vp]),
    "mrl_exchange_destroy": (_i, [_vp, _vp]),
    "mrl_query_submit_exchange": (_i, [_vp, _vp, _vp, _u32, C.POINTER(CodecDesc), C.POINTER(ScanCfgC), _vp, _vp, _vp,
                                       _u32]),
    "mrl_query_scan_exchange": (_i, [_vp, _vp, _vp, _u32, C.POINTER(CodecDesc), _vp, C.POINTER(ScanCfgC), _vp, _vp,
                                     _vp, _vp, _vp, _vp, _vp]),
    "mrl_segment_load": (_i, [_vp, C.c_char_p, _u32, C.POINTER(_vp)]),
    "mrl_ring_search": (_i, [_vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "mrl_rerank_exact": (_i, [_vp, _vp, _vp, _u64, _u32, _vp, _u32, _vp, _vp]),
    "mrl_merge_topk": (_i, [_vp, _vp, _u32, _u32, _u32, _vp, _vp, _vp]),
    "mrl_pack_records": (_i, [_vp, _vp, _vp, _vp, _u32, _u32, _vp]),
    "mrl_merge_topk_batch": (_i, [_vp, _vp, _u32, _u32, _u32, _u32, _vp, _vp, _vp]),
    "mrl_ring_create": (_i, [_vp, _u32, _u32, C.POINTER(_vp)]),
    "mrl_ring_push": (_i, [_vp, _vp, _vp]),
    "mrl_ring_drain": (_i, [_vp, _vp, _u32]),
    "mrl_ring_push_device": (_i, [_vp, _vp, _vp, _u32]),
    "mrl_ring_search_batch": (_i, [_vp, _vp, _u32, _u32, _vp, _u32, _u32, _vp]),
    "mrl_segment_append_device": (_i, [_vp, _vp, _vp, _u64]),
    "mrl_ring_len": (_u32, [_vp]),
    "mrl_ring_rows": (_i, [_vp, C.POINTER(_vp)]),
    "mrl_ring_destroy": (_i, [_vp, _vp]),
    "mrl_engine_scan": (_i, [_vp, _vp, _vp, _u32, C.POINTER(CodecDesc), _vp, C.POINTER(ScanCfgC), _vp, _vp, _vp,
                             _vp, _vp, _vp, _vp]),
    "mrl_scan_device_static": (_i, [_vp, _vp, _vp, _u32, _u32, C.POINTER(ScanCfgC), _vp, _vp, _vp, _vp, _vp, _vp]),
    "mrl_debug_vector_scores": (_i, [_vp, _vp, _vp, _u32, C.POINTER(ScanCfgC), _vp, _vp, _vp, _vp, _vp]),
    "mrl_scan_blocks_stats": (_i, [_vp, _vp, _vp, _u32, C.POINTER(ScanCfgC), _vp, _vp, _vp, _vp, _vp, _vp]),
    "mrl_debug_score_bound": (_i, [_vp, _vp, _vp, _u32, C.POINTER(ScanCfgC), C.POINTER(C.c_float)]),
    "mrl_debug_control_words": (_i, [_vp, C.POINTER(_u32)]),
    "mrl_encode_blocks": (_i, [_vp, _vp, _u64, _u32, _vp, _vp, C.POINTER(CodecDesc), _vp]),
    "mrl_encode_device": (_i, [_vp, _vp, _u64, _u32, _u32, C.POINTER(CodecDesc), _vp, _u32, C.POINTER(_vp)]),
    "mrl_eden_fit_device": (_i, [_vp, _vp, _u64, _u32, _u32, _u32, _vp]),
    "mrl_synth_docs_device": (_i, [_vp, _u64, _u64, _u64, _u32, _vp]),
    "mrl_synth_queries_device": (_i, [_vp, _u64, _u64, _u64, _u64, _u32, C.c_float, _vp, _vp]),
    "mrl_scan_geometry": (_i, [_vp, _u32, C.POINTER(_u32), C.POINTER(_u32)]),
    "mrl_set_list_len": (_i, [_vp, _u32]),
    "mrl_set_scan_ctas": (_i, [_vp, _u32]),
    "mrl_set_batch_engine": (_i, [_vp, _u32]),
}

_lib = None


def load():
    """Load libmrl_b200.so; raise if it is absent (no fallback path exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C csrc` "
                              "(mrl-index-rust-vector_b200/csrc) or __graft_entry__.build()")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _lib = lib
    return _lib


def check(ctx, rc: int):
    if rc != MRL_OK:
        msg = load().mrl_last_error(ctx) if ctx else b"invalid argument"
        raise MrlError(rc, (msg or b"").decode(errors="replace"))
