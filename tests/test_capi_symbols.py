"""libmrl_b200.so loads without a GPU and exports every entry point include/mrl_cuda.h declares
(no compute calls here), and the C mirrors of the reference structs have the expected layout."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include")) if f.endswith(".h")]


def declared_symbols():
    names = set()
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(mrl_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("mrl_ctx_create", "mrl_segment_upload", "mrl_plan_build", "mrl_scan", "mrl_last_error",
                 "mrl_encode_blocks", "mrl_scan_device"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from mrl_b200 import _capi

    lib = _capi.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"missing exports: {missing}"
    # and the ctypes binding covers exactly the declared surface
    assert set(_capi.SIGNATURES) == set(declared_symbols())


def test_struct_layouts_match_oracle_mirror():
    import ora
    from mrl_b200._capi import QueryPlanC, ScanCfgC

    assert C.sizeof(QueryPlanC) == C.sizeof(ora.QueryPlan) == 5776
    for (a, _), (b, _) in zip(QueryPlanC._fields_, ora.QueryPlan._fields_):
        assert a == b
        assert getattr(QueryPlanC, a).offset == getattr(ora.QueryPlan, b).offset
    assert C.sizeof(ScanCfgC) == 28


def test_context_creation_fails_cleanly_without_gpu():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from mrl_b200 import _capi

    lib = _capi.load()
    ctx = C.c_void_p()
    assert lib.mrl_ctx_create(0, C.byref(ctx)) == _capi.MRL_ERR_CUDA
    assert not ctx.value
