"""C ABI checks that need no GPU: the library loads, exports every symbol
include/moe_b200.h declares, and rejects bad configurations with a status code
and a message (no exceptions across the boundary)."""
import ctypes as C
import os
import re

import pytest

from moe_ascend_opt_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "moe_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_[a-z0-9_]+)\s*\(", src)))


def test_header_symbols_exported():
    names = header_functions()
    assert len(names) >= 14
    lib = C.CDLL(capi.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) <= set(capi.SYMBOLS)


@pytest.mark.parametrize("E,H,I,qt,g,msg", [
    (8, 100, 64, 0, 128, "hidden_size must be multiple of 32"),
    (8, 128, 48, 1, 128, "intermediate_size must be multiple of 32"),
    (8, 128, 64, 7, 128, "quant_type"),
    (0, 128, 64, 0, 128, "positive"),
    (8, 256, 128, 2, 96, "group_size"),
])
def test_create_rejects_bad_config(E, H, I, qt, g, msg):
    cfg = capi.MoeConfig(E, H, I, qt, g, 0, 0)
    h = C.c_void_p()
    rc = capi.lib().moe_engine_create(C.byref(cfg), C.byref(h))
    assert rc == capi.MOE_ERR_INVALID
    assert msg in capi.lib().moe_last_error().decode()
    assert not h.value


def test_null_arguments():
    L = capi.lib()
    assert L.moe_engine_create(None, None) == capi.MOE_ERR_INVALID
    assert L.moe_engine_forward(None, None, None, None, None, 1, 8, 1, 1, None) == capi.MOE_ERR_INVALID
    assert L.moe_engine_destroy(None) == capi.MOE_OK
    assert L.moe_quantize_rows_q8_0(None, 1, 2, 33, None, None, None) == capi.MOE_ERR_INVALID
    assert L.moe_route_topk(None, 1, 8, 9, 1, None, None, None) == capi.MOE_ERR_INVALID


def test_error_is_thread_local():
    import threading
    L = capi.lib()
    cfg = capi.MoeConfig(8, 100, 64, 0, 128, 0, 0)
    L.moe_engine_create(C.byref(cfg), C.byref(C.c_void_p()))
    seen = {}

    def other():
        seen["msg"] = L.moe_last_error().decode()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] == ""
    assert "hidden_size" in L.moe_last_error().decode()
