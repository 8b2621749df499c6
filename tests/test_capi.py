"""The C ABI library loads, exports every entry point declared in
include/warpgbm_b200.h, and validates arguments -- without a GPU."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "warpgbm_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(wgb_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    fns = header_functions()
    for name in ["wgb_compute_histogram3", "wgb_compute_split", "wgb_custom_cuda_binner",
                 "wgb_predict_forest", "wgb_bin_matrix", "wgb_level_hist", "wgb_level_split",
                 "wgb_level_partition", "wgb_predict_packed"]:
        assert name in fns


def test_library_exports_every_declared_symbol():
    from warpgbm_b200 import _lib
    L = _lib.lib()
    raw = ctypes.CDLL(L._name)
    missing = [f for f in header_functions() if not hasattr(raw, f)]
    assert not missing, missing
    # and the Python binding knows every one of them
    assert set(header_functions()) <= set(_lib.EXPORTED)


def test_struct_layout_matches_binding():
    from warpgbm_b200 import _lib
    L = _lib.lib()
    assert L.wgb_sizeof_node() == ctypes.sizeof(_lib.WgbNode) == 64
    assert L.wgb_sizeof_ws() == ctypes.sizeof(_lib.WgbWs)


def test_argument_errors_are_reported_not_launched():
    """Validation happens before any CUDA call, so this runs on a CPU box."""
    from warpgbm_b200 import _lib
    L = _lib.lib()
    rc = L.wgb_compute_split(None, None, 1, 4, 8, 0.0, 20.0, 1e-6, None, None, 0, None)
    assert rc == 1 and b"threads" in L.wgb_last_error()
    rc = L.wgb_bin_matrix(None, 10, 4, 4, None, 1, None, 4, None)
    assert rc == 1 and b"num_bins" in L.wgb_last_error()
    rc = L.wgb_compute_histogram3(None, 0, 4, None, None, 0, None, 1, None, None, None, 1, 8,
                                  48, 4, None)
    assert rc == 1 and b"threads_per_block" in L.wgb_last_error()
    rc = L.wgb_compute_histogram3(None, 0, 4, None, None, 0, None, 1, None, None, None, 1, 8,
                                  64, 17, None)
    assert rc == 1 and b"rows_per_thread" in L.wgb_last_error()
    with pytest.raises(_lib.WgbError, match="num_bins"):
        _lib.call("wgb_bin_matrix", None, 10, 4, 4, None, 200, None, 4, None)
    # zero-sized work is a no-op
    assert L.wgb_custom_cuda_binner(None, 0, None, 0, None, None) == 0
    assert L.wgb_predict_forest(None, 0, 4, None, 0, 8, 0.1, None, None) == 0
