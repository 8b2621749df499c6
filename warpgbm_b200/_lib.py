"""ctypes binding of libwgb_b200.so (declarations: include/warpgbm_b200.h).

Loading fails loudly: there is no CPU or PyTorch fallback for any operation
of this package.
"""
from __future__ import annotations

import ctypes
import os

from . import _build

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_f32 = ctypes.c_float


class WgbNode(ctypes.Structure):
    _fields_ = [
        ("sumq", _i64), ("count", _i64), ("lsumq", _i64), ("lcount", _i64),
        ("lstart", _i32), ("lcnt", _i32), ("slot", _i32), ("built", _i32),
        ("fpos", _i32), ("bin", _i32), ("child", _i32), ("leaf", _f32),
    ]


assert ctypes.sizeof(WgbNode) == 64

# numpy view of wgb_node records
NODE_DTYPE = [
    ("sumq", "<i8"), ("count", "<i8"), ("lsumq", "<i8"), ("lcount", "<i8"),
    ("lstart", "<i4"), ("lcnt", "<i4"), ("slot", "<i4"), ("built", "<i4"),
    ("fpos", "<i4"), ("bin", "<i4"), ("child", "<i4"), ("leaf", "<f4"),
]


class WgbWs(ctypes.Structure):
    _fields_ = [
        ("bins", _p), ("bins_fm", _p), ("era", _p), ("root_order", _p), ("y", _p), ("pred", _p),
        ("g", _p), ("qg", _p),
        ("feats", _p), ("kpos", _p), ("bins_sub", _p), ("kpos_sub", _p), ("S_sub", _i64),
        ("order", _p * 2), ("posnode", _p * 2), ("flags", _p),
        ("tile_cnt", _p), ("tile_off", _p), ("part", _p),
        ("hg", _p),
        ("chunks", _p), ("nchunks", _p),
        ("cand", _p), ("era_gain", _p),
        ("nodes", _p), ("nn", _p), ("nact", _p),
        ("maxabs", _p), ("shift", _p), ("rootsum", _p), ("sync", _p), ("part_hist", _p), ("part_hist_elems", _i64),
        ("era_sched", _p), ("era_ops", _p), ("crit_out", _p),
        ("hstage", _p), ("hstage_elems", _i64), ("win", _p),
        ("N", _i64), ("S", _i64), ("N_global", _i64),
        ("F", _i32), ("k", _i32), ("E", _i32), ("B", _i32), ("D", _i32), ("K", _i32),
        ("cls", _i32),
        ("chunk_cap", _i32), ("ntiles", _i32), ("ncand_blk", _i32),
        ("hist_ew", _i32), ("regular", _i32), ("era_nops", _i32), ("era_depth", _i32), ("ntree", _i32),
        ("nslice", _i32), ("slice", _i32), ("ks", _i32), ("win_words", _i32),
        ("mcw", _f32), ("eps", _f32), ("msg", _f32), ("lr", _f32), ("mean_factor", _f32),
    ]


_SIGS = {
    "wgb_last_error": ([], ctypes.c_char_p),
    "wgb_version": ([], _i32),
    "wgb_sizeof_node": ([], _i32),
    "wgb_sizeof_ws": ([], _i32),
    "wgb_compute_histogram3": ([_p, _i64, _i64, _p, _p, _i64, _p, _i32, _p, _p, _p, _i32, _i32,
                                _i32, _i32, _p], _i32),
    "wgb_compute_histogram3_noalloc": ([_p, _i64, _i64, _p, _p, _i64, _p, _i32, _p, _p, _p, _i32, _i32,
                                        _i32, _i32, _p], _i32),
    "wgb_compute_split": ([_p, _p, _i32, _i32, _i32, _f32, _f32, _f32, _p, _p, _i32, _p], _i32),
    "wgb_custom_cuda_binner": ([_p, _i64, _p, _i32, _p, _p], _i32),
    "wgb_predict_forest": ([_p, _i64, _i64, _p, _i32, _i32, _f32, _p, _p], _i32),
    "wgb_bin_matrix": ([_p, _i64, _i32, _i64, _p, _i32, _p, _i64, _p], _i32),
    "wgb_tree_residual": ([_p, _p], _i32),
    "wgb_tree_reset": ([_p, _p], _i32),
    "wgb_tree_quantize": ([_p, _p], _i32),
    "wgb_tree_subset": ([_p, _p], _i32),
    "wgb_tree_root": ([_p, _p], _i32),
    "wgb_level_hist": ([_p, _i32, _p], _i32),
    "wgb_built_slots": ([_i32, ctypes.POINTER(_i32), ctypes.POINTER(_i32)], None),
    "wgb_level_slots": ([_p, _i32, ctypes.POINTER(_i32), ctypes.POINTER(_i32)], None),
    "wgb_level_split": ([_p, _i32, _p], _i32),
    "wgb_level_pick": ([_p, _i32, _p], _i32),
    "wgb_era_mean_plan": ([_i32, _i64, _i32, _i32, _p, _p, _i64, ctypes.POINTER(_i32)], _i64),
    "wgb_level_partition": ([_p, _i32, _p], _i32),
    "wgb_bins_feature_major": ([_p, _p, _p], _i32),
    "wgb_hist_part_elems": ([_i64, _i32, _i32, _i64], _i64),
    "wgb_prebinned_ingest": ([_p, _i64, _i32, _i64, _p, _i64, _p, _p, _p], _i32),
    "wgb_tree_finish": ([_p, _p], _i32),
    "wgb_predict_packed": ([_p, _i64, _i64, _p, _p, _i32, _i32, _f32, _p, _p], _i32),
    "wgb_predict_heap": ([_p, _i64, _i64, _p, _i32, _i32, _i32, _f32, _p, _p], _i32),
    "wgb_h2d": ([_p, _p, _i64, _p], _i32),
    "wgb_grow_tree": ([_p, _p, _p], _i32),
    "wgb_decode_tree": ([_p, _i32, _i32, _i32, _p, _p, _i32, _p, _i32, _p, _p, _p, _i64], _i64),
    "wgb_comm_unique_id": ([_p], _i32),
    "wgb_comm_init": ([_i32, _i32, _p, ctypes.POINTER(_p)], _i32),
    "wgb_comm_destroy": ([_p], _i32),
    "wgb_comm_allreduce": ([_p, _p, _i64, _i32, _p], _i32),
    "wgb_comm_reduce_scatter": ([_p, _p, _p, _i64, _p], _i32),
    "wgb_comm_allgather_i32": ([_p, _p, _i64, _p], _i32),
    "wgb_quantile_edges": ([_p, _i64, _i32, _i64, _p, _i32, _p, _p, _p], _i32),
    "wgb_quantile_pass": ([_i32, _p, _i64, _i32, _i64, _i32, _p, _p, _p, _p, _p], _i32),
    "wgb_quantile_pick": ([_i32, _p, _p, _i64, _p, _i32, _i32, _p, _p, _p], _i32),
}

EXPORTED = tuple(_SIGS)

_LIB = None


def lib():
    """Load libwgb_b200.so, building it first if the sources are newer."""
    global _LIB
    if _LIB is None:
        path = _build.LIB
        if _build.needs_build():
            path = _build.build()
        if not os.path.exists(path):
            raise RuntimeError(f"warpgbm_b200 CUDA library missing: {path}")
        L = ctypes.CDLL(path)
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        if L.wgb_sizeof_node() != ctypes.sizeof(WgbNode) or L.wgb_sizeof_ws() != ctypes.sizeof(WgbWs):
            raise RuntimeError("libwgb_b200.so struct layout does not match warpgbm_b200/_lib.py")
        _LIB = L
    return _LIB


class WgbError(RuntimeError):
    pass


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib().wgb_last_error()
        msg = msg.decode() if msg else ""
        raise WgbError(f"{what or 'warpgbm_b200'} failed (status {rc}): {msg}")


# kernels each entry point launches (bench.py reports the count it saw)
_KERNELS = {
    "wgb_tree_reset": 1, "wgb_tree_residual": 1, "wgb_tree_subset": 1, "wgb_tree_quantize": 1, "wgb_tree_root": 1,
    "wgb_level_hist": 3, "wgb_level_split": 2, "wgb_level_pick": 1, "wgb_level_partition": 3,
    "wgb_tree_finish": 0,
    "wgb_grow_tree": 0, "wgb_bins_feature_major": 1, "wgb_prebinned_ingest": 1,
    "wgb_bin_matrix": 1, "wgb_predict_packed": 1, "wgb_predict_heap": 1, "wgb_quantile_edges": 2, "wgb_quantile_pass": 1, "wgb_quantile_pick": 1,
    "wgb_compute_histogram3": 6, "wgb_compute_histogram3_noalloc": 6,
    "wgb_compute_split": 1, "wgb_custom_cuda_binner": 1, "wgb_predict_forest": 1,
}
LAUNCHES = [0]


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
    LAUNCHES[0] += _KERNELS.get(name, 0)


def era_mean_plan(E: int, M: int, num_sms: int = 0, max_threads_per_sm: int = 0):
    """(sched int32 [E], ops uint8 [n], depth) of wgb_era_mean_plan."""
    import numpy as np
    depth = _i32()
    n = lib().wgb_era_mean_plan(E, M, num_sms, max_threads_per_sm, None, None, 0, ctypes.byref(depth))
    if n < 0:
        check(-n, "wgb_era_mean_plan")
    sched = np.empty(E, np.int32)
    ops = np.empty(max(n, 1), np.uint8)
    n2 = lib().wgb_era_mean_plan(E, M, num_sms, max_threads_per_sm, sched.ctypes.data, ops.ctypes.data, n,
                                 ctypes.byref(depth))
    if n2 != n:
        raise WgbError(f"wgb_era_mean_plan returned {n2}, expected {n}")
    return sched, ops[:n], depth.value


def built_slots(d: int, ws_ptr=None):
    """(first, count) of level d's built histogram slots (of the workspace's
    batch of trees when ws_ptr is given)."""
    a, b = _i32(), _i32()
    if ws_ptr is None:
        lib().wgb_built_slots(d, ctypes.byref(a), ctypes.byref(b))
    else:
        lib().wgb_level_slots(ws_ptr, d, ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value
