"""Drop-in replacement of the reference's ``warpgbm.cuda.node_kernel``.

Same four functions, argument order and in-place semantics as the pybind
module of warpgbm/cuda/node_kernel.cpp:41-46, executed by the sm_100a kernels
of libwgb_b200.so through its C ABI on the current torch CUDA stream.  Unlike
the reference, bad arguments raise instead of printf-ing a launch error.
"""
from __future__ import annotations

import torch

from . import _lib


def _stream():
    return ctypes_stream(torch.cuda.current_stream())


def ctypes_stream(s: torch.cuda.Stream):
    return s.cuda_stream


def _need(t: torch.Tensor, name: str, dtype, contiguous=True):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def compute_histogram3(bin_indices, residuals, sample_indices, feature_indices, era_indices,
                       grad_hist, hess_hist, num_bins, threads_per_block=256, rows_per_thread=1):
    """histogram_kernel.cu:63-104 -- accumulates into grad_hist/hess_hist [E,k,B]."""
    _need(bin_indices, "bin_indices", torch.int8)
    _need(residuals, "residuals", torch.float32)
    _need(sample_indices, "sample_indices", torch.int32)
    _need(feature_indices, "feature_indices", torch.int32)
    _need(era_indices, "era_indices", torch.int32)
    _need(grad_hist, "grad_hist", torch.float32)
    _need(hess_hist, "hess_hist", torch.float32)
    E, k, B = grad_hist.shape
    if tuple(hess_hist.shape) != (E, k, B) or k != feature_indices.numel() or B != num_bins:
        raise ValueError("histogram shapes do not match [num_eras, k, num_bins]")
    with torch.cuda.device(bin_indices.device):
        _lib.call("wgb_compute_histogram3", bin_indices.data_ptr(), bin_indices.shape[0],
                  bin_indices.shape[1], residuals.data_ptr(), sample_indices.data_ptr(),
                  sample_indices.numel(), feature_indices.data_ptr(), k, era_indices.data_ptr(),
                  grad_hist.data_ptr(), hess_hist.data_ptr(), E, int(num_bins),
                  int(threads_per_block), int(rows_per_thread), _stream())


def compute_split(G, H, min_split_gain, min_child_samples, eps, per_era_gain,
                  per_era_direction, threads=128):
    """best_split_kernel.cu:57-88 -- per-era gain and direction [E,k,B-1]."""
    for t, n in ((G, "G"), (H, "H"), (per_era_gain, "per_era_gain"),
                 (per_era_direction, "per_era_direction")):
        _need(t, n, torch.float32)
    E, k, B = G.shape
    if tuple(per_era_gain.shape) != (E, k, B - 1) or tuple(per_era_direction.shape) != (E, k, B - 1):
        raise ValueError("output shapes must be [E, k, B-1]")
    with torch.cuda.device(G.device):
        _lib.call("wgb_compute_split", G.data_ptr(), H.data_ptr(), E, k, B, float(min_split_gain),
                  float(min_child_samples), float(eps), per_era_gain.data_ptr(),
                  per_era_direction.data_ptr(), int(threads), _stream())


def custom_cuda_binner(X, bin_edges, bin_indices):
    """binner.cu:29-52 -- one column."""
    _need(X, "X", torch.float32)
    _need(bin_edges, "bin_edges", torch.float32)
    _need(bin_indices, "bin_indices", torch.int8)
    if bin_indices.numel() != X.numel():
        raise ValueError("bin_indices must have X's length")
    with torch.cuda.device(X.device):
        _lib.call("wgb_custom_cuda_binner", X.data_ptr(), X.numel(), bin_edges.data_ptr(),
                  bin_edges.numel(), bin_indices.data_ptr(), _stream())


def predict_forest(bin_indices, tree_tensor, learning_rate, out):
    """predict.cu:48-76 -- accumulates lr * leaf of every tree into out."""
    _need(bin_indices, "bin_indices", torch.int8)
    _need(tree_tensor, "tree_tensor", torch.float32)
    _need(out, "out", torch.float32)
    T, max_nodes, six = tree_tensor.shape
    if six != 6 or out.numel() != bin_indices.shape[0]:
        raise ValueError("tree_tensor must be [T, max_nodes, 6] and out [N]")
    with torch.cuda.device(out.device):
        _lib.call("wgb_predict_forest", bin_indices.data_ptr(), bin_indices.shape[0],
                  bin_indices.shape[1], tree_tensor.data_ptr(), T, max_nodes,
                  float(learning_rate), out.data_ptr(), _stream())
