"""CPU oracle for WarpGBM's tree-growing hot path.

TEST INFRASTRUCTURE ONLY.  This package checks the CUDA product in
``warpgbm_b200``; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may import it.  Nothing in ``warpgbm_b200``
imports it, and the product raises if its CUDA library is missing instead of
falling back here.

It restates quantverse/warpgbm v2.2.0 (``warpgbm/core.py`` and the four
kernels in ``warpgbm/cuda/``) on the CPU: the kernels in plain C
(``wgb_oracle.c``, loaded through ctypes), the host logic in numpy below.

Two modes:

``mode="reference"``
    fp32 histogram sums in sample order, fp32 sibling subtraction
    (core.py:636-643), leaf = torch mean of the residuals (core.py:599),
    era means as torch's CUDA ``mean`` adds them (cuda_era_mean: the
    reference runs on CUDA).  Pinned against fixtures produced by the
    reference's own ``core.py`` (tests/golden).

``mode="canonical"``
    What the CUDA product computes, so that it can be compared bit for bit:
    residuals quantised per tree to ``q = rint(g * 2^s)`` with
    ``s = 29 - frexp_exponent(max|g|)``; histograms are exact int64 sums;
    leaf = ``float(sum_q) * 2^-s * (1 / float(n))`` in fp32; era means as
    torch's CUDA ``mean`` adds them (cuda_era_mean); base prediction from an
    exact fixed-point sum of y.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_p = ctypes.c_void_p


def lib():
    """Load (building if needed) oracle/libwgb_oracle.so."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = os.path.join(_HERE, "libwgb_oracle.so")
    src = os.path.join(_HERE, "wgb_oracle.c")
    if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    L = ctypes.CDLL(path)
    sig = {
        "orc_bin_matrix": [_p, _i64, _i64, _i64, _p, _i32, _p, _i64],
        "orc_quantile_edges": [_p, _i64, _i64, _p, _i32, _p],
        "orc_quantile_edges_matrix": [_p, _i64, _i64, _i64, _p, _i32, _p],
        "orc_hist_ref": [_p, _i64, _p, _p, _i64, _p, _i32, _p, _i32, _i32, _p, _p],
        "orc_quant_shift": [_f32],
        "orc_quantize": [_p, _i64, _i32, _p],
        "orc_hist_q": [_p, _i64, _p, _p, _i64, _p, _i32, _p, _i32, _i32, _p, _p],
        "orc_hist_dequant": [_p, _p, _i64, _i32, _i32, _p, _p],
        "orc_split": [_p, _p, _i32, _i32, _i32, _f32, _f32, _p, _p],
        "orc_des_pick": [_p, _p, _i32, _i32, _i32, _f32, _i32, _f32],
        "orc_predict_flat": [_p, _i64, _i64, _p, _i32, _i32, _f32, _p],
        "orc_num_threads": [],
        "orc_set_num_threads": [_i32],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = None
    L.orc_quant_shift.restype = _i32
    L.orc_des_pick.restype = _i64
    L.orc_num_threads.restype = _i32
    _LIB = L
    return L


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# --------------------------------------------------------------------------
# kernel restatements (numpy in, numpy out)
# --------------------------------------------------------------------------

def linspace_q(num_bins: int) -> np.ndarray:
    """torch.linspace(0, 1, B+1, dtype=float32)[1:-1] (core.py:529-531).

    ATen's formula: step = 1/(steps-1); i < steps//2 -> step*i, else
    1 - step*(steps-1-i) with one fused multiply-add.  The float64 evaluation
    below is exact before the single rounding to float32."""
    steps = num_bins + 1
    step = np.float32(np.float32(1.0) / np.float32(steps - 1))
    half = steps // 2
    out = []
    for i in range(steps):
        if i < half:
            out.append(np.float32(step * np.float32(i)))
        else:
            out.append(np.float32(1.0 - float(step) * float(steps - 1 - i)))
    return np.array(out[1:-1], dtype=np.float32)


def quantile_edges(col: np.ndarray, q: np.ndarray) -> np.ndarray:
    """torch.quantile(col, q) on one float32 column (core.py:532-534)."""
    col = _c(col, np.float32)
    q = _c(q, np.float32)
    out = np.empty(len(q), np.float32)
    lib().orc_quantile_edges(_ptr(col), col.shape[0], 1, _ptr(q), len(q), _ptr(out))
    return out


def quantile_edges_matrix(X: np.ndarray, q: np.ndarray) -> np.ndarray:
    """quantile_edges of every column (OpenMP over columns), [F, len(q)]."""
    X = _c(X, np.float32)
    q = _c(q, np.float32)
    n, F = X.shape
    out = np.empty((F, len(q)), np.float32)
    lib().orc_quantile_edges_matrix(_ptr(X), n, F, F, _ptr(q), len(q), _ptr(out))
    return out


def bin_matrix(X: np.ndarray, edges: np.ndarray) -> np.ndarray:
    """binner.cu semantics for every column; edges [F, B-1]."""
    X = _c(X, np.float32)
    edges = _c(edges, np.float32)
    n, F = X.shape
    out = np.empty((n, F), np.int8)
    lib().orc_bin_matrix(_ptr(X), n, F, F, _ptr(edges), edges.shape[1], _ptr(out), F)
    return out


def hist_ref(bins, g, samples, feats, era, E, B):
    """histogram_kernel.cu semantics; returns fresh G, H float32 [E, k, B]."""
    bins = _c(bins, np.int8)
    g = _c(g, np.float32)
    samples = _c(samples, np.int32)
    feats = _c(feats, np.int32)
    era = _c(era, np.int32)
    k = len(feats)
    G = np.zeros((E, k, B), np.float32)
    H = np.zeros((E, k, B), np.float32)
    lib().orc_hist_ref(_ptr(bins), bins.shape[1], _ptr(g), _ptr(samples), len(samples),
                       _ptr(feats), k, _ptr(era), E, B, _ptr(G), _ptr(H))
    return G, H


def quant_shift(maxabs: float) -> int:
    return int(lib().orc_quant_shift(float(np.float32(maxabs))))


def quantize(g: np.ndarray, s: int) -> np.ndarray:
    g = _c(g, np.float32)
    q = np.empty(g.shape[0], np.int32)
    lib().orc_quantize(_ptr(g), g.shape[0], s, _ptr(q))
    return q


def hist_q(bins, q, samples, feats, era, E, B):
    """Canonical histogram: int64 sums / int32 counts, [E, k, B+1]
    (slot B collects negative bins)."""
    bins = _c(bins, np.int8)
    q = _c(q, np.int32)
    samples = _c(samples, np.int32)
    feats = _c(feats, np.int32)
    era = _c(era, np.int32)
    k = len(feats)
    G = np.zeros((E, k, B + 1), np.int64)
    C = np.zeros((E, k, B + 1), np.int32)
    lib().orc_hist_q(_ptr(bins), bins.shape[1], _ptr(q), _ptr(samples), len(samples),
                     _ptr(feats), k, _ptr(era), E, B, _ptr(G), _ptr(C))
    return G, C


def dequant(G, C, s):
    """[..., B+1] int sums -> float32 [..., B] G, H (canonical)."""
    B = G.shape[-1] - 1
    lead = G.shape[:-1]
    G2 = _c(G, np.int64).reshape(-1, B + 1)
    C2 = _c(C, np.int32).reshape(-1, B + 1)
    Gf = np.empty((G2.shape[0], B), np.float32)
    Hf = np.empty((G2.shape[0], B), np.float32)
    lib().orc_hist_dequant(_ptr(G2), _ptr(C2), G2.shape[0], B, s, _ptr(Gf), _ptr(Hf))
    return Gf.reshape(lead + (B,)), Hf.reshape(lead + (B,))


def split(G, H, mcw, eps):
    """best_split_kernel.cu semantics: per-era gain and direction [E,k,B-1]."""
    G = _c(G, np.float32)
    H = _c(H, np.float32)
    E, k, B = G.shape
    gain = np.empty((E, k, B - 1), np.float32)
    d = np.empty((E, k, B - 1), np.float32)
    lib().orc_split(_ptr(G), _ptr(H), E, k, B, float(np.float32(mcw)),
                    float(np.float32(eps)), _ptr(gain), _ptr(d))
    return gain, d


def cuda_mean_factor(E: int, k: int, nb: int) -> np.float32:
    """torch's CUDA mean multiplies the sum by
    float(num_outputs) / float(numel) (ATen mean_kernel_impl)."""
    return np.float32(np.float32(k * nb) / np.float32(E * k * nb))


def _cuda_mean_layout(E: int, M: int, num_sms: int, max_threads_per_sm: int):
    """(rows, ctas) of torch's CUDA reduce kernel for the mean over axis 0 of
    a contiguous fp32 [E, M] array (ATen/native/cuda/Reduce.cuh of torch
    2.11, ``setReduceConfig`` / ``set_block_dimension``): the eras are spread
    over ``rows`` block rows and ``ctas`` thread blocks (both 1 when a thread
    sums its output alone)."""
    vec = 4
    while M % vec:
        vec //= 2
    dim0 = M // vec
    mnt = 512 // vec

    def p2(n):
        return mnt if n >= mnt else 1 << (int(n).bit_length() - 1)

    bw = min(p2(dim0), 32)
    bh = min(p2(E), mnt // bw)
    bw = min(p2(dim0), mnt // bh)
    if not E >= min(bh * 16, 256):
        return 1, 1
    vpt = -(-E // bh)
    grid = -(-dim0 // bw)
    target = num_sms * (max_threads_per_sm // (bw * bh))
    ctas = 1
    if vpt >= 256 and grid <= target:
        ctas = max(min(-(-target // grid), -(-vpt // 16)), -(-vpt // 256))
    return bh, max(ctas, 1)


def cuda_era_mean(x: np.ndarray, num_sms: int = 148, max_threads_per_sm: int = 2048) -> np.ndarray:
    """Mean over axis 0 of a contiguous fp32 ``[E, ...]`` array in the order
    in which torch's CUDA reduction adds (the reference's
    ``per_era_gain.mean(dim=0)``, core.py:581-582), restated from the
    published ``ATen/native/cuda/Reduce.cuh`` of torch 2.11:

    * launch shape (``setReduceConfig`` / ``set_block_dimension``): outputs
      are vectorised by ``vec`` = the largest of 4, 2, 1 dividing the output
      count M; ``mnt = 512 / vec`` threads; block width and height are the
      powers of two ``bw = min(p2(M/vec), 32)``, ``bh = min(p2(E), mnt/bw)``,
      ``bw = min(p2(M/vec), mnt/bh)`` (``p2`` = largest power of two <= n,
      capped at ``mnt``); the eras are split over the ``bh`` rows of the
      block when ``E >= min(16 bh, 256)``, and also over ``ctas`` thread
      blocks when a row would still sum 256 eras or more and the output grid
      is small (``ctas = max(min(ceil(target / grid), ceil(vpt / 16)),
      ceil(vpt / 256))``, ``vpt = ceil(E / bh)``, ``target`` = SMs x blocks
      per SM);
    * per thread (``thread_reduce_impl``): thread (row y, block c) takes the
      eras e = y + bh*c (mod bh*ctas); its t-th era goes to accumulator
      ``t % 4``, each summed in era order from 0, then ``((a0 + a1) + a2) +
      a3``;
    * across the block rows (``block_y_reduce``): a halving tree,
      ``r[y] += r[y + off]`` for off = bh/2, ..., 1;
    * across blocks (``global_reduce``): row y of the last block adds the
      block results c = y, y + bh, ... in order from 0, then the halving
      tree again;
    * ``* factor`` with ``factor = float(M) / float(E * M)``.

    ``num_sms`` / ``max_threads_per_sm`` (a B200: 148, 2048) only decide the
    number of blocks.  A single output (M == 1) is reduced along another
    path (vectorised loads of the contiguous eras, warp shuffles), which is
    not restated: it raises."""
    x = np.ascontiguousarray(x, np.float32)
    E = x.shape[0]
    M = x.size // E
    if E < 1 or M < 2:
        raise NotImplementedError("a single output is reduced along another path")
    flat = x.reshape(E, M)
    Y, C = _cuda_mean_layout(E, M, num_sms, max_threads_per_sm)
    L = Y * C
    acc = np.zeros((L, 4, M), np.float32)
    for e in range(E):
        lane, t = e % L, e // L
        acc[lane, t % 4] = acc[lane, t % 4] + flat[e]
    r = ((acc[:, 0] + acc[:, 1]) + acc[:, 2]) + acc[:, 3]
    v = r.reshape(C, Y, M)                     # lane y + Y*c -> [c, y]

    def halve(a):                              # block_y_reduce over axis -2
        off = a.shape[-2] // 2
        while off > 0:
            a[..., :off, :] = a[..., :off, :] + a[..., off:2 * off, :]
            off //= 2
        return a[..., 0, :]

    vc = halve(v)                              # [C, M]
    if C > 1:
        u = np.zeros((Y, M), np.float32)
        for c in range(C):
            u[c % Y] = u[c % Y] + vc[c]
        res = halve(u)
    else:
        res = vc[0]
    factor = np.float32(np.float32(M) / np.float32(E * M))
    return (res * factor).astype(np.float32).reshape(x.shape[1:])


def des_pick(gain, d, msg, mean_mode):
    """core.py:577-594: flat index of the chosen [k, B-1] cell, or -1.

    mean_mode 1: the era means as torch's CUDA ``mean(dim=0)`` computes them
    (cuda_era_mean; the reference runs on CUDA); mean_mode 0: a sequential
    era sum divided by E (torch's CPU mean for the few eras of the golden
    fixtures).  The agreement |mean dir| is exact in any order (sums of
    -1/0/1 in fp32), times the same factor."""
    gain = _c(gain, np.float32)
    d = _c(d, np.float32)
    E, k, nb = gain.shape
    if E == 1 or mean_mode == 0 or k * nb < 2:
        factor = cuda_mean_factor(E, k, nb) if mean_mode == 1 else np.float32(1.0)
        return int(lib().orc_des_pick(_ptr(gain), _ptr(d), E, k, nb + 1,
                                      float(np.float32(msg)), mean_mode, float(factor)))
    crit = cuda_era_mean(gain).reshape(-1)
    factor = cuda_mean_factor(E, k, nb)
    agree = np.abs(d.reshape(E, -1).sum(axis=0, dtype=np.float64).astype(np.float32) * factor)
    mask = (agree == agree.max()) & (crit > np.float32(msg))
    if not mask.any():
        return -1
    return int(np.argmax(np.where(mask, crit, np.float32(-np.inf))))


def predict_flat(bins, forest, lr, out):
    """predict.cu semantics over flattened trees, summed in tree order."""
    bins = _c(bins, np.int8)
    forest = _c(forest, np.float32)
    assert out.dtype == np.float32 and out.flags.c_contiguous
    T, max_nodes, _ = forest.shape
    lib().orc_predict_flat(_ptr(bins), bins.shape[0], bins.shape[1], _ptr(forest), T,
                           max_nodes, float(np.float32(lr)), _ptr(out))
    return out


def canonical_mean(y: np.ndarray) -> np.float32:
    """Base prediction of the canonical mode: exact fixed-point sum of y.

    t = 62 - L - e with n < 2^L and max|y| < 2^e; sum of rint(y*2^t) in
    int64 is exact; mean = float32(float64(sum) * 2^-t / n)."""
    y = np.asarray(y, np.float32)
    n = y.shape[0]
    m = float(np.max(np.abs(y))) if n else 0.0
    if not (m > 0.0) or not math.isfinite(m):
        return np.float32(0.0) if m == 0.0 else np.float32(np.mean(y, dtype=np.float64))
    L = int(n).bit_length()
    e = math.frexp(m)[1]
    t = 62 - L - e
    qy = np.rint(y.astype(np.float64) * math.ldexp(1.0, t)).astype(np.int64)
    s = int(qy.sum())
    return np.float32(math.ldexp(float(s), -t) / float(n))


def canonical_leaf(sum_q: int, n: int, s: int) -> np.float32:
    """Leaf = float(sum_q) * 2^-s * (1/float(n)), each step an fp32 op."""
    # int64 -> float32 rounds once (C cast), the power-of-two scaling is exact
    sf = np.float32(np.float32(np.int64(sum_q)) * np.float32(math.ldexp(1.0, -s)))
    factor = np.float32(np.float32(1.0) / np.float32(n))
    return np.float32(sf * factor)


# --------------------------------------------------------------------------
# host logic (core.py) restated
# --------------------------------------------------------------------------

def flatten_tree(tree, max_nodes):
    """core.py:1215-1252: pre-order ids, rows [feat, bin, left, right,
    is_leaf, leaf_value], NaN-filled."""
    flat = np.full((max_nodes, 6), np.nan, np.float32)
    counter = [0]

    def walk(node):
        i = counter[0]
        counter[0] += 1
        if "leaf_value" in node:
            flat[i, 4] = 1.0
            flat[i, 5] = node["leaf_value"]
        else:
            flat[i, 0] = float(node["feature"])
            flat[i, 1] = float(node["bin"])
            flat[i, 2] = counter[0]
            walk(node["left"])
            flat[i, 3] = counter[0]
            walk(node["right"])
            flat[i, 4] = 0.0

    walk(tree)
    return flat


def _torch_mean_f32(x: np.ndarray) -> np.float32:
    import torch
    return np.float32(torch.from_numpy(np.ascontiguousarray(x, np.float32)).mean().item())


class OracleGBM:
    """CPU restatement of ``WarpGBM`` fit/predict (core.py:293-1030).

    Parameters mirror the reference constructor.  ``mode`` selects the
    reference or canonical arithmetic (module docstring).  ``feature_subsets``
    (list of int arrays, one per tree / round) replaces ``torch.randperm``
    when ``colsample_bytree < 1``, so the oracle can replay the subsets the
    run under test drew.  ``edges`` (float32 [F, B-1]) may be supplied to bin
    float input with externally computed quantile edges.
    """

    def __init__(self, objective="regression", num_bins=10, max_depth=3,
                 learning_rate=0.1, n_estimators=100, min_child_weight=20,
                 min_split_gain=0.0, L2_reg=1e-6, colsample_bytree=1.0,
                 mode="reference"):
        assert mode in ("reference", "canonical")
        self.objective = objective
        self.num_bins = num_bins
        self.max_depth = max_depth
        self.learning_rate = learning_rate
        self.n_estimators = n_estimators
        self.min_child_weight = min_child_weight
        self.min_split_gain = min_split_gain
        self.L2_reg = L2_reg
        self.colsample_bytree = colsample_bytree
        self.mode = mode

    # ---- preprocessing: core.py:487-541 --------------------------------
    def preprocess(self, X, era_id, edges=None):
        B = self.num_bins
        n, F = X.shape
        if np.issubdtype(X.dtype, np.integer) and np.all(X.max(axis=0) < B):
            bins = X.astype(np.int8)
            self.bin_edges = np.tile(np.arange(1, B, dtype=np.float32), (F, 1))
            self.prebinned = True
        else:
            if edges is None:
                q = linspace_q(B)
                Xf = X.astype(np.float32)
                edges = np.stack([quantile_edges(Xf[:, f], q) for f in range(F)])
            self.bin_edges = np.asarray(edges, np.float32)
            bins = bin_matrix(X.astype(np.float32), self.bin_edges)
            self.prebinned = False
        uniq, inv = np.unique(era_id, return_inverse=True)
        return bins, inv.astype(np.int32), uniq

    def bin_inference(self, X):
        """core.py:934-955."""
        B = self.num_bins
        if np.issubdtype(X.dtype, np.integer) and X.shape[1] == self.num_features \
                and np.all(X.max(axis=0) < B):
            return X.astype(np.int8)
        return bin_matrix(X.astype(np.float32), self.bin_edges)

    # ---- histogram / split per node -------------------------------------
    def _hist(self, rows):
        if self.mode == "reference":
            return hist_ref(self.bins, self.residual, rows, self.feats, self.era,
                            self.E, self.num_bins)
        Gq, Cq = hist_q(self.bins, self.qres, rows, self.feats, self.era, self.E,
                        self.num_bins)
        return Gq, Cq

    def _split_from_hist(self, hist):
        if self.mode == "reference":
            G, H = hist
        else:
            G, H = dequant(hist[0], hist[1], self.qshift)
        gain, d = split(G, H, self.min_child_weight, self.L2_reg)
        idx = des_pick(gain, d, self.min_split_gain, 1)
        return idx, gain

    def _leaf(self, rows):
        if self.mode == "reference":
            return _torch_mean_f32(self.residual[rows])
        return canonical_leaf(int(self.qres[rows].astype(np.int64).sum()), len(rows),
                              self.qshift)

    # ---- grow_tree: core.py:597-658 --------------------------------------
    def _grow(self, hist, rows, depth, col):
        lr = np.float32(self.learning_rate)
        if depth == self.max_depth:
            v = self._leaf(rows)
            self.pred[rows, col] += np.float32(lr * v)
            return {"leaf_value": float(v), "samples": int(len(rows))}
        idx, gain = self._split_from_hist(hist)
        if idx < 0:
            v = self._leaf(rows)
            self.pred[rows, col] += np.float32(lr * v)
            return {"leaf_value": float(v), "samples": int(len(rows))}
        nb = self.num_bins - 1
        lf, bb = idx // nb, idx % nb
        gfi = int(self.feats[lf])
        # core.py:624-627: per-era importance, fp32, depth-first order
        self.imp[:, gfi] += gain[:, lf, bb].astype(np.float32)
        mask = self.bins[rows, gfi] <= bb
        left, right = rows[mask], rows[~mask]
        if len(left) <= len(right):
            hl = self._hist(left)
            hr = tuple(p - c for p, c in zip(hist, hl))
        else:
            hr = self._hist(right)
            hl = tuple(p - c for p, c in zip(hist, hr))
        lc = self._grow(hl, left, depth + 1, col)
        rc = self._grow(hr, right, depth + 1, col)
        return {"feature": gfi, "bin": int(bb), "left": lc, "right": rc}

    def _tree(self, residual, col, feats):
        self.residual = np.ascontiguousarray(residual, np.float32)
        self.feats = np.asarray(feats, np.int32)
        if self.mode == "canonical":
            self.qshift = quant_shift(float(np.max(np.abs(self.residual))))
            self.qres = quantize(self.residual, self.qshift)
        rows = np.arange(self.num_samples, dtype=np.int32)
        return self._grow(self._hist(rows), rows, 0, col)

    def _subset(self, i):
        F = self.num_features
        if self.colsample_bytree < 1.0:
            return np.asarray(self.feature_subsets[i], np.int32)
        return np.arange(F, dtype=np.int32)

    # ---- fit: core.py:293-485, 692-818 -----------------------------------
    def fit(self, X, y, era_id=None, edges=None, feature_subsets=None,
            residual_hook=None):
        self.feature_subsets = feature_subsets
        n, F = X.shape
        self.num_samples, self.num_features = n, F
        if era_id is None:
            era_id = np.ones(n, dtype=np.int32)
        self.bins, self.era, self.unique_eras = self.preprocess(X, era_id, edges)
        self.E = len(self.unique_eras)
        self.imp = np.zeros((self.E, F), np.float32)
        if self.objective == "regression":
            return self._fit_regression(np.asarray(y))
        return self._fit_classification(np.asarray(y), residual_hook)

    def _fit_regression(self, y):
        y = y.astype(np.float32)
        if self.mode == "reference":
            self.base_prediction = float(_torch_mean_f32(y))
        else:
            self.base_prediction = float(canonical_mean(y))
        self.pred = np.zeros((self.num_samples, 1), np.float32) + np.float32(self.base_prediction)
        self.forest = []
        for i in range(self.n_estimators):
            res = y - self.pred[:, 0]
            self.forest.append(self._tree(res, 0, self._subset(i)))
        self.per_era_feature_importance_ = self.imp
        self.feature_importance_ = self.imp.sum(axis=0)
        return self

    def _fit_classification(self, y, residual_hook):
        """core.py:417-485, 746-818 (no eval set)."""
        import torch
        from sklearn.preprocessing import LabelEncoder
        self.label_encoder = LabelEncoder()
        yenc = self.label_encoder.fit_transform(y)
        self.classes_ = self.label_encoder.classes_
        K = self.num_classes = len(self.classes_)
        yt = torch.from_numpy(yenc).to(torch.int32)
        Fm = torch.zeros((self.num_samples, K), dtype=torch.float32)
        for k in range(K):
            prior = (yt == k).float().mean()
            if prior > 0:
                Fm[:, k] = torch.log(prior + 1e-10)
        self.pred = Fm.numpy().copy()
        self.forest = []
        for i in range(self.n_estimators):
            logits = torch.from_numpy(self.pred)
            ex = torch.exp(logits - torch.max(logits, dim=1, keepdim=True)[0])
            probs = ex / torch.sum(ex, dim=1, keepdim=True)
            onehot = torch.zeros(self.num_samples, K)
            onehot[torch.arange(self.num_samples), yt.long()] = 1.0
            grads = (probs - onehot).numpy()
            feats = self._subset(i)
            trees = []
            for k in range(K):
                res = -grads[:, k]
                if residual_hook is not None:
                    res = residual_hook(i, k, res)
                trees.append(self._tree(res, k, feats))
            self.forest.append(trees)
        self.per_era_feature_importance_ = self.imp
        self.feature_importance_ = self.imp.sum(axis=0)
        return self

    # ---- predict: core.py:917-1030 ---------------------------------------
    def flat_forest(self):
        mx = 2 ** (self.max_depth + 1)
        if self.objective == "regression":
            return np.stack([flatten_tree(t, mx) for t in self.forest if t])
        return np.stack([flatten_tree(t, mx) for r in self.forest for t in r])

    def predict_binned(self, bins):
        out = np.zeros(bins.shape[0], np.float32) + np.float32(self.base_prediction)
        return predict_flat(bins, self.flat_forest(), self.learning_rate, out)

    def predict(self, X):
        if self.objective == "regression":
            return self.predict_binned(self.bin_inference(X))
        p = self.predict_proba(X)
        return self.label_encoder.inverse_transform(np.argmax(p, axis=1))

    def predict_proba(self, X):
        import torch
        bins = self.bin_inference(X)
        n, K = bins.shape[0], self.num_classes
        Fm = torch.zeros((n, K), dtype=torch.float32)
        for k in range(K):
            prior_k = (self.classes_ == self.classes_[k]).sum() / len(self.classes_)
            if prior_k > 0:
                Fm[:, k] = torch.log(torch.tensor(prior_k + 1e-10))
        mx = 2 ** (self.max_depth + 1)
        F = Fm.numpy().copy()
        for rnd in self.forest:
            for k, t in enumerate(rnd):
                tp = np.zeros(n, np.float32)
                predict_flat(bins, flatten_tree(t, mx)[None], self.learning_rate, tp)
                F[:, k] += tp
        Ft = torch.from_numpy(F)
        ex = torch.exp(Ft - torch.max(Ft, dim=1, keepdim=True)[0])
        return (ex / torch.sum(ex, dim=1, keepdim=True)).numpy()
