"""``WarpGBM`` -- the reference's sklearn-style estimator on the B200 engine.

Host mirror of quantverse/warpgbm v2.2.0 ``warpgbm/core.py``: same
constructor, ``fit`` / ``predict`` / ``predict_proba`` / importance / save /
load API and the same Directional Era Splitting semantics.  The compute runs
in libwgb_b200.so (include/warpgbm_b200.h):

* binning: one ``wgb_bin_matrix`` launch over the whole matrix (edges from
  ``torch.quantile`` on the device, exactly the op core.py:529-534 calls);
* trees: level-wise, without host synchronisation inside a tree --
  histogram of every node of a level in one launch, split search, on-device
  partition and leaf updates;
* prediction: ``wgb_predict_heap`` (trees as complete binary trees in
  shared memory, depth <= 12) or ``wgb_predict_packed``, all trees (and all
  classes) in one launch, summed in tree order.

Histograms are exact integer sums of residuals quantised per tree to a
power-of-two grid (q = rint(g * 2^s), s = 29 - exponent(max|g|)), so every
decision is independent of summation order, run to run and across GPU
counts.  With ``distributed=True`` inside an initialised torch.distributed
process group, every rank passes its own row shard to ``fit``; histograms
and the few global scalars are summed over ranks (NCCL over NVLink), and all
ranks grow identical trees.
"""
from __future__ import annotations

import math
import pickle
from typing import List, Optional

import numpy as np
import torch
from sklearn.base import BaseEstimator, RegressorMixin
from sklearn.preprocessing import LabelEncoder

from . import _lib
from .metrics import accuracy_torch, log_loss_torch, rmsle_torch, softmax

HIST_R = 2048          # rows per histogram chunk (csrc/wgb_common.cuh)
PART_TILE = 2048       # positions per partition tile
SPLIT_WARPS = 8           # features per single-era split block (csrc/wgb_common.cuh)


def split_era_features(B: int) -> int:
    """Features per block of the era split search (csrc/wgb_engine.cu)."""
    return 32 if B - 1 <= 32 else 8


def _round_up(x, m):
    return (x + m - 1) // m * m


def bins_stride(F: int) -> int:
    """Row stride of the device bin matrix: features padded to 32 bytes."""
    return _round_up(max(F, 1), 32)


def cuda_mean_factor(E: int, k: int, nb: int) -> float:
    """torch's CUDA mean = sum * float(outputs)/float(numel) (ATen mean kernel)."""
    return float(np.float32(np.float32(k * nb) / np.float32(E * k * nb)))


# ---------------------------------------------------------------------------
# multi-GPU plumbing
# ---------------------------------------------------------------------------

class _Comm:
    """torch.distributed collectives for the row-sharded fit (no-ops when
    running on one rank)."""

    def __init__(self, enabled: bool):
        import torch.distributed as dist
        self.dist = dist
        self.on = bool(enabled) and dist.is_available() and dist.is_initialized() \
            and dist.get_world_size() > 1
        self.world = dist.get_world_size() if self.on else 1
        self.rank = dist.get_rank() if self.on else 0
        # a gloo group moves CUDA tensors through host memory (NCCL uses them in place)
        self.host_staging = self.on and dist.get_backend() == "gloo"

    def _inplace(self, t, op):
        if self.host_staging and t.is_cuda:
            h = t.cpu()
            op(h)
            t.copy_(h)
        else:
            op(t)
        return t

    def max_(self, t):
        if self.on:
            self._inplace(t, lambda x: self.dist.all_reduce(x, op=self.dist.ReduceOp.MAX))
        return t

    def sum_(self, t):
        if self.on:
            self._inplace(t, lambda x: self.dist.all_reduce(x, op=self.dist.ReduceOp.SUM))
        return t

    def reduce_scatter_(self, out, inp):
        """out = this rank's block of the element-wise sum over ranks of inp
        ([world * out.numel()], block r to rank r).  gloo: an all-reduce of
        the whole buffer, then the block (the same integer sums)."""
        if not self.on:
            out.copy_(inp[: out.numel()])
        elif self.host_staging:
            h = inp.cpu()
            self.dist.all_reduce(h, op=self.dist.ReduceOp.SUM)
            m = out.numel()
            out.copy_(h[self.rank * m:(self.rank + 1) * m])
        else:
            self.dist.reduce_scatter_tensor(out, inp)
        return out

    def all_gather_inplace_(self, buf, count):
        """buf[r*count:(r+1)*count] of every rank r to all ranks."""
        if self.on:
            mine = buf[self.rank * count:(self.rank + 1) * count].clone()
            if self.host_staging:
                outs = list(buf[: self.world * count].view(self.world, count).unbind(0))
                self.all_gather(outs, mine)
            else:
                self.dist.all_gather_into_tensor(buf[: self.world * count], mine)
        return buf

    def bcast_(self, t, src=0):
        if self.on:
            self._inplace(t, lambda x: self.dist.broadcast(x, src))
        return t

    def all_gather(self, outs, t):
        if self.host_staging and t.is_cuda:
            ho = [torch.empty_like(o, device="cpu") for o in outs]
            self.dist.all_gather(ho, t.cpu())
            for o, h in zip(outs, ho):
                o.copy_(h)
        else:
            self.dist.all_gather(outs, t)

    def all_to_all_single(self, out, inp, out_splits, in_splits):
        if self.host_staging and inp.is_cuda:
            ho = torch.empty_like(out, device="cpu")
            self.dist.all_to_all_single(ho, inp.cpu(), output_split_sizes=out_splits,
                                        input_split_sizes=in_splits)
            out.copy_(ho)
        else:
            self.dist.all_to_all_single(out, inp, output_split_sizes=out_splits,
                                        input_split_sizes=in_splits)

    def gather_var(self, t: torch.Tensor) -> List[torch.Tensor]:
        """all_gather of 1-D tensors of different lengths."""
        if not self.on:
            return [t]
        n = torch.tensor([t.numel()], dtype=torch.int64, device=t.device)
        ns = [torch.zeros_like(n) for _ in range(self.world)]
        self.all_gather(ns, n)
        ns = [int(x.item()) for x in ns]
        m = max(ns)
        pad = torch.zeros(m, dtype=t.dtype, device=t.device)
        pad[: t.numel()] = t
        outs = [torch.empty_like(pad) for _ in range(self.world)]
        self.all_gather(outs, pad)
        return [o[:c] for o, c in zip(outs, ns)]


_NATIVE_COMMS = {}


def native_comm(comm: _Comm, dev):
    """The library's own NCCL communicator over the ranks of `comm` (cached
    per process group), which wgb_grow_tree uses to sum each level's
    histograms on the engine's stream; None for one rank or a gloo group."""
    if not comm.on or comm.host_staging:
        return None
    import atexit
    import ctypes
    pg = comm.dist.group.WORLD
    key = (id(pg), comm.rank, comm.world, str(dev))
    h = _NATIVE_COMMS.get(key)
    if h is None:
        uid = torch.zeros(128, dtype=torch.uint8, device=dev)
        if comm.rank == 0:
            host = np.zeros(128, np.uint8)
            _lib.call("wgb_comm_unique_id", host.ctypes.data)
            uid.copy_(torch.from_numpy(host))
        comm.bcast_(uid)
        ids = np.ascontiguousarray(uid.cpu().numpy())
        h = ctypes.c_void_p()
        _lib.call("wgb_comm_init", comm.rank, comm.world, ids.ctypes.data, ctypes.byref(h))
        _NATIVE_COMMS[key] = h
        atexit.register(lambda hh=h: _lib.lib().wgb_comm_destroy(hh))
    return h


def fused_partition(ws) -> bool:
    """The engine's choice for a workspace (wgb_engine.cu fused_partition):
    one-era fits partition each level in one launch (k_partition)."""
    return ws.E == 1


def level_launches(D: int, E: int, fused: bool = True, sliced: bool = False) -> int:
    """Kernels one tree (or one batch of trees) launches in wgb_grow_tree."""
    n = 4                                            # reset, residual, quantize, root
    for d in range(D):
        n += (5 if d == 0 else 3) if E == 1 else (4 if d == 0 else 2)   # zero, histogram (+ chunk plan, root cells)
        n += 3 if d == 0 else 2                      # split (+ root totals), final
        n += 1 if sliced else 0                      # pick
        n += 1 if fused else 3                       # partition, or flags, offsets, scatter
    return n


def global_unique_eras(era: torch.Tensor, comm: _Comm):
    """torch.unique(era, return_inverse=True) over the union of all ranks'
    eras (core.py:540): sorted unique ids and the dense id of each local row."""
    local = torch.unique(era)
    uniq = torch.unique(torch.cat(comm.gather_var(local)))
    inv = torch.searchsorted(uniq, era).to(torch.int32)
    return uniq, inv


def exact_mean(y: torch.Tensor, comm: _Comm) -> float:
    """Base prediction: mean of y from an exact fixed-point sum, identical at
    every GPU count.  t = 62 - L - e (n < 2^L, max|y| < 2^e);
    mean = float32(float64(sum rint(y * 2^t)) * 2^-t / n)."""
    n = y.numel()
    if comm.on:
        nt = torch.tensor([n], dtype=torch.int64, device=y.device)
        comm.sum_(nt)
        n = int(nt.item())
    m = torch.zeros(1, dtype=torch.float32, device=y.device)
    if y.numel():
        m[0] = y.abs().max()
    comm.max_(m)
    m = float(m.item())
    if n == 0:
        raise ValueError("cannot fit on zero rows")
    if not math.isfinite(m):
        raise ValueError("y contains NaN or infinite values")
    if m == 0.0:
        return 0.0
    L = n.bit_length()
    e = math.frexp(m)[1]
    t = 62 - L - e
    q = torch.round(y.double() * math.ldexp(1.0, t)).to(torch.int64).sum().reshape(1)
    comm.sum_(q)
    return float(np.float32(math.ldexp(float(int(q.item())), -t) / float(n)))


def exchange_columns(Xd: torch.Tensor, comm: _Comm):
    """Row shards in, column slices out: rank r receives every rank's rows
    (in rank order) of columns [r*per, (r+1)*per), per = ceil(F / world)
    (padding columns are zero).  One all_to_all."""
    n, F = Xd.shape
    W = comm.world
    per = (F + W - 1) // W
    Xp = torch.zeros((n, per * W), dtype=Xd.dtype, device=Xd.device)
    Xp[:, :F] = Xd
    send = Xp.reshape(n, W, per).permute(1, 0, 2).contiguous().reshape(-1, per)
    ns = comm.gather_var(torch.tensor([n], dtype=torch.int64, device=Xd.device))
    counts = [int(c.item()) for c in ns]
    recv = torch.empty((sum(counts), per), dtype=Xd.dtype, device=Xd.device)
    comm.all_to_all_single(recv, send, counts, [n] * W)
    return recv, per


def sharded_quantile_edges(Xd: torch.Tensor, q: torch.Tensor, comm: _Comm) -> torch.Tensor:
    """Quantile edges [F, B-1] of every column of the row-sharded float
    matrix, bit-identical to torch.quantile over the full column
    (core.py:529-534): up to 32 quantiles by a radix select over the ranks'
    summed digit histograms (_sharded_select); more by exchanging columns so
    each rank holds complete columns of a feature slice, then all-gathering
    the edges."""
    F = Xd.shape[1]
    if not comm.on:
        return _quantile_columns(Xd, q)
    if q.numel() <= QS_MAXQ:
        return _sharded_select(Xd, q, comm)
    cols, per = exchange_columns(Xd, comm)
    mine = _quantile_columns(cols, q)                      # [per, B-1]
    outs = [torch.empty_like(mine) for _ in range(comm.world)]
    comm.all_gather(outs, mine)
    return torch.cat(outs, 0)[:F].contiguous()


QS_MAXQ, QS_H0, QS_HCOL, QS_STATE = 32, 4096, 64 * 256, 2 * 64 + 1  # wgb_quantile_pass / _pick sizes


def _sharded_select(Xd: torch.Tensor, q: torch.Tensor, comm: _Comm, chunk_elems: int = 1 << 28):
    """Quantile edges [F, B-1] of the row-sharded float matrix without moving
    rows: the radix select of wgb_quantile_edges one digit pass at a time --
    every rank histograms the digit of its own rows (wgb_quantile_pass), one
    int32 sum over the ranks per pass, and every rank resolves the same
    digits from the sums (wgb_quantile_pick).  Bit-identical to
    torch.quantile over the concatenated column (core.py:529-534)."""
    n, F = Xd.shape
    dev = Xd.device
    ng = int(comm.sum_(torch.tensor([n], dtype=torch.int64, device=dev)).item())
    if ng > (1 << 24):
        raise ValueError("quantile() input tensor is too large")  # torch's own limit
    nq = q.numel()
    Xd = Xd.contiguous()
    qd = q.contiguous()
    out = torch.empty((F, nq), dtype=torch.float32, device=dev)
    step = max(1, min(F, chunk_elems // max(n + 3, 1)))
    ld = (n + 3) // 4 * 4
    XT = torch.empty(max(ld * step, 4), dtype=torch.float32, device=dev)
    hist = torch.empty(step * QS_HCOL, dtype=torch.int32, device=dev)
    state = torch.empty(step * QS_STATE, dtype=torch.int32, device=dev)
    nanf = torch.empty(step, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    for c0 in range(0, F, step):
        m = min(F, c0 + step) - c0
        for p in range(4):
            _lib.call("wgb_quantile_pass", p, Xd.data_ptr() + 4 * c0, n, m, F, nq, XT.data_ptr(),
                      state.data_ptr(), hist.data_ptr(), nanf.data_ptr(), st)
            comm.sum_(hist[: m * (QS_H0 if p == 0 else QS_HCOL)])
            if p == 0:
                comm.sum_(nanf[:m])
            _lib.call("wgb_quantile_pick", p, hist.data_ptr(), nanf.data_ptr(), ng, qd.data_ptr(), nq, m,
                      state.data_ptr(), out[c0:c0 + m].data_ptr(), st)
    return out


def _quantile_columns(Xd: torch.Tensor, q: torch.Tensor, chunk_elems: int = 1 << 28):
    """Edges [F, B-1] = torch.quantile(X[:, f], q) for every column, bit for
    bit, by wgb_quantile_edges (radix selection, no sort), in column chunks of
    at most chunk_elems elements of column-major scratch."""
    n, F = Xd.shape
    if n > (1 << 24):
        raise ValueError("quantile() input tensor is too large")  # torch's own limit
    Xd = Xd.contiguous()
    out = torch.empty((F, q.numel()), dtype=torch.float32, device=Xd.device)
    step = max(1, min(F, chunk_elems // max(n + 3, 1)))
    ld = (n + 3) // 4 * 4                                  # 16-byte aligned columns
    XT = torch.empty(ld * step, dtype=torch.float32, device=Xd.device)
    qd = q.contiguous()
    st = torch.cuda.current_stream().cuda_stream
    for c0 in range(0, F, step):
        c1 = min(F, c0 + step)
        _lib.call("wgb_quantile_edges", Xd.data_ptr() + 4 * c0, n, c1 - c0, F, qd.data_ptr(),
                  q.numel(), XT.data_ptr(), out[c0:c1].data_ptr(), st)
    return out


_NP2T = {np.dtype(np.float32): torch.float32, np.dtype(np.int8): torch.int8,
         np.dtype(np.int32): torch.int32, np.dtype(np.int64): torch.int64,
         np.dtype(np.int16): torch.int16, np.dtype(np.uint8): torch.uint8,
         np.dtype(np.float64): torch.float64}


def _to_dev(a, dev, dtype=None):
    """numpy array or tensor -> contiguous tensor on dev.  Large host arrays
    go through wgb_h2d (pinned staging, parallel host copies overlapped with
    the DMA) instead of the driver's single pageable staging buffer."""
    if isinstance(a, np.ndarray) and a.nbytes >= (32 << 20):
        tdt = dtype if dtype is not None else _NP2T.get(a.dtype)
        if tdt is not None:
            ndt = np.dtype(str(tdt).replace("torch.", ""))
            src = np.ascontiguousarray(a, dtype=ndt)
            out = torch.empty(src.shape, dtype=tdt, device=dev)
            with torch.cuda.device(dev):
                _lib.call("wgb_h2d", out.data_ptr(), src.ctypes.data, src.nbytes,
                          torch.cuda.current_stream().cuda_stream)
            return out
    if torch.is_tensor(a):
        t = a
    else:
        t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None and t.dtype != dtype and t.device.type == "cpu" and t.element_size() != \
            torch.empty((), dtype=dtype).element_size():
        t = t.to(dtype)
    t = t.to(dev, non_blocking=False)
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


# ---------------------------------------------------------------------------
# forest packing
# ---------------------------------------------------------------------------

def pack_trees(trees) -> (np.ndarray, np.ndarray):
    """Pre-order packing for wgb_predict_packed: internal node
    (feature, bin | right_id << 8), leaf (-1, float bits)."""
    nodes, offs = [], [0]
    for tree in trees:
        buf = []

        def walk(nd):
            i = len(buf)
            buf.append(None)
            if "leaf_value" in nd:
                bits = np.array([nd["leaf_value"]], np.float32).view(np.int32)[0]
                buf[i] = (-1, int(bits))
            else:
                walk(nd["left"])
                right = len(buf)
                walk(nd["right"])
                buf[i] = (int(nd["feature"]), (int(nd["bin"]) & 0xFF) | (right << 8))
        walk(tree)
        nodes.extend(buf)
        offs.append(len(nodes))
    arr = np.array(nodes, np.int32).reshape(-1, 2) if nodes else np.zeros((0, 2), np.int32)
    return arr, np.array(offs, np.int32)


def compact_tree(nodes, gains, feats, D, E, ntree=1, root=0):
    """One tree's level-packed node records -> pre-order arrays, vectorised
    per level (no per-node Python).  `nodes` holds a batch of `ntree` trees
    grown together (level d = ntree << d records; tree t's root is node t of
    level 0); `root` picks the tree.  Returns (packed [n,2] int32 in the
    wgb_predict_packed format, leaf values [n] f32, samples [n] int64,
    split pre-order ids, split global features, split per-era gains [s, E]).
    Only nodes reachable from the root are real (the record buffer keeps
    stale entries of earlier trees)."""
    fpos_all = nodes["fpos"].astype(np.int64)
    child_all = nodes["child"].astype(np.int64)
    base = [ntree * ((1 << d) - 1) for d in range(D + 1)]
    real = [np.full(1, root, np.int64)]                  # level-local ids of real nodes
    split = []                                           # per level: bool mask over real
    for d in range(D + 1):
        r = real[d]
        sp = (fpos_all[base[d] + r] >= 0) if d < D else np.zeros(r.shape, bool)
        split.append(sp)
        if d < D:
            c = child_all[base[d] + r[sp]]
            real.append(np.stack([c, c + 1], 1).reshape(-1))
    # subtree sizes bottom-up (indexed by level-local id)
    size = [None] * (D + 1)
    for d in range(D, -1, -1):
        r = real[d]
        sz = np.ones(r.shape, np.int64)
        if d < D and split[d].any():
            c = child_all[base[d] + r[split[d]]]
            sz[split[d]] += size[d + 1][c] + size[d + 1][c + 1]
        full = np.zeros((ntree << d), np.int64)
        full[r] = sz
        size[d] = full
    n = int(size[0][root])
    pre = [None] * (D + 1)
    pre[0] = np.zeros(ntree, np.int64)
    packed = np.zeros((n, 2), np.int32)
    leaf = np.zeros(n, np.float32)
    samples = np.zeros(n, np.int64)
    sp_pre, sp_feat, sp_gain = [], [], []
    leaf_bits = np.ascontiguousarray(nodes["leaf"]).view(np.int32)
    for d in range(D + 1):
        r = real[d]
        full_pre = pre[d]
        pr = full_pre[r]
        g = base[d] + r
        lf = ~split[d]
        packed[pr[lf], 0] = -1
        packed[pr[lf], 1] = leaf_bits[g[lf]]
        leaf[pr[lf]] = nodes["leaf"][g[lf]]
        samples[pr[lf]] = nodes["count"][g[lf]]
        if d < D:
            nxt = np.zeros((ntree << (d + 1)), np.int64)
            if split[d].any():
                ps, gs = pr[split[d]], g[split[d]]
                c = child_all[gs]
                nxt[c] = ps + 1
                nxt[c + 1] = ps + 1 + size[d + 1][c]
                gfi = feats[fpos_all[gs]].astype(np.int64)
                packed[ps, 0] = gfi
                packed[ps, 1] = (nodes["bin"][gs].astype(np.int64) & 0xFF) | (nxt[c + 1] << 8)
                sp_pre.append(ps)
                sp_feat.append(gfi)
                sp_gain.append(gains.reshape(-1, E)[gs])
            pre[d + 1] = nxt
    if sp_pre:
        sp_pre = np.concatenate(sp_pre)
        order = np.argsort(sp_pre, kind="stable")
        sp_pre, sp_feat = sp_pre[order], np.concatenate(sp_feat)[order]
        sp_gain = np.concatenate(sp_gain)[order]
    else:
        sp_pre = sp_feat = np.zeros(0, np.int64)
        sp_gain = np.zeros((0, E), np.float32)
    return packed, leaf, samples, sp_pre, sp_feat, sp_gain


HEAP_DMAX = 12          # deepest forest the heap predictor takes (csrc/wgb_ops.cu)
HEAP_PASS = 127 << 16   # pass-through slot: feature 0, split bin 127 (every row goes left)


def heap_forest(parts, D):
    """Pre-order packed trees (pack_trees / compact_tree format) -> the heap
    layout of wgb_predict_heap: uint32 [T, 2^(D+1)], slot i's children
    2i+1 / 2i+2, internal slot = feature | split bin << 16, the value of the
    leaf reached at depth-D slot h in word h + 1, leaves above depth D as
    pass-through chains to their leftmost depth-D descendant.  Built level
    by level over all trees at once.  Returns None if a tree is deeper than
    D or uses a feature index >= 2^16."""
    T = len(parts)
    W = 2 << D
    H = np.zeros((T, W), np.uint32)
    H[:, : (1 << D) - 1] = HEAP_PASS
    if T == 0:
        return H
    sizes = np.array([len(p) for p in parts], np.int64)
    offs = np.zeros(T + 1, np.int64)
    offs[1:] = np.cumsum(sizes)
    allp = np.concatenate(parts).astype(np.int64)
    tid = np.arange(T, dtype=np.int64)
    slot = np.zeros(T, np.int64)
    pid = offs[:-1].copy()
    for d in range(D + 1):
        if tid.size == 0:
            break
        feat, w = allp[pid, 0], allp[pid, 1]
        leaf = feat < 0
        if leaf.any():
            # value at the leftmost depth-D descendant of this slot (word h + 1)
            h = (slot[leaf] + 1) * (1 << (D - d)) - 1
            H[tid[leaf], h + 1] = (w[leaf] & 0xFFFFFFFF).astype(np.uint32)
        inner = ~leaf
        if not inner.any():
            break
        if d == D or int(feat[inner].max()) >= (1 << 16):
            return None
        ti, si, fi, wi = tid[inner], slot[inner], feat[inner], w[inner]
        H[ti, si] = (fi | ((wi & 0xFF) << 16)).astype(np.uint32)
        left, right = pid[inner] + 1, offs[ti] + (wi >> 8)
        tid = np.concatenate([ti, ti])
        slot = np.concatenate([2 * si + 1, 2 * si + 2])
        pid = np.concatenate([left, right])
    return H


def tree_dict(packed, leaf, samples):
    """Reference nested-dict tree from compact pre-order arrays."""
    f = packed[:, 0].tolist()
    w = packed[:, 1].tolist()
    lv = leaf.tolist()
    sm = samples.tolist()

    def build(i):
        if f[i] < 0:
            return {"leaf_value": lv[i], "samples": sm[i]}
        return {"feature": f[i], "bin": w[i] & 0xFF, "left": build(i + 1), "right": build(w[i] >> 8)}
    return build(0)


class WarpGBM(BaseEstimator, RegressorMixin):
    def __init__(
        self,
        objective="regression",
        num_bins=10,
        max_depth=3,
        learning_rate=0.1,
        n_estimators=100,
        min_child_weight=20,
        min_split_gain=0.0,
        threads_per_block=64,
        rows_per_thread=4,
        L2_reg=1e-6,
        device="cuda",
        colsample_bytree=1.0,
        random_state=None,
        warm_start=False,
        distributed=False,
    ):
        self._validate_hyperparams(
            objective=objective, num_bins=num_bins, max_depth=max_depth,
            learning_rate=learning_rate, n_estimators=n_estimators,
            min_child_weight=min_child_weight, min_split_gain=min_split_gain,
            threads_per_block=threads_per_block, rows_per_thread=rows_per_thread,
            L2_reg=L2_reg, colsample_bytree=colsample_bytree,
        )
        self.objective = objective
        self.num_bins = num_bins
        self.max_depth = max_depth
        self.learning_rate = learning_rate
        self.n_estimators = n_estimators
        self.min_child_weight = min_child_weight
        self.min_split_gain = min_split_gain
        self.threads_per_block = threads_per_block
        self.rows_per_thread = rows_per_thread
        self.L2_reg = L2_reg
        self.device = device
        self.colsample_bytree = colsample_bytree
        self.random_state = random_state
        self.warm_start = warm_start
        self.distributed = distributed
        self.forest = [{} for _ in range(self.n_estimators)]
        self.bin_edges = None
        self.base_prediction = None
        self.unique_eras = None
        self.num_classes = None
        self.classes_ = None
        self.num_features = None
        self.num_samples = None
        self.label_encoder = None
        self.feature_importance_ = None
        self.per_era_feature_importance_ = None
        self.training_loss = []
        self.eval_loss = []
        self._is_fitted = False
        self._trees_trained = 0
        self._packed = None

    # ------------------------------------------------------------------
    # forest: nested-dict trees (the reference's format), built on first
    # access from the compact arrays that fit() and predict use
    # ------------------------------------------------------------------
    @property
    def forest(self):
        lazy = self.__dict__.get("_lazy")
        if lazy:
            f = self.__dict__["_forest"]
            for (i, c) in sorted(lazy):
                t = tree_dict(*self._compact[(i, c)][:3])
                if isinstance(f[i], list):
                    f[i][c] = t
                else:
                    f[i] = t
            lazy.clear()
        return self.__dict__.get("_forest")

    @forest.setter
    def forest(self, v):
        self.__dict__["_forest"] = v
        self.__dict__["_lazy"] = set()
        self.__dict__["_compact"] = {}

    # ------------------------------------------------------------------
    # validation (core.py:83-143, 216-291)
    # ------------------------------------------------------------------
    def _validate_hyperparams(self, **kw):
        if kw["objective"] not in ["regression", "multiclass", "binary"]:
            raise ValueError(
                f"objective must be 'regression', 'binary', or 'multiclass', got {kw['objective']}.")
        for p in ["num_bins", "max_depth", "n_estimators", "min_child_weight",
                  "threads_per_block", "rows_per_thread"]:
            if not isinstance(kw[p], int):
                raise TypeError(f"{p} must be an integer, got {type(kw[p])}.")
        for p in ["learning_rate", "min_split_gain", "L2_reg", "colsample_bytree"]:
            if not isinstance(kw[p], (float, int)):
                raise TypeError(f"{p} must be a float, got {type(kw[p])}.")
        if not (2 <= kw["num_bins"] <= 127):
            raise ValueError("num_bins must be between 2 and 127 inclusive.")
        if kw["max_depth"] < 1:
            raise ValueError("max_depth must be at least 1.")
        if not (0.0 < kw["learning_rate"] <= 1.0):
            raise ValueError("learning_rate must be in (0.0, 1.0].")
        if kw["n_estimators"] <= 0:
            raise ValueError("n_estimators must be positive.")
        if kw["min_child_weight"] < 1:
            raise ValueError("min_child_weight must be a positive integer.")
        if kw["min_split_gain"] < 0:
            raise ValueError("min_split_gain must be non-negative.")
        if kw["threads_per_block"] <= 0 or kw["threads_per_block"] % 32 != 0:
            raise ValueError("threads_per_block should be a positive multiple of 32 (warp size).")
        if not (1 <= kw["rows_per_thread"] <= 16):
            raise ValueError("rows_per_thread must be positive between 1 and 16 inclusive.")
        if kw["L2_reg"] < 0:
            raise ValueError("L2_reg must be non-negative.")
        if kw["colsample_bytree"] <= 0 or kw["colsample_bytree"] > 1:
            raise ValueError(
                f"Invalid colsample_bytree: {kw['colsample_bytree']}. Must be a float value > 0 and <= 1.")

    def validate_fit_params(self, X, y, era_id, X_eval, y_eval, eval_every_n_trees,
                            early_stopping_rounds, eval_metric):
        # numpy arrays as in the reference; CUDA tensors are also accepted
        # (data already resident on the device skips the host->device copy)
        arr = (np.ndarray, torch.Tensor)
        if not isinstance(X, arr) or not isinstance(y, arr):
            raise TypeError("X and y must be numpy arrays.")
        if X.ndim != 2:
            raise ValueError(f"X must be 2-dimensional, got shape {X.shape}")
        if y.ndim != 1:
            raise ValueError(f"y must be 1-dimensional, got shape {y.shape}")
        if X.shape[0] != y.shape[0]:
            raise ValueError(
                f"X and y must have the same number of rows. Got {X.shape[0]} and {y.shape[0]}.")
        if era_id is not None:
            if not isinstance(era_id, arr):
                raise TypeError("era_id must be a numpy array.")
            if era_id.ndim != 1:
                raise ValueError(f"era_id must be 1-dimensional, got shape {era_id.shape}")
            if len(era_id) != len(y):
                raise ValueError(
                    f"era_id must have same length as y. Got {len(era_id)} and {len(y)}.")
        if any(a is not None for a in (X_eval, y_eval, eval_every_n_trees)):
            if X_eval is None or y_eval is None or eval_every_n_trees is None:
                raise ValueError(
                    "If using eval set, X_eval, y_eval, and eval_every_n_trees must all be defined.")
            if not isinstance(X_eval, arr) or not isinstance(y_eval, arr):
                raise TypeError("X_eval and y_eval must be numpy arrays.")
            if X_eval.ndim != 2:
                raise ValueError(f"X_eval must be 2-dimensional, got shape {X_eval.shape}")
            if y_eval.ndim != 1:
                raise ValueError(f"y_eval must be 1-dimensional, got shape {y_eval.shape}")
            if X_eval.shape[0] != y_eval.shape[0]:
                raise ValueError(
                    f"X_eval and y_eval must have same number of rows. Got {X_eval.shape[0]} and {y_eval.shape[0]}.")
            if not isinstance(eval_every_n_trees, int) or eval_every_n_trees <= 0:
                raise ValueError(
                    f"eval_every_n_trees must be a positive integer, got {eval_every_n_trees}.")
            if early_stopping_rounds is not None:
                if not isinstance(early_stopping_rounds, int) or early_stopping_rounds <= 0:
                    raise ValueError(
                        f"early_stopping_rounds must be a positive integer, got {early_stopping_rounds}.")
            else:
                early_stopping_rounds = self.n_estimators + 1
            valid = ["mse", "corr", "rmsle", "logloss", "accuracy"]
            if eval_metric not in valid:
                raise ValueError(f"Invalid eval_metric: {eval_metric}. Choose from {valid}.")
        return early_stopping_rounds

    # ------------------------------------------------------------------
    # fit (core.py:293-485)
    # ------------------------------------------------------------------
    def fit(self, X, y, era_id=None, X_eval=None, y_eval=None, eval_every_n_trees=None,
            early_stopping_rounds=None, eval_metric="mse"):
        early_stopping_rounds = self.validate_fit_params(
            X, y, era_id, X_eval, y_eval, eval_every_n_trees, early_stopping_rounds, eval_metric)
        self._comm = _Comm(self.distributed)
        if self.random_state is not None:
            torch.manual_seed(self.random_state)
            np.random.seed(self.random_state)
            if torch.cuda.is_available():
                torch.cuda.manual_seed(self.random_state)
                torch.cuda.manual_seed_all(self.random_state)
        if not self.warm_start or not self._is_fitted:
            self._is_fitted = False
            self._trees_trained = 0
            self.forest = [{} for _ in range(self.n_estimators)] if self.objective == "regression" else []
            self.training_loss = []
            self.eval_loss = []
            self._packed = None
        else:
            if X.shape[1] != self.num_features:
                raise ValueError(
                    f"X has {X.shape[1]} features, but model was trained with {self.num_features} features.")
            if self._trees_trained >= self.n_estimators:
                print(f"Model already has {self._trees_trained} trees (n_estimators={self.n_estimators}). "
                      "No additional training needed.")
                return self
        if era_id is None and self._comm.on:
            # every rank takes part in the era exchange (a single rank with no
            # era ids has one era and needs none: _fit)
            era_id = np.ones(X.shape[0], dtype="int32")
        if self.objective in ("multiclass", "binary") and torch.is_tensor(y):
            y = y.cpu().numpy()
        self._dev = torch.device(self.device if str(self.device).startswith("cuda") else "cuda")
        if self._dev.index is None:
            self._dev = torch.device("cuda", torch.cuda.current_device())
        _lib.lib()  # fail loudly before any work if the CUDA library is missing
        with torch.cuda.device(self._dev):
            if self.objective in ("multiclass", "binary"):
                if not self.warm_start or not self._is_fitted:
                    self.label_encoder = LabelEncoder()
                    y_enc = self.label_encoder.fit_transform(y)
                    self.classes_ = self.label_encoder.classes_
                    self.num_classes = len(self.classes_)
                else:
                    y_enc = self.label_encoder.transform(y)
                if self.objective == "binary" and self.num_classes != 2:
                    raise ValueError(f"binary objective requires exactly 2 classes, got {self.num_classes}")
                if self.objective == "multiclass" and self.num_classes < 2:
                    raise ValueError(f"multiclass objective requires at least 2 classes, got {self.num_classes}")
                return self._fit(X, y_enc, era_id, X_eval, y_eval, eval_every_n_trees,
                                 early_stopping_rounds, eval_metric, classification=True)
            return self._fit(X, y, era_id, X_eval, y_eval, eval_every_n_trees,
                             early_stopping_rounds, eval_metric, classification=False)

    # ------------------------------------------------------------------
    def _upload_bins(self, X_np, fit: bool):
        """core.py:487-541 / 934-955: pre-binned integer input is copied,
        float input is binned with quantile edges (computed at fit)."""
        dev = self._dev
        B = self.num_bins
        n, F = X_np.shape
        if torch.is_tensor(X_np):
            is_int = not X_np.is_floating_point()
        else:
            is_int = np.issubdtype(X_np.dtype, np.integer)
        prebinned_ok = fit or F == self.num_features
        if not fit and F != self.num_features:
            # core.py:902-915 bins columns 0..num_features-1 of the input with
            # the stored edges: extra columns are ignored, missing ones raise
            # numpy's IndexError
            nf = self.num_features
            if F < nf:
                raise IndexError(f"index {F} is out of bounds for axis 1 with size {F}")
            X_np = X_np[:, :nf]
            F = nf
        S = bins_stride(F)
        if is_int and prebinned_ok:
            Xi = _to_dev(X_np, dev)
            if Xi.dtype == torch.int8:
                # one pass: padded copy, column maxima, global min / max
                bins = torch.empty((n, S), dtype=torch.int8, device=dev)
                colmax = torch.empty(F, dtype=torch.int32, device=dev)
                minmax = torch.empty(2, dtype=torch.int32, device=dev)
                _lib.call("wgb_prebinned_ingest", Xi.data_ptr(), n, F, F, bins.data_ptr(), S,
                          colmax.data_ptr(), minmax.data_ptr(), torch.cuda.current_stream().cuda_stream)
                mx = colmax.to(torch.int64)
                if fit:
                    self._comm.max_(mx)
                if bool((mx < B).all().item()):
                    print("Detected pre-binned integer input — skipping quantile binning." if fit
                          else "Detected pre-binned input at predict-time — skipping binning.")
                    if fit:
                        self.bin_edges = torch.arange(1, B, dtype=torch.float32, device=dev).repeat(F, 1)
                        mn = minmax[0:1].to(torch.int64)
                        mxb = minmax[1:2].to(torch.int64)
                        self._comm.max_(mxb)
                        mn = -self._comm.max_(-mn)
                        self._bins_regular = bool(mn.item() >= 0 and mxb.item() < B)
                    return bins, True
                del bins
                return self._upload_float(Xi.to(torch.float32), fit)
            mx = torch.full((F,), -(2 ** 62), dtype=torch.int64, device=dev)
            if n:
                mx = Xi.amax(dim=0).to(torch.int64)
            if fit:
                self._comm.max_(mx)
            if bool((mx < B).all().item()):
                print("Detected pre-binned integer input — skipping quantile binning." if fit
                      else "Detected pre-binned input at predict-time — skipping binning.")
                bins = torch.zeros((n, S), dtype=torch.int8, device=dev)
                bins[:, :F] = Xi.to(torch.int8)
                if fit:
                    self.bin_edges = torch.arange(1, B, dtype=torch.float32, device=dev).repeat(F, 1)
                    # regular = every stored bin in [0, B) (negative or wrapped
                    # pre-binned values take the kernel's slower checked path)
                    mn = torch.zeros(1, dtype=torch.int64, device=dev)
                    mxb = torch.zeros(1, dtype=torch.int64, device=dev)
                    if n:
                        mn[0] = bins[:, :F].amin()
                        mxb[0] = bins[:, :F].amax()
                    self._comm.max_(mxb)
                    mn = -self._comm.max_(-mn)
                    self._bins_regular = bool(mn.item() >= 0 and mxb.item() < B)
                return bins, True
            Xd = Xi.to(torch.float32)
        else:
            Xd = _to_dev(X_np, dev, torch.float32)
        return self._upload_float(Xd, fit)

    def _upload_float(self, Xd, fit: bool):
        """Quantile edges (at fit) and binning of a float32 device matrix."""
        dev, B = self._dev, self.num_bins
        n, F = Xd.shape
        S = bins_stride(F)
        if fit:
            print("quantile binning.")
            self._bins_regular = True  # binner output is always in [0, B)
            q = torch.linspace(0, 1, B + 1, device=dev, dtype=torch.float32)[1:-1]
            self.bin_edges = sharded_quantile_edges(Xd, q, self._comm)
        if self.bin_edges.shape[0] < F:
            raise ValueError(f"{F} columns to bin with edges of {self.bin_edges.shape[0]} features")
        bins = torch.empty((n, S), dtype=torch.int8, device=dev)
        _lib.call("wgb_bin_matrix", Xd.data_ptr(), n, F, F, self.bin_edges.data_ptr(), B,
                  bins.data_ptr(), S, torch.cuda.current_stream().cuda_stream)
        return bins, False

    def _alloc_ws(self, N, F, k, E, K, ntree=1, nslice=1, slice_=0):
        """Device workspace for growing `ntree` trees together (one per class
        in a multiclass round: a level's node set spans the batch).  With
        nslice > 1 ranks the fit is feature-sliced: this rank keeps the
        histograms of ks = ceil(k / nslice) positions and a staging buffer
        for one level's local histograms of all positions."""
        dev = self._dev
        B, D = self.num_bins, self.max_depth
        S = bins_stride(F)
        T = ntree
        NP = T * N                      # level-0 positions: tree t's rows at [tN, (t+1)N)
        nslots = T << (D - 1)
        ks = (k + nslice - 1) // nslice if nslice > 1 else k
        se = E * ks * (B + 1)
        P = 2 * se + 2                  # int64 per slot: sums, counts, root sum, spare
        stage_slots = T * max(1, 1 << max(D - 2, 0))  # most built slots of one level
        stage_elems = stage_slots * nslice * P if nslice > 1 else 0
        win_words = (8 + E + 1) & ~1    # even: every record's int64 totals stay 8-byte aligned
        hist_bytes = (nslots * P + stage_elems) * 8
        free, _ = torch.cuda.mem_get_info(dev)
        if hist_bytes > 0.6 * free:
            raise MemoryError(
                f"level-wise histograms need {hist_bytes / 2**30:.1f} GiB "
                f"({nslots} slots x {E} eras x {k} features x {B + 1} bins); "
                f"only {free / 2**30:.1f} GiB free -- reduce max_depth or features")
        i32 = dict(dtype=torch.int32, device=dev)
        t = {}
        t["order0"] = torch.empty(max(NP, 1), **i32)
        t["order1"] = torch.empty(max(NP, 1), **i32)
        t["posnode0"] = torch.empty(max(NP, 1), **i32)
        t["posnode1"] = torch.empty(max(NP, 1), **i32)
        t["flags"] = torch.empty(max(NP, 1) + 16, dtype=torch.uint8, device=dev)  # word reads past the end
        ntiles = max(1, (NP + PART_TILE - 1) // PART_TILE)
        t["tile_cnt"] = torch.empty(ntiles, **i32)
        t["tile_off"] = torch.empty(ntiles + 1, **i32)
        t["part"] = torch.empty((max(nslots, 1), 4), **i32)
        t["hg"] = torch.empty(nslots * P, dtype=torch.int64, device=dev)
        chunk_cap = (NP + HIST_R - 1) // HIST_R + nslots
        t["chunks"] = torch.empty((max(chunk_cap, 1), 4), **i32)
        # per-chunk histogram words: single-era levels store them and reduce per
        # node instead of issuing global atomics from every chunk
        part_elems = int(_lib.lib().wgb_hist_part_elems(S, F, B, chunk_cap)) if E == 1 else 0
        if part_elems and part_elems * 8 < 0.2 * torch.cuda.mem_get_info(dev)[0]:
            t["part_hist"] = torch.empty(part_elems * 2, dtype=torch.int32, device=dev)
        else:
            part_elems = 0
        # per-node partial arg-max: blocks of 8 features with one era, of
        # 32 (or 8 for num_bins > 33) with eras
        fb = SPLIT_WARPS if E == 1 else split_era_features(B)
        ncand = (ks + fb - 1) // fb
        t["cand"] = torch.empty((nslots, ncand, 4), **i32)
        if E > 1:
            # order in which the reference's per_era_gain.mean(dim=0) adds the
            # eras on this device (core.py:581-582)
            props = torch.cuda.get_device_properties(dev)
            sched, ops, depth = _lib.era_mean_plan(E, k * (B - 1), props.multi_processor_count,
                                                   props.max_threads_per_multi_processor)
            t["era_sched"] = torch.from_numpy(sched).to(dev)
            t["era_ops"] = torch.from_numpy(ops).to(dev)
        t["era_gain"] = torch.zeros(T * ((1 << D) - 1) * E, dtype=torch.float32, device=dev)
        t["nodes"] = torch.zeros(T * ((1 << (D + 1)) - 1) * 64, dtype=torch.uint8, device=dev)
        t["nn"] = torch.zeros(D + 1, **i32)
        t["nact"] = torch.zeros(D + 1, **i32)
        t["nchunks"] = torch.zeros(1, **i32)
        t["shift"] = torch.zeros(T, **i32)
        t["maxabs"] = torch.zeros(T, dtype=torch.float32, device=dev)
        t["rootsum"] = torch.zeros(T, dtype=torch.int64, device=dev)
        t["sync"] = torch.zeros(4, dtype=torch.int32, device=dev)
        t["g"] = torch.empty(max(NP, 1), dtype=torch.float32, device=dev)
        t["qg"] = torch.empty(max(NP, 1), **i32)
        t["feats"] = torch.empty(k, **i32)
        t["kpos"] = torch.empty(F, **i32)
        if nslice > 1:
            t["hstage"] = torch.empty(max(stage_elems, 1), dtype=torch.int64, device=dev)
            t["win"] = torch.zeros(nslice * nslots * win_words, **i32)
        self._t = t
        ws = _lib.WgbWs()
        ws.order[0], ws.order[1] = t["order0"].data_ptr(), t["order1"].data_ptr()
        ws.posnode[0], ws.posnode[1] = t["posnode0"].data_ptr(), t["posnode1"].data_ptr()
        for name in ("flags", "tile_cnt", "tile_off", "part", "hg", "chunks", "cand",
                     "era_gain", "nodes", "rootsum", "sync", "g", "qg", "feats", "kpos", "nn", "nact",
                     "nchunks", "shift", "maxabs"):
            setattr(ws, name, t[name].data_ptr())
        ws.N, ws.S, ws.F, ws.k, ws.E, ws.B, ws.D, ws.K = N, S, F, k, E, B, D, K
        ws.chunk_cap, ws.ntiles, ws.ncand_blk = max(chunk_cap, 1), ntiles, ncand
        ws.part_hist = t["part_hist"].data_ptr() if part_elems else None
        ws.part_hist_elems = part_elems
        ws.hist_ew = 0  # automatic
        ws.ntree = T
        if nslice > 1:
            ws.nslice, ws.slice, ws.ks, ws.win_words = nslice, slice_, ks, win_words
            ws.hstage, ws.hstage_elems = t["hstage"].data_ptr(), stage_elems
            ws.win = t["win"].data_ptr()
        ws.regular = 1 if self._bins_regular else 0
        ws.mcw = float(np.float32(self.min_child_weight))
        ws.eps = float(np.float32(self.L2_reg))
        ws.msg = float(np.float32(self.min_split_gain))
        ws.lr = float(np.float32(self.learning_rate))
        ws.mean_factor = cuda_mean_factor(E, k, B - 1)
        if E > 1:
            ws.era_sched, ws.era_ops = t["era_sched"].data_ptr(), t["era_ops"].data_ptr()
            ws.era_nops, ws.era_depth = int(t["era_ops"].numel()), depth
        self._ws = ws
        return ws

    def _fit(self, X, y, era_id, X_eval, y_eval, every, esr, eval_metric, classification):
        comm, dev = self._comm, self._dev
        st = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
        with torch.no_grad():
            self.num_samples, self.num_features = X.shape
            N, F = X.shape
            resume = self.warm_start and self._is_fitted and self._trees_trained > 0
            if not classification:
                # the base prediction reads two scalars back from the device:
                # done first, while the GPU is idle anyway, so that from the
                # binning to the last tree nothing waits on the host
                Yf = _to_dev(y, dev, torch.float32)
                if not resume:
                    self.base_prediction = exact_mean(Yf, comm)
            bins, _ = self._upload_bins(X, fit=True)
            if era_id is None:
                # the reference's default, era_id = ones: one era, every row in it;
                # nothing to upload, no host round trip
                self.unique_eras, era_dense = torch.ones(1, dtype=torch.int32, device=dev), None
            else:
                era_d = _to_dev(era_id, dev)
                self.unique_eras, era_dense = global_unique_eras(era_d, comm)
            self.num_eras = E = int(self.unique_eras.numel())
            K = self.num_classes if classification else 1
            k = max(1, int(self.colsample_bytree * F)) if self.colsample_bytree < 1.0 else F
            if comm.on:
                nglob = torch.tensor([N], dtype=torch.int64, device=dev)
                comm.sum_(nglob)
                self._n_global = int(nglob.item())
            else:
                self._n_global = N
            if E > 1:
                root_order = torch.sort(era_dense, stable=True).indices.to(torch.int32)
            else:
                root_order = torch.arange(N, dtype=torch.int32, device=dev)
            # a multiclass round grows its K class trees together (one level
            # launch sequence over the K trees' nodes)
            ntree = K if classification else 1
            if ntree > 1:
                root_order = root_order.repeat(ntree)
            # several ranks: each keeps and searches a slice of the positions
            # (reduce-scatter of the level histograms, all-gather of the best
            # split per node); _feature_slices = False sums every histogram on
            # every rank instead
            nslice = comm.world if comm.on and getattr(self, "_feature_slices", True) else 1
            ws = self._alloc_ws(N, F, k, E, K, ntree, nslice, comm.rank)
            self._ncomm = native_comm(comm, dev)
            ws.bins, ws.root_order = bins.data_ptr(), root_order.data_ptr()
            ws.era = era_dense.data_ptr() if E > 1 else None
            ws.N_global = self._n_global
            keep = [bins, root_order, era_dense]
            # with colsample_bytree < 1 each tree gets its k features as their own
            # matrix (wgb_tree_subset): the histograms then read and update k
            # features per row instead of all F
            S_sub = _round_up(k, 32)
            if k < F and N and N * S_sub < 0.25 * torch.cuda.mem_get_info(dev)[0]:
                bins_sub = torch.empty(N * S_sub, dtype=torch.int8, device=dev)
                kpos_sub = torch.empty(S_sub, dtype=torch.int32, device=dev)
                ws.bins_sub, ws.kpos_sub, ws.S_sub = bins_sub.data_ptr(), kpos_sub.data_ptr(), S_sub
                keep += [bins_sub, kpos_sub]
            # feature-major copy for the partition's bin reads, when it fits
            NT = (N + 15) // 16 * 16
            if N and F * NT < 0.25 * torch.cuda.mem_get_info(dev)[0]:
                bins_fm = torch.empty(F * NT, dtype=torch.int8, device=dev)
                _lib.call("wgb_bins_feature_major", ctypes_ptr(ws), bins_fm.data_ptr(), st())
                ws.bins_fm = bins_fm.data_ptr()
                keep.append(bins_fm)
            else:
                ws.bins_fm = None

            if classification:
                Yl = _to_dev(y, dev, torch.int32)
                pred = torch.zeros((N, K), dtype=torch.float32, device=dev)
                # core.py:449-456: prior_k = mean(Y == k) as torch's CUDA mean
                # (count * float(1/n)), from global counts, then log on device
                cnts = torch.stack([(Yl == c).sum() for c in range(K)]).to(torch.int64)
                comm.sum_(cnts)
                inv_n = np.float32(np.float32(1.0) / np.float32(self._n_global))
                for c, cnt in enumerate(cnts.tolist()):
                    prior = np.float32(np.float32(cnt) * inv_n)
                    if prior > 0:
                        pred[:, c] = torch.log(torch.tensor(prior, dtype=torch.float32, device=dev) + 1e-10)
                ws.y = None
                self.Y_gpu = Yl
            else:
                pred = torch.zeros((N, 1), dtype=torch.float32, device=dev) + np.float32(self.base_prediction)
                ws.y = Yf.data_ptr()
                self.Y_gpu = Yf
                keep.append(Yf)
            if resume:
                self._ensure_packed()
                self._predict_into(bins, pred, 0, self._trees_trained)
            ws.pred = pred.data_ptr()
            self._pred = pred
            keep.append(pred)
            self._keep = keep

            if X_eval is not None:
                self._eval_bins, _ = self._upload_bins(X_eval, fit=False)
                if classification:
                    ye = y_eval.cpu().numpy() if torch.is_tensor(y_eval) else y_eval
                    self._Y_eval = _to_dev(self.label_encoder.transform(ye), dev, torch.int32)
                    self.eval_metric = eval_metric if eval_metric != "mse" else "logloss"
                    self._eval_pred = self._init_proba_logits(self._eval_bins.shape[0])
                else:
                    self._Y_eval = _to_dev(y_eval, dev, torch.float32)
                    self.eval_metric = eval_metric
                    self._eval_pred = torch.zeros(self._eval_bins.shape[0], 1, dtype=torch.float32,
                                                  device=dev) + np.float32(self.base_prediction)
                self._eval_upto = 0
                self.eval_every_n_trees, self.early_stopping_rounds = every, esr
            else:
                self._eval_bins = None
                self.eval_every_n_trees = self.early_stopping_rounds = None

            if not self._is_fitted or not self.warm_start:
                self.per_era_feature_importance_ = np.zeros((E, F), dtype=np.float32)
                self.training_loss, self.eval_loss = [], []
            self.stop = False
            start = self._trees_trained if resume else 0
            if self.objective == "regression" and len(self.forest) < self.n_estimators:
                self.forest.extend([{} for _ in range(self.n_estimators - len(self.forest))])
            D = self.max_depth
            rec_nodes = ntree * ((1 << (D + 1)) - 1) * 64
            rec_gain = ntree * ((1 << D) - 1) * E
            T_new = self.n_estimators - start      # one record per grow call (a round's K trees)
            self._rec_nodes = torch.empty((T_new, rec_nodes), dtype=torch.uint8, pin_memory=True)
            self._rec_gain = torch.empty((T_new, max(rec_gain, 1)), dtype=torch.float32, pin_memory=True)
            self._rec_feats = torch.empty((T_new, k), dtype=torch.int32, pin_memory=True)
            self._rec_done = 0
            self._rec_decoded = 0
            self._rec_meta = []
            self._rec_events = []
            self._residuals = []
            if not resume:
                self.feature_subsets_ = []
            subsets = self.colsample_bytree < 1.0
            if not subsets:  # every tree uses all features in order
                self._t["feats"].copy_(torch.arange(F, dtype=torch.int32, device=dev))
                self._t["kpos"].copy_(torch.arange(F, dtype=torch.int32, device=dev))
            for i in range(start, self.n_estimators):
                if subsets:
                    feats = torch.randperm(F, device=dev, dtype=torch.int32)[:k]
                    comm.bcast_(feats)
                    self._t["feats"].copy_(feats)
                    self._t["kpos"].fill_(-1)
                    self._t["kpos"][feats.long()] = torch.arange(k, dtype=torch.int32, device=dev)
                if classification:
                    # core.py:782: residual of class c = -(softmax(F) - onehot)[:, c]
                    grads = softmax(pred, dim=1)
                    grads[torch.arange(N, device=dev), Yl.long()] -= 1.0
                    self._t["g"][: K * N].view(K, N).copy_(grads.t().neg())
                    self._grow_tree(ws, 0, st, i, None)
                    self._trees_trained = i + 1
                    self._eval_classification(i)
                else:
                    self._grow_tree(ws, 0, st, i, 0)
                    self._trees_trained = i + 1
                    self._eval_regression(i)
                if self.stop:
                    break
            self._finalize_records(classification)
            self._flush_train_loss()
            self.feature_importance_ = self.per_era_feature_importance_.sum(axis=0)
            self._is_fitted = True
            if classification:
                print(f"Finished training multiclass forest. Total rounds: {self._trees_trained} "
                      f"({self._trees_trained * self.num_classes} trees)")
            else:
                print(f"Finished training forest. Total trees: {self._trees_trained}")
            self._release()
        return self

    def _grow_tree(self, ws, cls, st, i, c):
        """Grow one tree (c = its class index) or, with c None, the batch of
        ws.ntree trees of round i (one per class)."""
        comm = self._comm
        ws.cls = cls
        p = ctypes_ptr(ws)
        instrumented = any(getattr(self, a, None) is not None
                           for a in ("_hist_events", "_comm_events", "_split_events", "_chunk_log"))
        if not instrumented and (not comm.on or self._ncomm is not None):
            # the whole tree from C++ (levels, and the per-level NCCL sums)
            _lib.call("wgb_grow_tree", p, self._ncomm, st())
            _lib.LAUNCHES[0] += level_launches(self.max_depth, ws.E, fused_partition(ws), ws.nslice > 1)
            self._after_tree(ws, i, c)
            return
        # the same sequence level by level from Python (a gloo group, or the
        # bench's per-level device timers)
        _lib.call("wgb_tree_reset", p, st())
        _lib.call("wgb_tree_residual", p, st())
        ctimer = getattr(self, "_comm_events", None)   # bench hook: device time of collectives
        if comm.on:
            if ctimer is not None:
                c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                c0.record()
            comm.max_(self._t["maxabs"])
            if ctimer is not None:
                c1.record()
                ctimer.append((c0, c1))
        _lib.call("wgb_tree_quantize", p, st())
        _lib.call("wgb_tree_subset", p, st())
        _lib.call("wgb_tree_root", p, st())
        sliced = ws.nslice > 1
        P = 2 * ws.E * (ws.ks if sliced else ws.k) * (ws.B + 1) + 2  # pool slot size
        wsp = ctypes_ptr(ws)
        timer = getattr(self, "_hist_events", None)
        for d in range(self.max_depth):
            if timer is not None:
                ev0 = torch.cuda.Event(enable_timing=True)
                ev1 = torch.cuda.Event(enable_timing=True)
                ev0.record()
            _lib.call("wgb_level_hist", p, d, st())
            if timer is not None:
                ev1.record()
                timer.append((ev0, ev1))
            clog = getattr(self, "_chunk_log", None)  # test hook: each level's chunk list
            if clog is not None:
                T = max(ws.ntree, 1)
                nodes = self._t["nodes"].view(-1, 64)[T * ((1 << d) - 1): T * ((1 << (d + 1)) - 1)]
                nch = int(self._t["nchunks"][0])
                clog.append((d, self._t["chunks"][:nch].cpu().numpy().copy(),
                             nodes.cpu().numpy().copy(), int(self._t["nn"][d])))
            if comm.on:
                first, count = _lib.built_slots(d, wsp)
                if ctimer is not None:
                    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    c0.record()
                if sliced:  # this rank's slice of the level's slots, summed over ranks
                    comm.reduce_scatter_(self._t["hg"][first * P:(first + count) * P],
                                         self._t["hstage"][: ws.nslice * count * P])
                else:
                    comm.sum_(self._t["hg"][first * P:(first + count) * P])
                if ctimer is not None:
                    c1.record()
                    ctimer.append((c0, c1))
            stimer = getattr(self, "_split_events", None)  # bench hook: split / partition device time
            if stimer is not None:
                s0, s1, s2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
                s0.record()
            _lib.call("wgb_level_split", p, d, st())
            if sliced:  # every rank's best split per node, the same choice everywhere
                cnt = (max(ws.ntree, 1) << d) * ws.win_words
                comm.all_gather_inplace_(self._t["win"], cnt)
                _lib.call("wgb_level_pick", p, d, st())
            if stimer is not None:
                s1.record()
            _lib.call("wgb_level_partition", p, d, st())
            if fused_partition(ws):
                _lib.LAUNCHES[0] -= 2  # one launch instead of three
            if stimer is not None:
                s2.record()
                stimer.append((s0, s1, s2))
        _lib.call("wgb_tree_finish", p, st())
        self._after_tree(ws, i, c)

    def _after_tree(self, ws, i, c):
        if getattr(self, "_record_residuals", False):  # test hook: residual of every tree
            g = self._t["g"][: ws.ntree * ws.N].view(ws.ntree, ws.N).cpu().numpy()
            self._residuals.extend(g[t].copy() for t in range(ws.ntree))
        self._store_record(i, c)

    def _store_record(self, i, c):
        j = self._rec_done
        self._rec_nodes[j].copy_(self._t["nodes"], non_blocking=True)
        self._rec_gain[j, : self._t["era_gain"].numel()].copy_(self._t["era_gain"], non_blocking=True)
        self._rec_feats[j].copy_(self._t["feats"], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._rec_events.append(ev)
        self._rec_meta.append((i, c))
        self._rec_done += 1
        self._drain_records(self.objective != "regression")

    # ------------------------------------------------------------------
    # tree records -> reference dict trees, importance (core.py:623-658)
    # ------------------------------------------------------------------
    def _decode_tree(self, j, t=0, ntree=1):
        """Tree t of record j -> compact pre-order arrays; per-era importance
        of its splits accumulated in pre-order (core.py:624-627 adds them
        while growing depth first, left before right).  Decoded on the host
        by the library (wgb_decode_tree; compact_tree is the same in numpy)."""
        D, E = self.max_depth, self.num_eras
        cap = (1 << (D + 1)) - 1
        packed = np.empty((cap, 2), np.int32)
        leaf = np.empty(cap, np.float32)
        samples = np.empty(cap, np.int64)
        imp = self.per_era_feature_importance_
        if imp.dtype != np.float32 or not imp.flags.c_contiguous:
            imp = self.per_era_feature_importance_ = np.ascontiguousarray(imp, np.float32)
        n = _lib.lib().wgb_decode_tree(self._rec_nodes[j].data_ptr(), D, ntree, t,
                                       self._rec_feats[j].data_ptr(), self._rec_gain[j].data_ptr(), E,
                                       imp.ctypes.data, imp.shape[1], packed.ctypes.data, leaf.ctypes.data,
                                       samples.ctypes.data, cap)
        if n < 0:
            _lib.check(-n, "wgb_decode_tree")
        return packed[:n].copy(), leaf[:n].copy(), samples[:n].copy()

    def _drain_records(self, classification):
        """Decode the records whose device->host copies have landed, without
        waiting: the host does it while the GPU grows the next trees."""
        j = self._rec_decoded
        while j < self._rec_done and self._rec_events[j].query():
            self._store_tree(j, classification)
            self._rec_events[j] = None
            j += 1
        self._rec_decoded = j

    def _finalize_records(self, classification):
        torch.cuda.current_stream().synchronize()
        for j in range(getattr(self, "_rec_decoded", 0), self._rec_done):
            self._store_tree(j, classification)
        self._rec_decoded = self._rec_done

    def _store_tree(self, j, classification):
        """Record j -> its tree (c an index) or its round's K class trees
        (c None, a batch grown together), decoded in class order."""
        i, c = self._rec_meta[j]
        if not hasattr(self, "feature_subsets_"):
            self.feature_subsets_ = []
        if c in (0, None):
            while len(self.feature_subsets_) <= i:
                self.feature_subsets_.append(None)
            self.feature_subsets_[i] = self._rec_feats[j].numpy().copy()
        f = self.__dict__["_forest"]
        if classification:
            while len(f) <= i:
                f.append([None] * self.num_classes)
        classes = [c] if c is not None else list(range(self.num_classes))
        for cc in classes:
            compact = self._decode_tree(j, 0 if c is not None else cc, 1 if c is not None else len(classes))
            self._compact[(i, cc)] = compact
            self._lazy.add((i, cc))
        self._packed = None

    def _sync_records(self, classification):
        if self._rec_done > getattr(self, "_rec_decoded", 0):
            torch.cuda.current_stream().synchronize()
            for j in range(self._rec_decoded, self._rec_done):
                self._store_tree(j, classification)
            self._rec_decoded = self._rec_done

    def _release(self):
        for name in ("_t", "_ws", "_keep", "_pred", "Y_gpu", "_eval_bins", "_eval_pred", "_Y_eval"):
            if hasattr(self, name):
                delattr(self, name)
        for name in ("_rec_nodes", "_rec_gain", "_rec_feats", "_rec_meta", "_rec_events"):
            if hasattr(self, name):
                delattr(self, name)
        self._rec_decoded = 0

    # ------------------------------------------------------------------
    # eval / early stopping (core.py:660-690, 820-853)
    # ------------------------------------------------------------------
    def _gather_cat(self, t):
        return torch.cat(self._comm.gather_var(t.reshape(-1))) if self._comm.on else t.reshape(-1)

    def get_eval_metric(self, y_true, y_pred):
        if self.eval_metric == "mse":
            return ((y_true - y_pred) ** 2).mean().item()
        elif self.eval_metric == "corr":
            return 1 - torch.corrcoef(torch.vstack([y_true, y_pred]))[0, 1].item()
        elif self.eval_metric == "rmsle":
            return rmsle_torch(y_true, y_pred).item()
        raise ValueError(f"Invalid eval_metric: {self.eval_metric}.")

    def _eval_regression(self, i):
        if self.eval_every_n_trees is None:
            return
        r = (self.Y_gpu - self._pred[:, 0])
        if self._comm.on:
            s = torch.stack([(r * r).sum().double(),
                             torch.tensor(float(r.numel()), dtype=torch.float64, device=r.device)])
            self._comm.sum_(s)
            self._defer_train_loss(s[0] / s[1])
        else:
            self._defer_train_loss((r ** 2).mean())
        if i % self.eval_every_n_trees == 0:
            train_loss = self._flush_train_loss()
            self._sync_records(False)
            self._advance_eval(i + 1)
            yt = self._gather_cat(self._Y_eval)
            yp = self._gather_cat(self._eval_pred[:, 0])
            eval_loss = self.get_eval_metric(yt, yp)
            self.eval_loss.append(eval_loss)
            if len(self.eval_loss) > self.early_stopping_rounds:
                if self.eval_loss[-(self.early_stopping_rounds + 1)] < self.eval_loss[-1]:
                    self.stop = True
            print(f"🌲 Tree {i+1}/{self.n_estimators} | Train MSE: {train_loss:.6f} | "
                  f"Eval {self.eval_metric}: {eval_loss:.6f}")

    def _eval_classification(self, i):
        if self.eval_every_n_trees is None:
            return
        probs = softmax(self._pred, dim=1)
        if self._comm.on:
            p = probs[torch.arange(probs.shape[0], device=probs.device), self.Y_gpu.long()]
            p = torch.clamp(p, 1e-15, 1 - 1e-15)
            s = torch.stack([-torch.log(p).sum().double(),
                             torch.tensor(float(p.numel()), dtype=torch.float64, device=p.device)])
            self._comm.sum_(s)
            self._defer_train_loss(s[0] / s[1])
        else:
            self._defer_train_loss(log_loss_torch(self.Y_gpu, probs))
        if i % self.eval_every_n_trees == 0:
            train_loss = self._flush_train_loss()
            self._sync_records(True)
            self._advance_eval(i + 1)
            eval_probs = softmax(self._eval_pred, dim=1)
            yt = self._gather_cat(self._Y_eval)
            if self._comm.on:
                eval_probs = torch.cat(self._comm.gather_var(eval_probs.reshape(-1))).reshape(-1, self.num_classes)
            if self.eval_metric == "accuracy":
                eval_loss = 1.0 - accuracy_torch(yt, torch.argmax(eval_probs, dim=1)).item()
            else:
                eval_loss = log_loss_torch(yt, eval_probs).item()
            self.eval_loss.append(eval_loss)
            if len(self.eval_loss) > self.early_stopping_rounds:
                if self.eval_loss[-(self.early_stopping_rounds + 1)] < self.eval_loss[-1]:
                    self.stop = True
            print(f"🌲 Round {i+1}/{self.n_estimators} ({self.num_classes} trees) | "
                  f"Train LogLoss: {train_loss:.6f} | Eval {self.eval_metric}: {eval_loss:.6f}")

    def _defer_train_loss(self, t):
        """The training loss of a tree / round stays on the device until the
        next eval point (or the end of the fit): no host sync per tree."""
        self.__dict__.setdefault("_tl_pending", []).append(t.reshape(1).double())

    def _flush_train_loss(self):
        pend = self.__dict__.get("_tl_pending") or []
        if pend:
            self.training_loss.extend(torch.cat(pend).tolist())
            pend.clear()
        return self.training_loss[-1] if self.training_loss else float("nan")

    def _advance_eval(self, upto):
        """Add the trees [_eval_upto, upto) to the running eval prediction
        (tree order, so equal to predicting with the whole forest)."""
        if upto <= self._eval_upto:
            return
        self._ensure_packed()
        self._predict_into(self._eval_bins, self._eval_pred, self._eval_upto, upto)
        self._eval_upto = upto

    # ------------------------------------------------------------------
    # prediction (core.py:917-1030)
    # ------------------------------------------------------------------
    def _flat_trees(self):
        if self.objective == "regression":
            return [t for t in self.forest if t]
        return [t for rnd in self.forest if rnd for t in rnd]

    def _tree_slots(self):
        """(i, c) of every trained tree in prediction order (round-major)."""
        f = self.__dict__.get("_forest") or []
        lazy, out = self.__dict__.get("_lazy", set()), []
        for i, r in enumerate(f):
            if isinstance(r, list):
                out.extend((i, c) for c, t in enumerate(r) if t or (i, c) in lazy)
            elif r or (i, 0) in lazy:
                out.append((i, 0))
        return out

    def _ensure_packed(self):
        if self._packed is None:
            compact, f = self.__dict__.get("_compact", {}), self.__dict__.get("_forest")
            parts = []
            for (i, c) in self._tree_slots():
                if (i, c) in compact:
                    parts.append(compact[(i, c)][0])
                else:   # a tree given as a dict (loaded model)
                    t = f[i][c] if isinstance(f[i], list) else f[i]
                    parts.append(pack_trees([t])[0])
            offs = np.zeros(len(parts) + 1, np.int32)
            if parts:
                offs[1:] = np.cumsum([len(p) for p in parts])
            nodes = np.concatenate(parts) if parts else np.zeros((0, 2), np.int32)
            dev = getattr(self, "_dev", torch.device("cuda", torch.cuda.current_device()))
            heap = heap_forest(parts, self.max_depth) if self.max_depth <= HEAP_DMAX else None
            self._packed = (torch.from_numpy(nodes.reshape(-1)).to(dev),
                            torch.from_numpy(offs).to(dev), offs,
                            torch.from_numpy(heap.reshape(-1).view(np.int32)).to(dev) if heap is not None else None)
        return self._packed

    def _predict_into(self, bins, out, r0, r1):
        """out[:, class] += lr * leaf for the trees of rounds [r0, r1)."""
        nodes, offs_d, offs, heap = self._ensure_packed()
        K = out.shape[1]
        t0, t1 = r0 * K, min(r1 * K, len(offs) - 1)
        if t1 <= t0:
            return
        lr = float(np.float32(self.learning_rate))
        st = torch.cuda.current_stream().cuda_stream
        if heap is not None:
            W = 2 << self.max_depth
            _lib.call("wgb_predict_heap", bins.data_ptr(), bins.shape[0], bins.shape[1],
                      heap.data_ptr() + 4 * t0 * W, t1 - t0, K, self.max_depth, lr, out.data_ptr(), st)
        else:
            _lib.call("wgb_predict_packed", bins.data_ptr(), bins.shape[0], bins.shape[1],
                      nodes.data_ptr(), offs_d[t0:].data_ptr(), t1 - t0, K, lr, out.data_ptr(), st)

    def _init_proba_logits(self, n):
        """core.py:1001-1007: the prior of class k is 1/K (sic), computed on the host."""
        Fm = torch.zeros((n, self.num_classes), dtype=torch.float32)
        for c in range(self.num_classes):
            prior_k = (self.classes_ == self.classes_[c]).sum() / len(self.classes_)
            if prior_k > 0:
                Fm[:, c] = torch.log(torch.tensor(prior_k + 1e-10))
        return Fm.to(self._dev)

    def bin_inference_data(self, X_np):
        if not hasattr(self, "_dev"):
            self._dev = torch.device("cuda", torch.cuda.current_device())
        self._comm = getattr(self, "_comm", None) or _Comm(False)
        if isinstance(self.bin_edges, np.ndarray):
            self.bin_edges = torch.from_numpy(self.bin_edges)
        self.bin_edges = self.bin_edges.to(self._dev)
        return self._upload_bins(X_np, fit=False)[0]

    def predict_binned(self, bins):
        out = torch.zeros((bins.shape[0], 1), dtype=torch.float32, device=bins.device) + \
            np.float32(self.base_prediction)
        self._predict_into(bins, out, 0, len(self._tree_slots()))
        return out[:, 0]

    def predict_proba_binned(self, bins):
        out = self._init_proba_logits(bins.shape[0])
        self._predict_into(bins, out, 0, len({i for i, _ in self._tree_slots()}))
        return softmax(out, dim=1)

    def predict(self, X_np):
        if self.objective in ("multiclass", "binary"):
            probs = self.predict_proba(X_np)
            return self.label_encoder.inverse_transform(np.argmax(probs, axis=1))
        with torch.cuda.device(self._device_for_predict()):
            bins = self.bin_inference_data(X_np)
            return self.predict_binned(bins).cpu().numpy()

    def predict_proba(self, X_np):
        if self.objective not in ["multiclass", "binary"]:
            raise ValueError("predict_proba only available for classification objectives")
        with torch.cuda.device(self._device_for_predict()):
            bins = self.bin_inference_data(X_np)
            return self.predict_proba_binned(bins).cpu().numpy()

    def _device_for_predict(self):
        if not hasattr(self, "_dev"):
            self._dev = torch.device("cuda", torch.cuda.current_device())
        return self._dev

    # ------------------------------------------------------------------
    # importance, save / load (core.py:1032-1213)
    # ------------------------------------------------------------------
    def get_feature_importance(self, importance_type="gain", normalize=True):
        if self.feature_importance_ is None:
            raise ValueError("Model has not been fitted yet.")
        if importance_type != "gain":
            raise ValueError(f"importance_type '{importance_type}' not supported. Use 'gain'.")
        imp = self.feature_importance_.copy()
        if normalize and imp.sum() > 0:
            imp = imp / imp.sum()
        return imp

    def get_per_era_feature_importance(self, normalize=True):
        if self.per_era_feature_importance_ is None:
            raise ValueError("Model has not been fitted yet.")
        imp = self.per_era_feature_importance_.copy()
        if normalize:
            for e in range(imp.shape[0]):
                s = imp[e].sum()
                if s > 0:
                    imp[e] /= s
        return imp

    def save_model(self, path):
        if not self._is_fitted:
            raise ValueError("Cannot save unfitted model. Call fit() first.")
        state = {k: getattr(self, k) for k in (
            "objective", "num_bins", "max_depth", "learning_rate", "n_estimators",
            "min_child_weight", "min_split_gain", "L2_reg", "colsample_bytree", "random_state",
            "warm_start", "forest", "base_prediction", "num_features", "num_classes", "classes_",
            "label_encoder", "feature_importance_", "per_era_feature_importance_", "_is_fitted",
            "_trees_trained", "training_loss", "eval_loss")}
        state["bin_edges"] = self.bin_edges.cpu() if torch.is_tensor(self.bin_edges) else self.bin_edges
        with open(path, "wb") as f:
            pickle.dump(state, f)
        print(f"Model saved to {path}")

    def load_model(self, path):
        with open(path, "rb") as f:
            state = pickle.load(f)
        for k, v in state.items():
            setattr(self, k, v)
        self.training_loss = state.get("training_loss", [])
        self.eval_loss = state.get("eval_loss", [])
        self._packed = None
        print(f"Model loaded from {path} ({self._trees_trained} trees)")
        return self

    def flatten_tree(self, tree, max_nodes):
        """core.py:1215-1252 (pre-order, [max_nodes, 6], NaN-filled)."""
        flat = torch.full((max_nodes, 6), float("nan"), dtype=torch.float32)
        counter = [0]

        def walk(nd):
            i = counter[0]
            counter[0] += 1
            if "leaf_value" in nd:
                flat[i, 4] = 1.0
                flat[i, 5] = nd["leaf_value"]
            else:
                flat[i, 0] = float(nd["feature"])
                flat[i, 1] = float(nd["bin"])
                flat[i, 2] = counter[0]
                walk(nd["left"])
                flat[i, 3] = counter[0]
                walk(nd["right"])
                flat[i, 4] = 0.0
        walk(tree)
        return flat


def ctypes_ptr(ws):
    import ctypes
    return ctypes.cast(ctypes.pointer(ws), ctypes.c_void_p)
