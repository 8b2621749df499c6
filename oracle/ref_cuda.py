"""The reference's own CUDA kernels driven by its regression fit loop
(TEST / BASELINE INFRASTRUCTURE ONLY -- the product never imports this file).

Purpose: time the reference's CUDA build on the same B200 as this build
("Ref CUDA 1xB200"), and check that the compiled reference kernels agree with
the golden fixtures.  The kernels are the reference's own, compiled from its
sources by oracle/build_ref.py; the host loop restates the steps of
warpgbm/core.py (quantverse/warpgbm v2.2.0) that call them, in the same
order, with the same torch ops and the same host synchronisations, because
that Python file cannot travel to the GPU box:

* ingest / binning, per column: host column -> device, torch.quantile edges,
  custom_cuda_binner (core.py:487-541); pre-binned integer input is copied
  column by column (core.py:499-517); eras via torch.unique (core.py:540);
* base prediction = mean(y) (core.py:386-388); root rows = arange(N);
* per tree: residual = y - pred, optional randperm feature subset, root
  histogram (core.py:710-726);
* per node (core.py:597-658): fresh zero G/H tensors + compute_histogram3
  (core.py:543-563); compute_split + the DES rule + argmax + two .item()
  (core.py:565-594); per-era importance with one .item() per era; boolean
  partition; smaller-child histogram and fp32 sibling subtraction; leaves
  = mean residual with pred[rows] += lr * leaf and one .item().

Regression only (the bench workload and the era-aware config).
"""
from __future__ import annotations

import time

import numpy as np
import torch


class RefCudaFit:
    def __init__(self, ops, num_bins=10, max_depth=3, learning_rate=0.1, n_estimators=100,
                 min_child_weight=20, min_split_gain=0.0, L2_reg=1e-6, colsample_bytree=1.0,
                 threads_per_block=64, rows_per_thread=4, random_state=None):
        self.ops = ops
        self.B, self.D, self.lr, self.T = num_bins, max_depth, learning_rate, n_estimators
        self.mcw, self.msg, self.l2 = min_child_weight, min_split_gain, L2_reg
        self.colsample = colsample_bytree
        self.tpb, self.rpt = threads_per_block, rows_per_thread
        self.random_state = random_state
        self.dev = torch.device("cuda")

    # core.py:487-541
    def _ingest(self, X, y, era):
        dev, B = self.dev, self.B
        N, F = X.shape
        Y = torch.from_numpy(y).type(torch.float32).to(dev)
        E = torch.from_numpy(era).type(torch.int32).to(dev)
        bins = torch.empty((N, F), dtype=torch.int8, device=dev)
        if np.issubdtype(X.dtype, np.integer) and np.all(X.max(axis=0) < B):
            for f in range(F):
                bins[:, f] = torch.as_tensor(X[:, f], device=dev).contiguous()
            edges = torch.arange(1, B, dtype=torch.float32).repeat(F, 1).to(dev)
        else:
            edges = torch.empty((F, B - 1), dtype=torch.float32, device=dev)
            for f in range(F):
                xf = torch.as_tensor(X[:, f], device=dev, dtype=torch.float32).contiguous()
                qs = torch.linspace(0, 1, B + 1, device=dev, dtype=xf.dtype)[1:-1]
                ef = torch.quantile(xf, qs, dim=0).contiguous()
                col = bins[:, f].contiguous()
                self.ops.custom_cuda_binner(xf, ef, col)
                bins[:, f] = col
                edges[f, :] = ef
        uniq, inv = torch.unique(E, return_inverse=True)
        return bins, inv, edges, uniq, Y

    def _hist(self, rows, feats):
        G = torch.zeros((self.E, len(feats), self.B), device=self.dev, dtype=torch.float32)
        H = torch.zeros((self.E, len(feats), self.B), device=self.dev, dtype=torch.float32)
        self.ops.compute_histogram3(self.bins, self.residual, rows, feats, self.era, G, H, self.B,
                                    self.tpb, self.rpt)
        return G, H

    def _split(self, G, H):
        self.ops.compute_split(G, H, self.msg, self.mcw, self.l2, self.peg, self.ped, self.tpb)
        if self.E == 1:
            crit = self.peg[0, :, :]
            mask = crit > self.msg
        else:
            agree = self.ped.mean(dim=0).abs()
            crit = self.peg.mean(dim=0)
            mask = (agree == agree.max()) & (crit > self.msg)
        if not mask.any():
            return -1, -1
        crit[mask == 0] = float("-inf")
        idx = torch.argmax(crit)
        nb = self.B - 1
        return (idx // nb).item(), (idx % nb).item()

    def _leaf(self, rows):
        v = self.residual[rows].mean()
        self.pred[rows] += self.lr * v
        return {"leaf_value": v.item(), "samples": rows.numel()}

    def _grow(self, G, H, rows, depth):
        if depth == self.D:
            return self._leaf(rows)
        f, b = self._split(G, H)
        if f == -1:
            return self._leaf(rows)
        gfi = self.feats_tree[f].item()
        g = self.peg[:, f, b]
        for e in range(self.E):
            self.imp[e, gfi] += g[e].item()
        m = self.bins[rows, self.feats_tree[f]] <= b
        L, R = rows[m], rows[~m]
        if L.numel() <= R.numel():
            GL, HL = self._hist(L, self.feats_tree)
            GR, HR = G - GL, H - HL
        else:
            GR, HR = self._hist(R, self.feats_tree)
            GL, HL = G - GR, H - HR
        left = self._grow(GL, HL, L, depth + 1)
        right = self._grow(GR, HR, R, depth + 1)
        return {"feature": self.feats_tree[f], "bin": b, "left": left, "right": right}

    def fit(self, X, y, era_id=None):
        """Returns self; .forest, .pred, .timings = {"ingest_s", "grow_s"} (CUDA-synchronised)."""
        if self.random_state is not None:
            torch.manual_seed(self.random_state)
            torch.cuda.manual_seed_all(self.random_state)
        if era_id is None:
            era_id = np.ones(X.shape[0], dtype="int32")
        with torch.no_grad():
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            self.bins, inv, self.edges, uniq, self.Y = self._ingest(X, y, era_id)
            N, F = X.shape
            self.E = len(uniq)
            self.era = inv.to(dtype=torch.int32)
            self.pred = torch.zeros_like(self.Y)
            self.base = self.Y.mean().item()
            self.pred += self.base
            root = torch.arange(N, device=self.dev, dtype=torch.int32)
            all_feats = torch.arange(F, device=self.dev, dtype=torch.int32)
            torch.cuda.synchronize()
            t1 = time.perf_counter()
            self.imp = np.zeros((self.E, F), dtype=np.float32)
            k = max(1, int(self.colsample * F)) if self.colsample < 1.0 else F
            self.peg = torch.zeros(self.E, k, self.B - 1, device=self.dev, dtype=torch.float32)
            self.ped = torch.zeros(self.E, k, self.B - 1, device=self.dev, dtype=torch.float32)
            self.forest = []
            for _ in range(self.T):
                self.residual = self.Y - self.pred
                if self.colsample < 1.0:
                    self.feats_tree = torch.randperm(F, device=self.dev, dtype=torch.int32)[:k]
                else:
                    self.feats_tree = all_feats
                G, H = self._hist(root, self.feats_tree)
                self.forest.append(self._grow(G, H, root, 0))
            torch.cuda.synchronize()
            t2 = time.perf_counter()
        self.timings = {"ingest_s": t1 - t0, "grow_s": t2 - t1}
        return self
