"""Parity against the reference itself at BASELINE scale.

The reference's own kernels (warpgbm/cuda/*.cu, compiled unchanged for
sm_100a into oracle/_ref/) and its host split code (core.py:565-594: torch
mean, mask, argmax, on the device) are run at every node of the trees this
build grew, on the same rows and residuals.  Our split must be the
reference's choice, except where the two candidates are closer than the
reference's own fp32 error: the reference sums residuals with fp32 atomics in
any order, so there its choice is not determined (the north star's near-tie
allowance).  That error is measured per node as the difference between the
reference's fp32 criterion and the same criterion from float64 sums.  The
walk then follows our split, so every node is compared on identical rows.
Leaves are checked against the reference's fp32 mean of the node's residuals
(core.py:599), predictions at the end.

Config 2 in full (1M x 1000, B=32, depth 5, 3 trees), a config-4 subset
(600 eras, DES, colsample 0.5, depth 8) and config 3 in full against the CPU
oracle in reference mode (final eval logloss within 1e-3, core.py:746-853).
"""
import numpy as np
import pytest
import torch

import oracle as O
from warpgbm_b200 import WarpGBM

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref_ops():
    from oracle.build_ref import load
    try:
        return load()
    except RuntimeError as e:
        pytest.skip(str(e))


def _gain64(G, H, mcw, eps):
    """best_split_kernel.cu:25-53 in float64 (criterion without fp32 error)."""
    GT, HT = G.sum(-1, keepdim=True), H.sum(-1, keepdim=True)
    GL, HL = G.cumsum(-1)[..., :-1], H.cumsum(-1)[..., :-1]
    GR, HR = GT - GL, HT - HL
    ok = (HL >= mcw) & (HR >= mcw)
    g = GL * GL / (HL + eps) + GR * GR / (HR + eps) - GT * GT / (HT + eps)
    d = torch.where(GL / (HL + eps) > GR / (HR + eps), 1.0, -1.0)
    return torch.where(ok, g, 0.0), torch.where(ok, d, 0.0)


class Guided:
    """Walks our trees with the reference's kernels at every node."""

    def __init__(self, ops, bins, era, E, params, dev):
        self.ops, self.bins, self.era, self.E, self.dev = ops, bins, era, E, dev
        self.B = params["num_bins"]
        self.mcw = float(params.get("min_child_weight", 20))
        self.msg = float(params.get("min_split_gain", 0.0))
        self.eps = float(params.get("L2_reg", 1e-6))
        self.exact = self.ties = self.leaves = 0
        self.worst_leaf = 0.0

    def ref_hist(self, g, rows, feats):
        k = feats.numel()
        G = torch.zeros((self.E, k, self.B), device=self.dev)
        H = torch.zeros((self.E, k, self.B), device=self.dev)
        self.ops.compute_histogram3(self.bins, g, rows, feats, self.era, G, H, self.B, 64, 4)
        return G, H

    def hist64(self, g, rows, feats):
        """float64 histogram of the node (exact enough to measure fp32 error)."""
        k = feats.numel()
        b = self.bins[rows.long()][:, feats.long()].long()              # [n, k]
        e = self.era[rows.long()].long() if self.E > 1 else torch.zeros_like(rows, dtype=torch.long)
        idx = (e[:, None] * k + torch.arange(k, device=self.dev)[None, :]) * self.B + b
        ok = (b >= 0) & (b < self.B)
        G = torch.zeros(self.E * k * self.B, dtype=torch.float64, device=self.dev)
        H = torch.zeros_like(G)
        G.index_add_(0, idx[ok], g[rows.long()].double()[:, None].expand(-1, k)[ok])
        H.index_add_(0, idx[ok], torch.ones_like(idx[ok], dtype=torch.float64))
        return G.view(self.E, k, self.B), H.view(self.E, k, self.B)

    def ref_split(self, G, H):
        """core.py:565-594 verbatim in behaviour: per-era kernel, mean, mask, argmax."""
        k = G.shape[1]
        peg = torch.zeros((self.E, k, self.B - 1), device=self.dev)
        ped = torch.zeros_like(peg)
        self.ops.compute_split(G, H, self.msg, self.mcw, self.eps, peg, ped, 64)
        if self.E == 1:
            crit, mask = peg[0].clone(), peg[0] > self.msg
        else:
            agree = ped.mean(dim=0).abs()
            crit = peg.mean(dim=0)
            mask = (agree == agree.max()) & (crit > self.msg)
        return crit, mask

    def node(self, nd, g, rows, feats, depth, D, pred_ref, lr):
        if "leaf_value" in nd:
            ref_leaf = g[rows.long()].mean()
            scale = max(abs(float(ref_leaf)), float(g[rows.long()].abs().mean()))
            err = abs(nd["leaf_value"] - float(ref_leaf))
            assert err <= 1e-5 * scale + 1e-12, (nd["leaf_value"], float(ref_leaf))
            self.worst_leaf = max(self.worst_leaf, err / max(scale, 1e-30))
            pred_ref[rows.long()] += lr * ref_leaf
            self.leaves += 1
            if depth < D:  # we found no split: the reference must find none either
                crit, mask = self.ref_split(*self.ref_hist(g, rows, feats))
                if bool(mask.any()):
                    self._tie_or_fail(g, rows, feats, crit, mask, None)
            return
        G, H = self.ref_hist(g, rows, feats)
        crit, mask = self.ref_split(G, H)
        fpos = int((feats == nd["feature"]).nonzero()[0, 0])
        ours = fpos * (self.B - 1) + nd["bin"]
        assert bool(mask.any()), "the reference finds no split where we split"
        masked = torch.where(mask, crit, torch.tensor(float("-inf"), device=self.dev))
        best = int(torch.argmax(masked))
        if best == ours:
            self.exact += 1
        else:
            self._tie_or_fail(g, rows, feats, crit, mask, ours)
        go_left = self.bins[rows.long(), nd["feature"]] <= nd["bin"]
        self.node(nd["left"], g, rows[go_left], feats, depth + 1, D, pred_ref, lr)
        self.node(nd["right"], g, rows[~go_left], feats, depth + 1, D, pred_ref, lr)

    def _tie_or_fail(self, g, rows, feats, crit, mask, ours):
        """The reference's best and our cell (or 'no split') are a near tie:
        their float64 criteria differ by no more than the reference's fp32
        error at those cells."""
        G64, H64 = self.hist64(g, rows, feats)
        g64, d64 = _gain64(G64, H64, self.mcw, self.eps)
        crit64 = g64.mean(0).reshape(-1)
        err = (crit.reshape(-1).double() - crit64).abs()
        masked = torch.where(mask.reshape(-1), crit.reshape(-1), torch.tensor(float("-inf"), device=self.dev))
        best = int(torch.argmax(masked))
        if ours is None:  # we saw no candidate above min_split_gain
            gap, bound = float(crit64[best]) - self.msg, 2 * float(err[best]) + 1e-12
        else:
            if self.E > 1 and not bool(mask.reshape(-1)[ours]):
                # our cell is not among the reference's maximum-agreement
                # cells: only a direction flipped by fp32 sums explains that
                agree64 = d64.mean(0).abs().reshape(-1)
                assert float(agree64[ours]) >= float(agree64.max()) - 1e-12, "era agreement differs"
            gap = abs(float(crit64[best] - crit64[ours]))
            bound = 2 * float(err[best] + err[ours]) + 1e-12
        assert gap <= bound, f"split differs from the reference's beyond its fp32 error ({gap} > {bound})"
        self.ties += 1


def _compare(model, ops, bins, y, era, params, dev):
    """Walk every tree of `model` with the reference's kernels; returns the
    Guided counters.  Residuals are y minus our prediction before each tree
    (identical to the fit's), so both sides see the same inputs."""
    N, F = bins.shape
    E = model.num_eras
    era_d = (torch.from_numpy(np.unique(era, return_inverse=True)[1].astype(np.int32)).to(dev)
             if era is not None else torch.zeros(N, dtype=torch.int32, device=dev))
    gd = Guided(ops, bins, era_d, E, params, dev)
    yd = torch.from_numpy(y).to(dev)
    D, lr = params["max_depth"], np.float32(params["learning_rate"])
    wb = torch.zeros((N, bins_stride_of(F)), dtype=torch.int8, device=dev)
    wb[:, :F] = bins
    pred_ref = torch.full((N,), np.float32(model.base_prediction), device=dev)
    rows = torch.arange(N, dtype=torch.int32, device=dev)
    for t, tree in enumerate(model._flat_trees()):
        out = torch.full((N, 1), np.float32(model.base_prediction), device=dev)
        model._predict_into(wb, out, 0, t)
        g = (yd - out[:, 0]).contiguous()
        sub = model.feature_subsets_[t] if params.get("colsample_bytree", 1.0) < 1.0 else np.arange(F)
        feats = torch.from_numpy(np.asarray(sub, np.int32)).to(dev)
        gd.node(tree, g, rows, feats, 0, D, pred_ref, lr)
    pg = model.predict_binned(wb).double()
    floor = 1e-5 * float(pred_ref.abs().max())
    assert float((pg - pred_ref.double()).abs().max()) <= floor + 1e-5 * float(pg.abs().max())
    return gd


def bins_stride_of(F):
    from warpgbm_b200.core import bins_stride
    return bins_stride(F)


def test_config2_full_shape_splits_match_the_reference_kernels(cuda, ref_ops):
    """BASELINE config 2 (1M x 1000 f32, B=32, depth 5), 3 trees."""
    import bench
    X, y = bench.make_data(0, 1_000_000, 1000)
    params = dict(num_bins=32, max_depth=5, n_estimators=3, learning_rate=0.01)
    m = WarpGBM(**params).fit(X, y)
    bins = m.bin_inference_data(X)[:, :1000].contiguous()
    gd = _compare(m, ref_ops, bins, y, None, params, cuda)
    print(f"config 2: {gd.exact} splits as the reference, {gd.ties} near ties, {gd.leaves} leaves "
          f"(worst leaf error {gd.worst_leaf:.2e} of scale)")
    assert gd.exact >= 0.9 * (gd.exact + gd.ties)


def test_config4_subset_splits_match_the_reference_kernels(cuda, ref_ops):
    """BASELINE config 4's DES path on a subset: 240k rows x 256 pre-binned
    features in {0..4}, 600 contiguous eras, B=5, depth 8, colsample 0.5."""
    rng = np.random.default_rng(44)
    n, F, E = 240_000, 256, 600
    X = rng.integers(0, 5, (n, F)).astype(np.int8)
    era = np.repeat(np.arange(E), n // E).astype(np.int32)
    c = np.abs(rng.standard_normal((E, 50)))
    c[:, :30] *= np.where(rng.random(30) < 0.5, -1.0, 1.0)
    c[:, 30:] *= np.where(rng.random((E, 20)) < 0.5, -1.0, 1.0)
    score = (X[:, :50] * c[era]).sum(1) + 2.0 * rng.standard_normal(n)
    y = np.zeros(n, np.float32)
    for e in range(E):
        s = score[e * (n // E):(e + 1) * (n // E)]
        y[e * (n // E):(e + 1) * (n // E)] = np.round(np.argsort(np.argsort(s)) / (len(s) - 1) * 4) / 4
    params = dict(num_bins=5, max_depth=8, n_estimators=3, learning_rate=0.01, colsample_bytree=0.5,
                  random_state=0)
    m = WarpGBM(**params).fit(X, y, era_id=era)
    bins = torch.from_numpy(X).to(cuda)
    gd = _compare(m, ref_ops, bins, y, era, params, cuda)
    print(f"config 4 subset: {gd.exact} splits as the reference, {gd.ties} near ties, {gd.leaves} leaves")
    assert gd.exact >= 0.9 * (gd.exact + gd.ties)


def test_config3_final_logloss_matches_the_reference_oracle(cuda):
    """BASELINE config 3 in full (multiclass, 5 classes, depth 6, lr 0.1,
    early stopping 5 on logloss every 10 rounds): the final eval logloss of
    this build against the reference-mode oracle (fp32 sums in sample order,
    torch-CPU softmax and means) grown for the same number of rounds."""
    import bench
    d = bench.config_data("c3", cuda)
    m = WarpGBM(**d["params"]).fit(d["X"], d["y"], **d["fit_kw"])
    R = m._trees_trained
    Xe, ye = d["fit_kw"]["X_eval"], d["fit_kw"]["y_eval"]
    p = {k: v for k, v in d["params"].items() if k != "random_state"}
    p["n_estimators"] = R
    o = O.OracleGBM(mode="reference", **p).fit(d["X"], d["y"], edges=m.bin_edges.cpu().numpy())

    def ll(P):
        idx = np.searchsorted(m.classes_, ye)
        return float(-np.mean(np.log(np.clip(P[np.arange(len(ye)), idx], 1e-15, 1 - 1e-15))))
    ours, ref = ll(m.predict_proba(Xe)), ll(o.predict_proba(Xe))
    print(f"config 3: {R} rounds, eval logloss {ours:.6f} (reference oracle {ref:.6f})")
    assert abs(ours - ref) < 1e-3
