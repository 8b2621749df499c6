"""Generate the golden fixtures in tests/golden/*.npz from the REFERENCE.

Runs quantverse/warpgbm's own ``warpgbm/core.py`` (imported read-only from the
reference checkout given as the first argument, or $WGB_REFERENCE) on the CPU: the compiled CUDA extension
``warpgbm.cuda.node_kernel`` is replaced by ``_TorchKernels`` below, a torch
restatement of the four kernels written independently of oracle/, and
``device="cuda"`` literals inside core.py are redirected to the CPU.  Every
other line of the reference (pre-binning detection, quantile edges, era
remapping, DES rule, argmax, partition, leaf means, importance, flattening,
multiclass softmax) runs unchanged, so the fixtures pin the oracle's host
logic to the reference's.

Usage:  python tests/golden/make_golden.py [/path/to/reference] [--models]
(--models writes only the two model pickles saved by the reference's own
save_model).  The fixtures are committed; the GPU box never needs the
reference.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


class _TorchKernels(types.ModuleType):
    """torch-CPU restatement of warpgbm/cuda/*.cu (one legal atomic order:
    contributions are added in sample order, trees in tree order)."""

    def __init__(self):
        super().__init__("warpgbm.cuda.node_kernel")

    @staticmethod
    def compute_histogram3(bin_indices, residuals, sample_indices, feature_indices,
                           era_indices, grad_hist, hess_hist, num_bins,
                           threads_per_block=256, rows_per_thread=1):
        # histogram_kernel.cu:36-59
        E, k, B = grad_hist.shape
        s = sample_indices.long().numpy()
        f = feature_indices.long().numpy()
        b = bin_indices.numpy()[s][:, f].astype(np.int64)
        e = era_indices.numpy()[s].astype(np.int64)
        g = residuals.numpy()[s].astype(np.float32)
        cell = (e[:, None] * k + np.arange(k)[None, :]) * B + b
        ok = (b >= 0) & (b < B)
        gflat = grad_hist.numpy().reshape(-1)
        hflat = hess_hist.numpy().reshape(-1)
        gv = np.broadcast_to(g[:, None], cell.shape)
        # np.add.at is unbuffered and applies updates in index order
        np.add.at(gflat, cell[ok], gv[ok])
        np.add.at(hflat, cell[ok], np.float32(1.0))

    @staticmethod
    def compute_split(G, H, min_split_gain, min_child_samples, eps, per_era_gain,
                      per_era_direction, threads=128):
        # best_split_kernel.cu:25-53, vectorised over (era, feature)
        E, k, B = G.shape
        mcw = torch.tensor(min_child_samples, dtype=torch.float32)
        ep = torch.tensor(eps, dtype=torch.float32)
        GT = torch.zeros(E, k)
        HT = torch.zeros(E, k)
        for b in range(B):
            GT = GT + G[:, :, b]
            HT = HT + H[:, :, b]
        GL = torch.zeros(E, k)
        HL = torch.zeros(E, k)
        for b in range(B - 1):
            GL = GL + G[:, :, b]
            HL = HL + H[:, :, b]
            GR = GT - GL
            HR = HT - HL
            ok = (HL >= mcw) & (HR >= mcw)
            t1 = (GL * GL) / (HL + ep)
            t2 = (GR * GR) / (HR + ep)
            t3 = (GT * GT) / (HT + ep)
            gain = (t1 + t2) - t3
            d = torch.where(GL / (HL + ep) > GR / (HR + ep), 1.0, -1.0)
            per_era_gain[:, :, b] = torch.where(ok, gain, torch.zeros(()))
            per_era_direction[:, :, b] = torch.where(ok, d, torch.zeros(()))

    @staticmethod
    def custom_cuda_binner(X, bin_edges, bin_indices):
        # binner.cu:16-25
        x = X.numpy()
        e = bin_edges.numpy()
        out = np.zeros(x.shape[0], np.int64)
        go = np.ones(x.shape[0], bool)
        for j in range(e.shape[0]):
            go &= x >= e[j]
            out += go
        bin_indices.copy_(torch.from_numpy(out.astype(np.int8)))

    @staticmethod
    def predict_forest(bin_indices, tree_tensor, learning_rate, out):
        # predict.cu:17-44, trees summed in tree order
        bins = bin_indices.numpy()
        tt = tree_tensor.numpy()
        o = out.numpy()
        lr = np.float32(learning_rate)
        n = bins.shape[0]
        rows = np.arange(n)
        for t in range(tt.shape[0]):
            node = np.zeros(n, np.int64)
            val = np.zeros(n, np.float32)
            active = np.ones(n, bool)
            while active.any():
                nd = tt[t][node]
                leaf = active & (nd[:, 4] > 0.5)
                val[leaf] = nd[leaf, 5]
                active &= ~leaf
                if not active.any():
                    break
                feat = np.where(active, nd[:, 0], 0).astype(np.int64)
                sb = np.where(active, nd[:, 1], 0).astype(np.int64)
                go_left = bins[rows, feat] <= sb
                nxt = np.where(go_left, nd[:, 2], nd[:, 3])
                node = np.where(active, nxt, node).astype(np.int64)
            o += np.float32(lr) * val


class _CpuTorch(types.ModuleType):
    """Stand-in for the ``torch`` name inside warpgbm.core: forwards
    everything, maps device='cuda' to 'cpu', and records randperm draws."""

    def __init__(self):
        super().__init__("torch")
        self.perms = []

    def __getattr__(self, name):
        fn = getattr(torch, name)
        if not callable(fn) or isinstance(fn, type):
            return fn

        def wrapped(*a, **kw):
            if str(kw.get("device", "")).startswith("cuda"):
                kw["device"] = "cpu"
            r = fn(*a, **kw)
            if name == "randperm":
                self.perms.append(r.numpy().copy())
            return r
        return wrapped


def load_reference(ref_root):
    sys.modules.pop("warpgbm", None)
    sys.modules.pop("warpgbm.core", None)
    sys.path.insert(0, ref_root)
    kern = _TorchKernels()
    cuda_pkg = types.ModuleType("warpgbm.cuda")
    cuda_pkg.node_kernel = kern
    cuda_pkg.__path__ = []
    sys.modules["warpgbm.cuda"] = cuda_pkg
    sys.modules["warpgbm.cuda.node_kernel"] = kern
    import warpgbm.core as core  # noqa: E402
    proxy = _CpuTorch()
    core.torch = proxy
    return core, proxy


def run_case(core, proxy, name, X, y, era, params, fit_kw=None, X_pred=None, save_model=None,
             write_npz=True):
    proxy.perms.clear()
    captured = {}

    class Recorder(core.WarpGBM):
        def preprocess_gpu_data(self, X_np, Y_np, era_id_np):
            out = super().preprocess_gpu_data(X_np, Y_np, era_id_np)
            captured["bins"] = out[0].numpy().copy()
            captured["edges"] = out[2].numpy().copy()
            captured["era_inv"] = out[1].numpy().astype(np.int32).copy()
            return out

    m = Recorder(device="cpu", **params)
    m.fit(X, y, era_id=era, **(fit_kw or {}))
    if save_model:  # the reference's own save_model (core.py:1103-1153)
        m.save_model(os.path.join(HERE, save_model))
    if not write_npz:
        return
    mx = 2 ** (m.max_depth + 1)
    if m.objective == "regression":
        flat = np.stack([m.flatten_tree(t, mx).numpy() for t in m.forest if t])
    else:
        flat = np.stack([m.flatten_tree(t, mx).numpy() for r in m.forest for t in r])
    Xp = X if X_pred is None else X_pred
    res = dict(
        X=X, y=y, era=era if era is not None else np.zeros(0, np.int32),
        bins=captured["bins"], edges=captured["edges"], era_inv=captured["era_inv"],
        forest=flat, imp=m.per_era_feature_importance_.astype(np.float32),
        perms=np.array(proxy.perms, np.int32) if proxy.perms else np.zeros(0, np.int32),
        params=np.array(repr(params)),
    )
    if X_pred is not None:
        res["X_pred"] = X_pred
    if fit_kw and "y_eval" in fit_kw:
        res["y_eval"] = fit_kw["y_eval"]
    if m.objective == "regression":
        res["base"] = np.float32(m.base_prediction)
        res["pred"] = m.predict(Xp).astype(np.float32)
    else:
        res["proba"] = m.predict_proba(Xp).astype(np.float32)
        res["labels"] = m.predict(Xp)
    if m.eval_loss:
        res["eval_loss"] = np.array(m.eval_loss, np.float64)
        res["training_loss"] = np.array(m.training_loss, np.float64)
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **res)
    print(f"wrote {path}: trees={flat.shape[0]} nodes/tree<={mx}")


def models(ref_root):
    """Pickles written by the reference's save_model (its tree dicts hold 0-d
    tensors in "feature" and the edges as a tensor): the C1 regression and
    the multiclass case, for the load-compatibility test."""
    core, proxy = load_reference(ref_root)
    torch.manual_seed(0)
    rng = np.random.default_rng(0)
    X = rng.standard_normal((4096, 16)).astype(np.float32)
    y = (2 * X[:, 0] - X[:, 1] + 0.5 * X[:, 2] * X[:, 3]
         + rng.normal(0, 0.1, 4096)).astype(np.float32)
    run_case(core, proxy, "c1_regression", X, y, None,
             dict(num_bins=32, max_depth=3, n_estimators=10, learning_rate=0.1, random_state=0),
             save_model="ref_model_c1.pkl", write_npz=False)
    rng = np.random.default_rng(3)
    n, F, K = 600, 8, 3
    lab = rng.integers(0, K, n)
    cent = rng.normal(0, 2, (K, F))
    X = (cent[lab] + rng.standard_normal((n, F))).astype(np.float32)
    run_case(core, proxy, "multiclass", X, lab.astype(np.int64), None,
             dict(objective="multiclass", num_bins=16, max_depth=3, n_estimators=4,
                  learning_rate=0.3, min_child_weight=5, random_state=3),
             save_model="ref_model_multiclass.pkl", write_npz=False)


def main(ref_root):
    core, proxy = load_reference(ref_root)
    torch.manual_seed(0)

    # C1 exactly
    rng = np.random.default_rng(0)
    X = rng.standard_normal((4096, 16)).astype(np.float32)
    y = (2 * X[:, 0] - X[:, 1] + 0.5 * X[:, 2] * X[:, 3]
         + rng.normal(0, 0.1, 4096)).astype(np.float32)
    run_case(core, proxy, "c1_regression", X, y, None,
             dict(num_bins=32, max_depth=3, n_estimators=10, learning_rate=0.1,
                  random_state=0))

    # era-aware DES regression, shuffled era order, float input
    rng = np.random.default_rng(1)
    n, F, E = 3000, 12, 4
    era = rng.integers(0, E, n).astype(np.int32) * 7 + 3   # sparse era ids
    X = rng.standard_normal((n, F)).astype(np.float32)
    sign = np.where((era // 7) % 2 == 0, 1.0, -1.0)
    y = (X[:, 0] + sign * X[:, 1] + 0.3 * rng.standard_normal(n)).astype(np.float32)
    run_case(core, proxy, "era_des", X, y, era,
             dict(num_bins=16, max_depth=4, n_estimators=8, learning_rate=0.2,
                  min_child_weight=10, random_state=1))

    # pre-binned int8, contiguous eras, colsample < 1 (randperm recorded)
    rng = np.random.default_rng(2)
    n, F = 2000, 10
    X = rng.integers(0, 8, (n, F)).astype(np.int8)
    era = np.repeat(np.arange(3), [700, 600, 700]).astype(np.int32)
    y = (X[:, 0] * 0.5 - X[:, 3] + rng.standard_normal(n)).astype(np.float32)
    run_case(core, proxy, "prebinned_colsample", X, y, era,
             dict(num_bins=8, max_depth=3, n_estimators=5, learning_rate=0.3,
                  colsample_bytree=0.6, min_child_weight=5, random_state=2))

    # multiclass, float input
    rng = np.random.default_rng(3)
    n, F, K = 600, 8, 3
    lab = rng.integers(0, K, n)
    cent = rng.normal(0, 2, (K, F))
    X = (cent[lab] + rng.standard_normal((n, F))).astype(np.float32)
    run_case(core, proxy, "multiclass", X, lab.astype(np.int64), None,
             dict(objective="multiclass", num_bins=16, max_depth=3, n_estimators=4,
                  learning_rate=0.3, min_child_weight=5, random_state=3))

    # binary with string labels
    rng = np.random.default_rng(4)
    n, F = 500, 6
    X = rng.standard_normal((n, F)).astype(np.float32)
    lab = np.where(X[:, 0] + 0.5 * X[:, 1] > 0, "yes", "no")
    run_case(core, proxy, "binary", X, lab, None,
             dict(objective="binary", num_bins=8, max_depth=2, n_estimators=3,
                  learning_rate=0.5, min_child_weight=5))

    # binning edge cases: ties, constant, NaN, inf, tiny magnitudes
    rng = np.random.default_rng(5)
    n = 257
    cols = [
        rng.integers(0, 3, n).astype(np.float32),          # heavy ties
        np.full(n, 1.5, np.float32),                       # constant
        rng.standard_normal(n).astype(np.float32),         # plain
        np.where(rng.random(n) < 0.02, np.nan, rng.standard_normal(n)).astype(np.float32),
        np.where(rng.random(n) < 0.05, np.inf, rng.standard_normal(n)).astype(np.float32),
        (rng.standard_normal(n) * 1e-30).astype(np.float32),
        np.concatenate([np.zeros(n // 2), -np.zeros(n - n // 2)]).astype(np.float32),
    ]
    X = np.stack(cols, axis=1)
    y = rng.standard_normal(n).astype(np.float32)
    run_case(core, proxy, "binning_edges", X, y, None,
             dict(num_bins=7, max_depth=1, n_estimators=1, learning_rate=0.1,
                  min_child_weight=1))

    # eval set + early stopping (regression, corr metric)
    rng = np.random.default_rng(6)
    n, F = 1500, 8
    X = rng.standard_normal((n, F)).astype(np.float32)
    y = (X[:, 0] - 2 * X[:, 1] + rng.standard_normal(n)).astype(np.float32)
    run_case(core, proxy, "eval_corr", X[:1000], y[:1000], None,
             dict(num_bins=16, max_depth=3, n_estimators=12, learning_rate=0.3),
             fit_kw=dict(X_eval=X[1000:], y_eval=y[1000:], eval_every_n_trees=2,
                         early_stopping_rounds=3, eval_metric="corr"),
             X_pred=X[1000:])


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    root = args[0] if args else os.environ.get("WGB_REFERENCE")
    if not root:
        sys.exit("usage: make_golden.py /path/to/reference [--models]  (or set WGB_REFERENCE)")
    if "--models" in sys.argv:
        models(root)
    else:
        main(root)
        models(root)
