"""The CPU oracle against the reference's own outputs (tests/golden/*.npz,
made by tests/golden/make_golden.py from warpgbm/core.py) and against torch.
No GPU needed."""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import GOLDEN_CASES, load_golden


def _fit(d, params, mode):
    params = dict(params)
    params.pop("random_state", None)
    era = d["era"] if d["era"].size else None
    subs = None
    if d["perms"].size:
        F = d["X"].shape[1]
        kk = max(1, int(params["colsample_bytree"] * F))
        subs = [p[:kk] for p in d["perms"]]
    return O.OracleGBM(mode=mode, **params).fit(d["X"], d["y"], era_id=era, feature_subsets=subs)


def _same_forest(a, b):
    return a.shape == b.shape and np.array_equal(np.nan_to_num(a, nan=-7.0), np.nan_to_num(b, nan=-7.0))


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_reference_mode_reproduces_reference_exactly(case):
    d, params = load_golden(case)
    m = _fit(d, params, "reference")
    assert np.array_equal(m.bins, d["bins"])
    assert np.array_equal(m.bin_edges, d["edges"], equal_nan=True)
    assert np.array_equal(m.era, d["era_inv"])
    assert _same_forest(m.flat_forest(), d["forest"])
    assert np.array_equal(m.per_era_feature_importance_, d["imp"])
    Xp = d["X_pred"] if "X_pred" in d else d["X"]
    if "pred" in d:
        assert np.float32(m.base_prediction) == d["base"]
        assert np.array_equal(m.predict(Xp), d["pred"])
    else:
        assert np.array_equal(m.predict_proba(Xp), d["proba"])
        assert np.array_equal(m.predict(Xp), d["labels"])


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_canonical_mode_within_tolerance_of_reference(case):
    """The product's arithmetic (exact fixed-point histograms) against the
    reference: same trees except at ties decided by fp32 noise, predictions
    within 1e-5 relative."""
    d, params = load_golden(case)
    m = _fit(d, params, "canonical")
    Xp = d["X_pred"] if "X_pred" in d else d["X"]
    if "pred" in d:
        assert _same_forest(m.flat_forest()[..., :5], d["forest"][..., :5])
        p = m.predict(Xp)
        scale = np.abs(d["pred"]).max()
        assert np.abs(p - d["pred"]).max() <= 1e-5 * scale
        np.testing.assert_allclose(m.flat_forest()[..., 5], d["forest"][..., 5], rtol=1e-5, atol=1e-6)
    else:
        # the first boosting round of the multiclass case holds pure nodes whose best "gain"
        # is fp32 rounding noise (~1e-5 vs terms ~30); either arithmetic may
        # pick a different noise split there.  Probabilities stay close.
        p = m.predict_proba(Xp)
        assert np.abs(p - d["proba"]).max() < 2e-3


def test_linspace_formula_matches_torch():
    for B in range(2, 128):
        q = torch.linspace(0, 1, B + 1, dtype=torch.float32)[1:-1].numpy()
        assert np.array_equal(O.linspace_q(B), q), B


@pytest.mark.parametrize("seed", range(4))
def test_quantile_matches_torch(seed):
    rng = np.random.default_rng(seed)
    for trial in range(40):
        n = int(rng.integers(1, 3000))
        kind = trial % 5
        if kind == 0:
            col = rng.standard_normal(n)
        elif kind == 1:
            col = rng.integers(0, 4, n).astype(float)
        elif kind == 2:
            col = np.where(rng.random(n) < 0.1, np.nan, rng.standard_normal(n))
        elif kind == 3:
            col = np.where(rng.random(n) < 0.1, np.inf, rng.standard_normal(n) * 1e-20)
        else:
            col = rng.exponential(1e5, n)
        col = col.astype(np.float32)
        B = int(rng.integers(2, 128))
        q = O.linspace_q(B)
        ref = torch.quantile(torch.from_numpy(col), torch.from_numpy(q)).numpy()
        assert np.array_equal(O.quantile_edges(col, q), ref, equal_nan=True)


def test_split_matches_torch_restatement():
    """orc_split against the independent torch restatement of
    best_split_kernel.cu used to generate the fixtures."""
    import importlib.util
    import os
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(os.path.dirname(__file__), "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    rng = np.random.default_rng(7)
    for E, k, B in [(1, 50, 32), (3, 17, 5), (5, 9, 127), (2, 4, 2)]:
        H = rng.integers(0, 60, (E, k, B)).astype(np.float32)
        G = (rng.standard_normal((E, k, B)) * H).astype(np.float32)
        gain, d = O.split(G, H, 20, 1e-6)
        tg = torch.zeros(E, k, B - 1)
        td = torch.zeros(E, k, B - 1)
        mg._TorchKernels.compute_split(torch.from_numpy(G), torch.from_numpy(H), 0.0, 20, 1e-6, tg, td)
        assert np.array_equal(gain, tg.numpy())
        assert np.array_equal(d, td.numpy())


def test_des_rule_semantics():
    """core.py:577-594 corner cases."""
    # E == 1: first maximum wins, crit must exceed min_split_gain
    gain = np.array([[[0.0, 2.0, 2.0], [1.0, 2.0, 0.5]]], np.float32)
    d = np.ones_like(gain)
    assert O.des_pick(gain, d, 0.0, 0) == 1
    assert O.des_pick(gain, d, 2.0, 0) == -1
    # E == 2: maximum agreement is taken over every cell before the gain mask
    gain = np.array([[[5.0, 1.0]], [[5.0, 1.0]]], np.float32)
    d = np.array([[[1.0, 1.0]], [[-1.0, 1.0]]], np.float32)
    assert O.des_pick(gain, d, 0.0, 0) == 1       # agreement 1 beats gain 5
    assert O.des_pick(gain, d, 1.0, 0) == -1      # max-agreement cell masked by gain
    assert O.des_pick(gain, d, 0.0, 1) == 1


def test_quantisation_grid():
    assert O.quant_shift(0.0) == 0
    assert O.quant_shift(1.0) == 28          # 1 = 0.5 * 2^1
    assert O.quant_shift(0.75) == 29
    assert O.quant_shift(1e-38) == 126       # clamp
    g = np.array([0.3, -0.3, 1.0, -1.0, 0.75], np.float32)
    s = O.quant_shift(float(np.abs(g).max()))
    q = O.quantize(g, s)
    assert np.abs(q).max() <= 2 ** 29
    assert q[2] == 2 ** 28 and q[3] == -(2 ** 28)


def test_canonical_histogram_is_exact_and_subtractive():
    rng = np.random.default_rng(3)
    n, F, B, E = 5000, 23, 9, 3
    bins = rng.integers(-2, B + 2, (n, F)).astype(np.int8)
    g = rng.standard_normal(n).astype(np.float32)
    era = rng.integers(0, E, n).astype(np.int32)
    s = O.quant_shift(float(np.abs(g).max()))
    q = O.quantize(g, s)
    feats = rng.permutation(F)[:11].astype(np.int32)
    rows = np.arange(n, dtype=np.int32)
    G, C = O.hist_q(bins, q, rows, feats, era, E, B)
    left = rows[rows % 3 == 0]
    right = rows[rows % 3 != 0]
    GL, CL = O.hist_q(bins, q, left, feats, era, E, B)
    GR, CR = O.hist_q(bins, q, right, feats, era, E, B)
    assert np.array_equal(G - GL, GR) and np.array_equal(C - CL, CR)
    # negative bins land in slot B, bins >= B nowhere
    for j, f in enumerate(feats):
        for e in range(E):
            m = era == e
            assert C[e, j, B] == np.sum(bins[m, f] < 0)
            assert C[e, j].sum() == np.sum(bins[m, f] < B)
            assert G[e, j].sum() == q[m & (bins[:, f] < B)].astype(np.int64).sum()
