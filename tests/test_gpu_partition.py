"""One-launch level partition (k_partition) of single-rank one-era fits on
the B200: trees and predictions stay bit-exact against the oracle.

The kernel writes each child's rows in whatever order the tiles reserve
their ranges (one global atomic per node, side and tile), so these cases
exercise what that order could break: row counts around the 2048-position
tile, many tiles sharing a node's cursors, deep trees whose node ids jump
past a tile's range (the per-row atomic fallback), and a multiclass batch
(K trees partitioned in one launch)."""
import numpy as np
import pytest

from test_gpu_engine import _flat, _oracle_for, _same
from warpgbm_b200 import WarpGBM

pytestmark = pytest.mark.gpu


def _data(n, F, seed):
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, F)).astype(np.float32)
    y = (X[:, 0] - 0.5 * X[:, 1] + rng.normal(0, 0.1, n)).astype(np.float32)
    return X, y


@pytest.mark.parametrize("n", [1, 2047, 2048, 2049, 3 * 2048 + 5, 70_000])
def test_tile_boundaries_bit_exact(cuda, n):
    X, y = _data(n, 5, n)
    params = dict(num_bins=8, max_depth=5, n_estimators=2, learning_rate=0.3)
    m = WarpGBM(**params).fit(X, y)
    o = _oracle_for(m, params, X, y, None)
    assert _same(_flat(m, 5), o.flat_forest())
    assert np.array_equal(m.predict(X), o.predict(X))


def test_deep_sparse_nodes_bit_exact(cuda):
    """Depth 12 with min_child_weight 1: thousands of node ids per level,
    many of them leaves, so one tile's splitting nodes can lie far apart."""
    X, y = _data(30_000, 6, 11)
    params = dict(num_bins=64, max_depth=12, n_estimators=2, learning_rate=0.3, min_child_weight=1)
    m = WarpGBM(**params).fit(X, y)
    o = _oracle_for(m, params, X, y, None)
    assert _same(_flat(m, 12), o.flat_forest())
    assert np.array_equal(m.predict(X), o.predict(X))


def test_multiclass_batch_bit_exact(cuda):
    rng = np.random.default_rng(5)
    n, F, K = 9000, 7, 4
    X = rng.standard_normal((n, F)).astype(np.float32)
    y = (np.argmax(X[:, :K] + rng.normal(0, 0.5, (n, K)), axis=1)).astype(np.int64)
    params = dict(num_bins=16, max_depth=4, n_estimators=3, learning_rate=0.2, objective="multiclass")
    m = WarpGBM(**params)
    m._record_residuals = True
    m.fit(X, y)
    o = _oracle_for(m, params, X, y, None)
    assert _same(_flat(m, 4, classification=True), o.flat_forest())
    assert np.abs(m.predict_proba(X) - o.predict_proba(X)).max() < 1e-6
