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


def _node_fields(raw):
    """lstart, lcnt, built of 64-byte wgb_node records (include/warpgbm_b200.h)."""
    i32 = raw.view(np.int32)
    return i32[:, 8], i32[:, 9], i32[:, 11]


@pytest.mark.parametrize("n,F", [(300_000, 300), (70_000, 1000), (5_000, 40)])
def test_level_chunks_cover_built_rows_once(cuda, n, F):
    """The histogram chunk list of every level (sized so that the chunks fill
    whole waves of the histogram kernel's CTA slots): each built node's local
    rows [lstart, lstart + lcnt) are cut into consecutive pieces of equal size
    (within one row), none above 2048 rows, and into no more pieces than a
    1024-row target gives; nothing else is listed.  The trees stay bit-exact."""
    X, y = _data(n, F, 3)
    params = dict(num_bins=32, max_depth=5, n_estimators=2, learning_rate=0.3)
    m = WarpGBM(**params)
    m._chunk_log = []
    m.fit(X, y)
    assert m._chunk_log
    for d, ch, raw, nn in m._chunk_log:
        lstart, lcnt, built = _node_fields(raw[:nn])
        want = {i for i in range(nn) if built[i] & 1 and lcnt[i] > 0}
        assert set(ch[:, 0].tolist()) == want, d
        for i in want:
            pieces = ch[ch[:, 0] == i]
            lo, hi = pieces[:, 1], pieces[:, 2]
            assert lo[0] == lstart[i] and hi[-1] == lstart[i] + lcnt[i], (d, i)
            assert np.array_equal(lo[1:], hi[:-1]), (d, i)  # consecutive, no gap or overlap
            size = hi - lo
            assert size.max() <= 2048 and size.max() - size.min() <= 1, (d, i, size)
            assert len(size) <= -(-int(lcnt[i]) // 1024), (d, i, size)  # pieces of >= 1024 rows' target
    o = _oracle_for(m, params, X, y, None)
    assert _same(_flat(m, 5), o.flat_forest())
