"""Host-side tree decoding (no GPU): the vectorised per-level decode of the
engine's level-packed node records must give the same nested-dict trees,
the same predict packing and the same pre-order importance accumulation as
a plain depth-first walk (the order warpgbm/core.py:624-627 adds gains in)."""
import numpy as np
import pytest

from warpgbm_b200 import _lib
from warpgbm_b200.core import compact_tree, pack_trees, tree_dict


def _records(rng, D, E, F, p_split):
    """Random records in the engine's layout: level d packed at
    [2^d - 1, 2^(d+1) - 1), children of the r-th splitting node of a level
    at 2r, 2r+1 of the next; unused slots hold stale garbage."""
    nn = (1 << (D + 1)) - 1
    nodes = np.zeros(nn, dtype=_lib.NODE_DTYPE)
    nodes["fpos"] = rng.integers(0, F, nn)          # stale entries look like splits
    nodes["child"] = rng.integers(0, 4, nn)
    nodes["bin"] = rng.integers(0, 31, nn)
    nodes["leaf"] = rng.standard_normal(nn).astype(np.float32)
    nodes["count"] = rng.integers(1, 10 ** 6, nn)
    gains = rng.random(((1 << D) - 1) * E).astype(np.float32)
    real = 1
    for d in range(D + 1):
        nsplit = 0
        for r in range(real):
            i = (1 << d) - 1 + r
            if d < D and rng.random() < p_split:
                nodes[i]["fpos"] = rng.integers(0, F)
                nodes[i]["child"] = 2 * nsplit
                nsplit += 1
            else:
                nodes[i]["fpos"] = -1
        real = 2 * nsplit
    return nodes, gains


def _walk(nodes, gains, feats, D, E, imp):
    def rec(d, n):
        nd = nodes[(1 << d) - 1 + n]
        if d < D and nd["fpos"] >= 0:
            gfi = int(feats[nd["fpos"]])
            g0 = ((1 << d) - 1 + n) * E
            imp[:, gfi] += gains[g0:g0 + E]
            return {"feature": gfi, "bin": int(nd["bin"]),
                    "left": rec(d + 1, int(nd["child"])), "right": rec(d + 1, int(nd["child"]) + 1)}
        return {"leaf_value": float(nd["leaf"]), "samples": int(nd["count"])}
    return rec(0, 0)


@pytest.mark.parametrize("D,E,p", [(1, 1, 1.0), (5, 1, 0.8), (10, 1, 0.97), (8, 3, 0.7), (4, 1, 0.0), (12, 2, 0.9)])
def test_vectorised_decode_matches_depth_first_walk(D, E, p):
    rng = np.random.default_rng(D * 100 + E)
    F = 40
    feats = rng.permutation(F).astype(np.int32)
    for _ in range(3):
        nodes, gains = _records(rng, D, E, F, p)
        imp_ref = np.zeros((E, F), np.float32)
        want = _walk(nodes, gains, feats, D, E, imp_ref)
        packed, leaf, samples, sp_pre, sp_feat, sp_gain = compact_tree(nodes, gains, feats, D, E)
        assert tree_dict(packed, leaf, samples) == want
        assert np.array_equal(packed, pack_trees([want])[0])
        imp = np.zeros((E, F), np.float32)
        if len(sp_feat):
            np.add.at(imp, (slice(None), sp_feat), sp_gain.T)
        assert np.array_equal(imp, imp_ref)


def test_forest_dicts_built_on_first_access_and_packing_without_them():
    """fit() keeps compact pre-order arrays and a lazy marker; the nested-dict
    forest (the reference's format) is built only when `forest` is read, and
    the predict packing never needs it."""
    from warpgbm_b200 import WarpGBM
    rng = np.random.default_rng(3)
    D, E, F = 4, 1, 12
    feats = np.arange(F, dtype=np.int32)
    m = WarpGBM(n_estimators=3, max_depth=D)
    want, packs = [], []
    for i in range(2):                                  # two trained trees, one untrained slot
        nodes, gains = _records(rng, D, E, F, 0.8)
        want.append(_walk(nodes, gains, feats, D, E, np.zeros((E, F), np.float32)))
        comp = compact_tree(nodes, gains, feats, D, E)
        m._compact[(i, 0)] = comp[:3]
        m._lazy.add((i, 0))
        packs.append(comp[0])
    assert m._tree_slots() == [(0, 0), (1, 0)]
    assert m.__dict__["_forest"][0] == {}              # not yet materialised
    assert (0, 0) in m._lazy
    f = m.forest
    assert f[0] == want[0] and f[1] == want[1] and f[2] == {}
    assert not m._lazy                                  # built once
    nodes_all, offs = pack_trees([t for t in f if t])
    assert np.array_equal(nodes_all, np.concatenate(packs))
    m.forest = [{} for _ in range(3)]                   # assignment drops the compact arrays
    assert m._compact == {} and m._tree_slots() == []
