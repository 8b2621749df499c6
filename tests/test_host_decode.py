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


@pytest.mark.parametrize("D,E,p,ntree", [(1, 1, 1.0, 1), (5, 1, 0.8, 1), (10, 1, 0.97, 1), (8, 3, 0.7, 1),
                                         (4, 1, 0.0, 1), (6, 1, 0.9, 5), (3, 2, 0.8, 3)])
def test_library_decode_matches_numpy_decode(D, E, p, ntree):
    """wgb_decode_tree (the library's host decode the fit uses) gives the
    same pre-order arrays and the same fp32 importance sums as compact_tree
    and the depth-first walk, for every tree of a batch grown together."""
    import ctypes
    rng = np.random.default_rng(D * 10 + ntree)
    F = 40
    feats = rng.permutation(F).astype(np.int32)
    # a batch of ntree trees: level d of the batch = the trees' level-d records in tree order
    recs = [_records(rng, D, E, F, p) for _ in range(ntree)]
    levels, gl = [], []
    for d in range(D + 1):
        for t, (nodes, gains) in enumerate(recs):
            lv = nodes[(1 << d) - 1:(1 << (d + 1)) - 1].copy()
            lv["child"] = np.where(lv["fpos"] >= 0, lv["child"] + t * (1 << (d + 1)), lv["child"])
            levels.append(lv)
            if d < D:
                gl.append(gains.reshape(-1, E)[(1 << d) - 1:(1 << (d + 1)) - 1])
    batch = np.ascontiguousarray(np.concatenate(levels))
    bgain = np.ascontiguousarray(np.concatenate(gl).reshape(-1).astype(np.float32))
    cap = (1 << (D + 1)) - 1
    L = _lib.lib()
    for t, (nodes, gains) in enumerate(recs):
        imp_ref = np.zeros((E, F), np.float32)
        want = _walk(nodes, gains, feats, D, E, imp_ref)
        packed = np.empty((cap, 2), np.int32)
        leaf = np.empty(cap, np.float32)
        samples = np.empty(cap, np.int64)
        imp = np.zeros((E, F), np.float32)
        n = L.wgb_decode_tree(batch.ctypes.data, D, ntree, t, feats.ctypes.data, bgain.ctypes.data, E,
                              imp.ctypes.data, F, packed.ctypes.data, leaf.ctypes.data, samples.ctypes.data, cap)
        assert n > 0
        assert tree_dict(packed[:n], leaf[:n], samples[:n]) == want
        assert np.array_equal(imp, imp_ref)
        pk, lf, sm, *_ = compact_tree(batch, bgain, feats, D, E, ntree, t)
        assert np.array_equal(pk, packed[:n]) and np.array_equal(sm, samples[:n])
    # malformed records are rejected, not followed
    bad = batch.copy()
    bad["child"][0] = 1 << 20
    bad["fpos"][0] = 0
    assert L.wgb_decode_tree(bad.ctypes.data, D, ntree, 0, feats.ctypes.data, None, E, None, F,
                             packed.ctypes.data, leaf.ctypes.data, samples.ctypes.data, cap) < 0


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


def _predict_dict(tree, row):
    while "leaf_value" not in tree:
        tree = tree["left"] if row[tree["feature"]] <= tree["bin"] else tree["right"]
    return np.float32(tree["leaf_value"])


def _predict_heap(H, D, row):
    node = 0
    for _ in range(D):
        w = int(H[node])
        f, sb = w & 0xFFFF, np.int8(np.uint8((w >> 16) & 0xFF))
        node = 2 * node + 1 + (1 if row[f] > sb else 0)
    return np.uint32(H[node + 1]).view(np.float32)


@pytest.mark.parametrize("D,p", [(1, 1.0), (3, 0.6), (6, 0.9), (10, 0.97), (12, 0.5), (5, 0.0)])
def test_heap_layout_walks_like_the_dict_trees(D, p):
    """heap_forest (the wgb_predict_heap layout: complete binary trees,
    early leaves as pass-through chains) reaches the same leaf as the
    nested-dict tree for every row, negative int8 bins included."""
    from warpgbm_b200.core import heap_forest
    rng = np.random.default_rng(D * 10 + int(p * 10))
    F = 40
    trees = []
    for t in range(4):
        nodes, gains = _records(rng, D, 1, F, p)
        feats = rng.permutation(F).astype(np.int32)
        packed, leaf, samples, *_ = compact_tree(nodes, gains, feats, D, 1)
        trees.append((packed, tree_dict(packed, leaf, samples)))
    H = heap_forest([pk for pk, _ in trees], D)
    assert H.shape == (4, 2 << D)
    rows = rng.integers(-5, 32, (300, F)).astype(np.int8)
    for t, (_, tree) in enumerate(trees):
        for row in rows:
            assert _predict_heap(H[t], D, row) == _predict_dict(tree, row)


def test_heap_layout_rejects_what_it_cannot_hold():
    from warpgbm_b200.core import heap_forest
    deep, _ = pack_trees([{"feature": 1, "bin": 0, "left": {"leaf_value": 1.0, "samples": 1},
                           "right": {"feature": 2, "bin": 3, "left": {"leaf_value": 2.0, "samples": 1},
                                     "right": {"leaf_value": 3.0, "samples": 1}}}])
    assert heap_forest([deep], 1) is None                 # deeper than D
    wide, _ = pack_trees([{"feature": 70000, "bin": 0, "left": {"leaf_value": 1.0, "samples": 1},
                           "right": {"leaf_value": 2.0, "samples": 1}}])
    assert heap_forest([wide], 3) is None                 # feature index beyond 16 bits
