"""Kernel-level parity: every C-ABI operation against the CPU oracle on the
same seeded inputs.  Integer / index results bit-exact; fp32 results
bit-exact where the arithmetic is the same, otherwise with the stated
tolerance."""
import numpy as np
import pytest
import torch

import oracle as O
from warpgbm_b200 import _lib, node_kernel
from warpgbm_b200.core import bins_stride

pytestmark = pytest.mark.gpu


def _st():
    return torch.cuda.current_stream().cuda_stream


def _edges_for(X, B, dev):
    Xd = torch.from_numpy(X).to(dev)
    q = torch.linspace(0, 1, B + 1, device=dev, dtype=torch.float32)[1:-1]
    return torch.quantile(Xd, q, dim=0).T.contiguous()


@pytest.mark.parametrize("n,F,B", [(1000, 13, 32), (4097, 128, 7), (3000, 300, 127), (17, 1, 2)])
def test_bin_matrix_matches_oracle(cuda, n, F, B):
    rng = np.random.default_rng(n + F)
    X = rng.standard_normal((n, F)).astype(np.float32)
    X[rng.random((n, F)) < 0.01] = np.nan
    if F > 2:
        X[:, 1] = np.round(X[:, 1])          # ties
        X[:, 2] = 3.0                        # constant
    edges = _edges_for(X, B, cuda)
    S = bins_stride(F)
    out = torch.full((n, S), 99, dtype=torch.int8, device=cuda)
    Xd = torch.from_numpy(X).to(cuda)
    _lib.call("wgb_bin_matrix", Xd.data_ptr(), n, F, F, edges.data_ptr(), B, out.data_ptr(), S, _st())
    got = out.cpu().numpy()
    ref = O.bin_matrix(X, edges.cpu().numpy())
    assert np.array_equal(got[:, :F], ref)
    assert (got[:, F:] == 0).all()


@pytest.mark.parametrize("F,xs", [(64, 64), (61, 61), (40, 45), (300, 300)])
@pytest.mark.parametrize("B", [2, 4, 9, 16, 32, 64, 127])
def test_bin_matrix_edge_lists(cuda, F, xs, B):
    """Binning against the oracle's leading-edge scan for edge lists of every
    shape: sorted, with ties, with infinities, unsorted, all-NaN, one NaN;
    aligned (16-byte row loads) and unaligned rows."""
    rng = np.random.default_rng(F * 1000 + B)
    n, nb = 3001, B - 1
    Xw = rng.standard_normal((n, xs)).astype(np.float32) * 2
    Xw[rng.random((n, xs)) < 0.02] = np.nan
    Xw[rng.random((n, xs)) < 0.02] = np.inf
    Xw[rng.random((n, xs)) < 0.02] = -np.inf
    Xw[rng.random((n, xs)) < 0.05] = 0.0
    edges = np.sort(rng.standard_normal((F, nb)).astype(np.float32) * 2, axis=1)
    for f in range(F):
        kind = f % 6
        if kind == 1:
            edges[f] = np.round(edges[f])                        # ties
        elif kind == 2:
            edges[f, : nb // 3] = -np.inf                        # infinities
            edges[f, nb - nb // 4:] = np.inf
        elif kind == 3 and nb > 1:
            edges[f] = rng.permutation(edges[f])                 # unsorted
        elif kind == 4:
            edges[f] = np.nan                                    # all NaN
        elif kind == 5 and nb > 2:
            edges[f, nb // 2] = np.nan                           # one NaN
    S = bins_stride(F)
    out = torch.full((n, S), 99, dtype=torch.int8, device=cuda)
    Xd = torch.from_numpy(Xw).to(cuda)
    ed = torch.from_numpy(edges).to(cuda)
    _lib.call("wgb_bin_matrix", Xd.data_ptr(), n, F, xs, ed.data_ptr(), B, out.data_ptr(), S, _st())
    got = out.cpu().numpy()
    ref = O.bin_matrix(np.ascontiguousarray(Xw[:, :F]), edges)
    assert np.array_equal(got[:, :F], ref)
    assert (got[:, F:] == 0).all()


@pytest.mark.parametrize("n,F", [(5000, 64), (3001, 37), (700, 130), (0, 9), (1, 1)])
def test_prebinned_ingest(cuda, n, F):
    """One-pass pre-binned copy: padded bins, per-column maxima (the reference's
    pre-binned test, core.py:499-502) and global min / max."""
    rng = np.random.default_rng(n + F)
    X = rng.integers(-5, 40, (n, F)).astype(np.int8)
    S = bins_stride(F)
    out = torch.full((max(n, 1), S), 99, dtype=torch.int8, device=cuda)
    colmax = torch.zeros(F, dtype=torch.int32, device=cuda)
    minmax = torch.zeros(2, dtype=torch.int32, device=cuda)
    Xd = torch.from_numpy(X).to(cuda)
    _lib.call("wgb_prebinned_ingest", Xd.data_ptr() if n else 0, n, F, F, out.data_ptr(), S,
              colmax.data_ptr(), minmax.data_ptr(), _st())
    if n == 0:
        assert (colmax.cpu().numpy() < -128).all()
        mm = minmax.cpu().numpy()
        assert mm[0] > 127 and mm[1] < -128
        return
    got = out.cpu().numpy()
    assert np.array_equal(got[:, :F], X)
    assert (got[:, F:] == 0).all()
    assert np.array_equal(colmax.cpu().numpy(), X.max(axis=0).astype(np.int32))
    assert list(minmax.cpu().numpy()) == [int(X.min()), int(X.max())]


def test_torch_cuda_quantile_equals_oracle(cuda):
    """Pins the oracle's quantile restatement (FMA lerp, linspace formula) to
    torch.quantile on the B200 -- the op the reference calls at core.py:532."""
    rng = np.random.default_rng(11)
    for B in (2, 5, 10, 32, 127):
        qd = torch.linspace(0, 1, B + 1, device=cuda, dtype=torch.float32)[1:-1]
        assert np.array_equal(qd.cpu().numpy(), O.linspace_q(B))
        for trial in range(20):
            n = int(rng.integers(1, 20000))
            col = rng.standard_normal(n).astype(np.float32) * float(rng.exponential(10))
            if trial % 4 == 1:
                col = np.round(col)
            if trial % 4 == 2:
                col[rng.random(n) < 0.05] = np.nan
            ref = torch.quantile(torch.from_numpy(col).to(cuda), qd).cpu().numpy()
            assert np.array_equal(O.quantile_edges(col, O.linspace_q(B)), ref, equal_nan=True)


def test_custom_cuda_binner_matches_oracle(cuda):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(10001).astype(np.float32)
    x[::97] = np.nan
    e = np.sort(rng.standard_normal(9)).astype(np.float32)
    out = torch.empty(x.size, dtype=torch.int8, device=cuda)
    node_kernel.custom_cuda_binner(torch.from_numpy(x).to(cuda), torch.from_numpy(e).to(cuda), out)
    ref = O.bin_matrix(x[:, None], e[None, :])[:, 0]
    assert np.array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("E,k,B", [(1, 1000, 32), (4, 37, 5), (2, 9, 127), (3, 3, 2)])
def test_compute_split_bit_exact(cuda, E, k, B):
    rng = np.random.default_rng(E * k + B)
    H = rng.integers(0, 80, (E, k, B)).astype(np.float32)
    G = (rng.standard_normal((E, k, B)) * H * 0.37).astype(np.float32)
    gain = torch.empty((E, k, B - 1), device=cuda)
    d = torch.empty_like(gain)
    node_kernel.compute_split(torch.from_numpy(G).to(cuda), torch.from_numpy(H).to(cuda), 0.0, 20,
                              1e-6, gain, d)
    rg, rd = O.split(G, H, 20, 1e-6)
    assert np.array_equal(gain.cpu().numpy(), rg)
    assert np.array_equal(d.cpu().numpy(), rd)


@pytest.mark.parametrize("n,F,k,E,B,sorted_eras", [
    (50000, 300, 200, 1, 32, True),
    (20000, 61, 61, 3, 10, False),      # unaligned rows (F % 4 != 0), unsorted eras
    (30000, 40, 20, 37, 5, True),
    # 8 features per lane (row stride % 8 == 0, > 128 features) with eras:
    # 4 era slots of 8 bin slots, 2 era slots of 34, unsorted eras
    (40000, 264, 150, 7, 5, True),
    (20000, 264, 200, 4, 32, True),
    (20000, 136, 136, 3, 10, False),
    (777, 8, 8, 1, 2, True),
    (0, 8, 8, 1, 4, True),
])
def test_compute_histogram3(cuda, n, F, k, E, B, sorted_eras):
    rng = np.random.default_rng(n + F + E)
    N = max(n, 1) + 5
    bins = rng.integers(-1, B + 1, (N, F)).astype(np.int8)   # includes skipped bins
    g = (rng.standard_normal(N) * 3).astype(np.float32)
    era = rng.integers(0, E, N).astype(np.int32)
    samples = rng.permutation(N)[:n].astype(np.int32)
    if sorted_eras:
        samples = samples[np.argsort(era[samples], kind="stable")]
    feats = rng.permutation(F)[:k].astype(np.int32)
    Gd = torch.zeros((E, k, B), device=cuda)
    Hd = torch.zeros((E, k, B), device=cuda)
    node_kernel.compute_histogram3(
        torch.from_numpy(bins).to(cuda), torch.from_numpy(g).to(cuda),
        torch.from_numpy(samples).to(cuda), torch.from_numpy(feats).to(cuda),
        torch.from_numpy(era).to(cuda), Gd, Hd, B, 64, 4)
    Gg, Hg = Gd.cpu().numpy(), Hd.cpu().numpy()
    if n == 0:
        assert not Gg.any() and not Hg.any()
        return
    # canonical: exact sums on the grid of max|g| over the sampled rows
    s = O.quant_shift(float(np.abs(g[samples]).max()))
    Gq, Cq = O.hist_q(bins, O.quantize(g, s), samples, feats, era, E, B)
    Gf, Hf = O.dequant(Gq, Cq, s)
    assert np.array_equal(Hg, Hf)
    assert np.array_equal(Gg, Gf)
    # reference semantics: fp32 sums, within 1e-5 of the bin's sum |g|
    Gr, Hr = O.hist_ref(bins, g, samples, feats, era, E, B)
    Ga, _ = O.hist_ref(bins, np.abs(g), samples, feats, era, E, B)
    assert np.array_equal(Hg, Hr)
    assert (np.abs(Gg - Gr) <= 1e-5 * Ga + 1e-30).all()


def test_predict_forest_flat_matches_oracle(cuda):
    rng = np.random.default_rng(2)
    d = np.load("tests/golden/c1_regression.npz")
    forest = d["forest"]
    bins = d["bins"]
    out = torch.full((bins.shape[0],), 0.25, device=cuda)
    node_kernel.predict_forest(torch.from_numpy(bins).to(cuda), torch.from_numpy(forest).to(cuda), 0.1, out)
    ref = np.full(bins.shape[0], 0.25, np.float32)
    O.predict_flat(bins, forest, 0.1, ref)
    assert np.array_equal(out.cpu().numpy(), ref)
    assert rng is not None


def test_root_histogram_full_width(cuda):
    """A C2-shaped root histogram (1M rows x 1000 features, B=32) against the
    oracle: exact integer sums, counts summing to the row count."""
    rng = np.random.default_rng(42)
    n, F, B = 1_000_000, 1000, 32
    bins = rng.integers(0, B, (n, F), dtype=np.int8)
    g = rng.standard_normal(n).astype(np.float32)
    samples = np.arange(n, dtype=np.int32)
    feats = np.arange(F, dtype=np.int32)
    era = np.zeros(n, np.int32)
    Gd = torch.zeros((1, F, B), device=cuda)
    Hd = torch.zeros((1, F, B), device=cuda)
    node_kernel.compute_histogram3(torch.from_numpy(bins).to(cuda), torch.from_numpy(g).to(cuda),
                                   torch.from_numpy(samples).to(cuda), torch.from_numpy(feats).to(cuda),
                                   torch.from_numpy(era).to(cuda), Gd, Hd, B)
    s = O.quant_shift(float(np.abs(g).max()))
    Gq, Cq = O.hist_q(bins, O.quantize(g, s), samples, feats, era, 1, B)
    Gf, Hf = O.dequant(Gq, Cq, s)
    assert np.array_equal(Hd.cpu().numpy(), Hf)
    assert np.array_equal(Gd.cpu().numpy(), Gf)
    assert (Hf.sum(axis=2) == n).all()


@pytest.mark.parametrize("nbytes", [1, 4097, (64 << 20) + 3, (200 << 20) + 12345])
def test_pipelined_h2d_copy_is_exact(cuda, nbytes):
    rng = np.random.default_rng(nbytes % 1000)
    src = rng.integers(0, 256, nbytes, dtype=np.uint8)
    dst = torch.empty(nbytes, dtype=torch.uint8, device=cuda)
    _lib.call("wgb_h2d", dst.data_ptr(), src.ctypes.data, nbytes, _st())
    assert np.array_equal(dst.cpu().numpy(), src)


def _quantile_cases(rng):
    n_list = [1, 2, 3, 7, 100, 4097, 300_000]
    for n in n_list:
        yield "normal", rng.standard_normal(n).astype(np.float32) * 3
    n = 50_000
    yield "ties", rng.integers(0, 5, n).astype(np.float32)
    yield "constant", np.full(n, -2.5, np.float32)
    yield "signed_zeros", np.where(rng.random(n) < 0.5, 0.0, -0.0).astype(np.float32)
    yield "inf", np.where(rng.random(n) < 0.05, np.inf, rng.standard_normal(n)).astype(np.float32)
    yield "neg_inf", np.where(rng.random(n) < 0.3, -np.inf, rng.standard_normal(n)).astype(np.float32)
    yield "nan", np.where(rng.random(n) < 0.001, np.nan, rng.standard_normal(n)).astype(np.float32)
    yield "tiny", (rng.standard_normal(n) * 1e-38).astype(np.float32)
    yield "heavy", rng.standard_cauchy(n).astype(np.float32)
    yield "clustered", (np.round(rng.standard_normal(n) * 4) / 4 + 1e6).astype(np.float32)


@pytest.mark.parametrize("B", [2, 5, 32, 127])
def test_quantile_edges_kernel_equals_torch_quantile(cuda, B):
    """wgb_quantile_edges (radix select) against torch.quantile on the B200,
    the op the reference calls (core.py:532), bit for bit."""
    from warpgbm_b200.core import _quantile_columns
    rng = np.random.default_rng(B)
    q = torch.linspace(0, 1, B + 1, device=cuda, dtype=torch.float32)[1:-1]
    for name, col in _quantile_cases(rng):
        x = torch.from_numpy(col).to(cuda)
        got = _quantile_columns(x[:, None], q)[0].cpu().numpy()
        ref = torch.quantile(x, q).cpu().numpy()
        assert np.array_equal(got, ref, equal_nan=True), (name, len(col), got, ref)
    # a multi-column matrix (transpose path, column chunking)
    X = rng.standard_normal((20_000, 37)).astype(np.float32)
    X[:, 5] = np.round(X[:, 5])
    Xd = torch.from_numpy(X).to(cuda)
    got = _quantile_columns(Xd, q, chunk_elems=20_000 * 8).cpu().numpy()
    ref = torch.quantile(Xd, q, dim=0).T.cpu().numpy()
    assert np.array_equal(got, ref, equal_nan=True)


@pytest.mark.parametrize("E,k,nb", [(3, 40, 4), (30, 40, 4), (60, 50, 4), (100, 300, 9), (600, 1188, 4),
                                    (600, 128, 4), (12, 30, 32), (200, 7, 3), (64, 2, 2), (40, 16, 4)])
def test_oracle_era_mean_order_equals_torch_cuda_mean(cuda, E, k, nb):
    """The oracle's restatement of the order in which torch's CUDA mean adds
    the eras (the reference's DES criterion, core.py:581-582) against torch
    on this GPU, bit for bit."""
    import torch
    g = torch.Generator(device=cuda)
    g.manual_seed(E * 1000 + k + nb)
    x = torch.randn((E, k, nb), generator=g, device=cuda) * 10.0
    want = x.mean(dim=0).cpu().numpy()
    got = O.cuda_era_mean(x.cpu().numpy())
    assert np.array_equal(got.view(np.int32), want.view(np.int32))


@pytest.mark.parametrize("F,D,objective", [(50, 4, "multiclass"), (7000, 3, "regression"),
                                           (300, 10, "regression"), (40, 13, "regression")])
def test_heap_and_packed_predictors_agree_with_oracle(cuda, F, D, objective):
    """wgb_predict_heap (complete-tree layout, depth <= 12) and
    wgb_predict_packed (pre-order, any depth), with rows staged in shared
    memory and -- for rows too wide to stage (7000 features) -- read from
    global memory, against the oracle's flattened-forest predict
    (predict.cu:17-44 semantics, tree order)."""
    from warpgbm_b200 import WarpGBM
    from warpgbm_b200.core import heap_forest
    rng = np.random.default_rng(F + D)
    n = 3000
    X = rng.standard_normal((n, F)).astype(np.float32)
    if objective == "multiclass":
        y = (X[:, 0] > 0).astype(int) + (X[:, F - 1] > 0.5).astype(int)
    else:
        y = (X[:, 0] - X[:, F - 1] + 0.1 * rng.standard_normal(n)).astype(np.float32)
    m = WarpGBM(objective=objective, n_estimators=6, max_depth=D, num_bins=16, min_child_weight=2).fit(X, y)
    bins = m.bin_inference_data(X)
    nodes, offs_d, offs, heap = m._ensure_packed()
    K = m.num_classes if objective == "multiclass" else 1
    T = len(offs) - 1
    st = torch.cuda.current_stream().cuda_stream
    out_p = torch.zeros((n, K), dtype=torch.float32, device=cuda)
    _lib.call("wgb_predict_packed", bins.data_ptr(), n, bins.shape[1], nodes.data_ptr(), offs_d.data_ptr(),
              T, K, float(np.float32(0.1)), out_p.data_ptr(), st)
    bins_h = bins[:, :F].cpu().numpy()
    parts = [nodes.cpu().numpy().reshape(-1, 2)[offs[t]:offs[t + 1]] for t in range(T)]
    flat = m._flat_trees()
    for c in range(K):
        want = np.zeros(n, np.float32)
        O.predict_flat(bins_h, np.stack([O.flatten_tree(t, 2 ** (D + 1)) for t in flat[c::K]]),
                       np.float32(0.1), want)
        assert np.array_equal(out_p[:, c].cpu().numpy(), want)
    if D <= 12:
        H = heap_forest(parts, D)
        Hd = torch.from_numpy(H.reshape(-1).view(np.int32)).to(cuda)
        out_h = torch.zeros((n, K), dtype=torch.float32, device=cuda)
        _lib.call("wgb_predict_heap", bins.data_ptr(), n, bins.shape[1], Hd.data_ptr(), T, K, D,
                  float(np.float32(0.1)), out_h.data_ptr(), st)
        assert torch.equal(out_h, out_p)
    else:
        assert heap is None
