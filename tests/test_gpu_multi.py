"""Row-sharded fit (WarpGBM(distributed=True)) against a single-process fit
on the same rows: identical trees, importance and predictions.

Two and three ranks always run on one GPU over a gloo group (host-staged
collectives), which exercises every exchange step of the sharded engine --
the feature-sliced one (each rank keeps and searches a slice of the
positions: reduce-scatter of the level histograms, all-gather of the best
split per node; three ranks give uneven slices) and the one that sums
every histogram on every rank; with two or more GPUs the sliced check also
runs over NCCL, one GPU per rank."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cases():
    rng = np.random.default_rng(5)
    n, F, E = 24_000, 40, 30
    Xp = rng.integers(0, 5, (n, F)).astype(np.int8)
    era = np.repeat(np.arange(E), n // E).astype(np.int32)
    yp = (Xp[:, 0] * 0.3 - Xp[:, 3] * np.where(era % 2, 1, -1) + rng.standard_normal(n)).astype(np.float32)
    Xf = rng.standard_normal((n, 33)).astype(np.float32)
    yf = (Xf[:, 0] - 2 * Xf[:, 1] * Xf[:, 2] + 0.3 * rng.standard_normal(n)).astype(np.float32)
    lab = (Xf[:, 0] + Xf[:, 4] > 0).astype(np.int64) + (Xf[:, 5] > 1).astype(np.int64)
    return [
        ("prebinned_eras_colsample", Xp, yp, era,
         dict(num_bins=5, max_depth=5, n_estimators=4, learning_rate=0.1, colsample_bytree=0.5,
              random_state=3, min_child_weight=5)),
        ("float_regression", Xf, yf, None,
         dict(num_bins=32, max_depth=4, n_estimators=4, learning_rate=0.2)),
        ("multiclass", Xf, lab, None,
         dict(objective="multiclass", num_bins=16, max_depth=3, n_estimators=3, learning_rate=0.3)),
    ]


def _fit_summary(m, X):
    from oracle import flatten_tree
    D = m.max_depth
    trees = [t for r in m.forest if r for t in (r if isinstance(r, list) else [r])]
    flat = np.stack([flatten_tree(t, 2 ** (D + 1)) for t in trees])
    pred = m.predict_proba(X) if m.objective != "regression" else m.predict(X)
    return {"flat": flat, "imp": m.per_era_feature_importance_, "pred": pred}


def _worker(rank, world, port, backend, outdir, slices):
    import contextlib
    import datetime
    import io
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    from warpgbm_b200 import WarpGBM
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = rank if backend == "nccl" else 0
    torch.cuda.set_device(dev)
    kw = {"device_id": torch.device("cuda", dev)} if backend == "nccl" else {}
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), **kw)
    out = {}
    for name, X, y, era, params in _cases():
        cut = np.linspace(0, len(y), world + 1).astype(int)
        sl = slice(cut[rank], cut[rank + 1])
        m = WarpGBM(distributed=True, **params)
        m._feature_slices = slices
        with contextlib.redirect_stdout(io.StringIO()):
            m.fit(X[sl], y[sl], era_id=None if era is None else era[sl])
            out[name] = _fit_summary(m, X)
    torch.save(out, os.path.join(outdir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _single():
    import contextlib
    import io
    from warpgbm_b200 import WarpGBM
    res = {}
    for name, X, y, era, params in _cases():
        with contextlib.redirect_stdout(io.StringIO()):
            m = WarpGBM(**params).fit(X, y, era_id=era)
            res[name] = _fit_summary(m, X)
    return res


def _check(backend, world, slices=True):
    single = _single()
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _port(), backend, d, slices), nprocs=world, join=True)
        outs = [torch.load(os.path.join(d, f"r{r}.pt"), weights_only=False) for r in range(world)]
    for name, ref in single.items():
        for r, o in enumerate(outs):
            got = o[name]
            # colsample subsets come from torch.randperm on cuda seeded by
            # random_state: the same draw in the single process and on rank 0
            assert np.array_equal(np.nan_to_num(got["flat"], nan=-7), np.nan_to_num(ref["flat"], nan=-7)), \
                (backend, name, r)
            assert np.array_equal(got["imp"], ref["imp"]), (backend, name, r)
            if name == "multiclass":
                assert np.abs(got["pred"] - ref["pred"]).max() < 1e-6
            else:
                assert np.array_equal(got["pred"], ref["pred"]), (backend, name, r)


@pytest.mark.parametrize("slices", [True, False])
def test_two_ranks_gloo_one_gpu_match_single_process(cuda, slices):
    _check("gloo", 2, slices)


def test_three_ranks_gloo_one_gpu_uneven_slices_match_single_process(cuda):
    _check("gloo", 3)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs for one NCCL rank per GPU")
def test_two_ranks_nccl_match_single_process(cuda):
    _check("nccl", 2)


def _edge_columns():
    rng = np.random.default_rng(9)
    n = 5000
    X = rng.standard_normal((n, 9)).astype(np.float32)
    X[:, 1] = np.round(X[:, 1] * 2) / 2                 # many ties
    X[::7, 2] = 0.0
    X[1::7, 2] = -0.0                                    # signed zeros
    X[5, 3] = np.nan                                     # one NaN: every edge NaN
    X[:, 4] = 3.0                                        # constant
    X[::11, 5] = np.inf
    X[3::11, 5] = -np.inf
    X[:, 6] = rng.exponential(1e-30, n).astype(np.float32)  # tiny magnitudes
    X[:, 7] = (rng.standard_normal(n) * 1e30).astype(np.float32)
    return X


def _edge_worker(rank, world, port, outdir, nq):
    import datetime
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    from warpgbm_b200.core import _Comm, sharded_quantile_edges
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    X = _edge_columns()
    cut = [0, 0, 1700, len(X)][: world + 1] if world == 3 else np.linspace(0, len(X), world + 1).astype(int)
    Xd = torch.from_numpy(X[cut[rank]:cut[rank + 1]]).cuda()
    q = torch.linspace(0, 1, nq + 2, device="cuda", dtype=torch.float32)[1:-1]
    e = sharded_quantile_edges(Xd, q, _Comm(True))
    torch.save(e.cpu(), os.path.join(outdir, f"e{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("nq", [31, 7, 63])
def test_sharded_quantile_edges_equal_torch_quantile(cuda, nq):
    """Quantile edges of row-sharded columns (3 gloo ranks on one GPU, one of
    them holding no rows): the digit histograms summed over the ranks (up to
    32 quantiles; more take the column exchange) select the same order
    statistics as the one-launch select over the concatenated column (bit
    for bit), and the edges equal torch.quantile's -- ties,
    signed zeros, infinities, a NaN column, a constant column, tiny and huge
    magnitudes.  (Against torch the comparison is by value, as for the
    one-launch select: a zero edge's sign bins nothing differently.)"""
    from warpgbm_b200.core import _quantile_columns
    X = _edge_columns()
    q = torch.linspace(0, 1, nq + 2, device="cuda", dtype=torch.float32)[1:-1]
    Xd = torch.from_numpy(X).cuda()
    want = torch.stack([torch.quantile(Xd[:, f], q) for f in range(X.shape[1])]).cpu().numpy()
    one = _quantile_columns(Xd, q).cpu().numpy()
    nan = np.isnan(want)
    assert nan[3].all() and np.array_equal(np.isnan(one), nan)
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_edge_worker, args=(3, _port(), d, nq), nprocs=3, join=True)
        for r in range(3):
            got = torch.load(os.path.join(d, f"e{r}.pt")).numpy()
            assert np.array_equal(np.isnan(got), nan), r
            assert np.array_equal(got[~nan].view(np.int32), one[~nan].view(np.int32)), \
                (r, np.argwhere((got.view(np.int32) != one.view(np.int32)) & ~nan)[:5])
            assert np.array_equal(got, want, equal_nan=True), (r, np.argwhere((got != want) & ~nan)[:5])
