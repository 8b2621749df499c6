"""Row-sharded host logic on world_size-2 gloo process groups (CPU only):
era union, base prediction, column exchange for the quantile edges, exact
histogram all-reduce, the feature-sliced exchange (reduce-scatter of a
level's slice-major staging buffer, all-gather of the per-node best-split
records; also with three ranks and uneven slices), and detection of a rank
that dies before a collective."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fn_name, outdir, timeout_s):
    import datetime
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    try:
        res = globals()[fn_name](rank, world)
        torch.save(res, os.path.join(outdir, f"r{rank}.pt"))
    except Exception as e:  # recorded for the parent
        torch.save({"error": f"{type(e).__name__}: {e}"}, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(fn_name, world=2, timeout_s=60):
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _free_port(), fn_name, d, timeout_s), nprocs=world, join=True)
        return [torch.load(os.path.join(d, f"r{r}.pt"), weights_only=False) for r in range(world)]


def _data():
    rng = np.random.default_rng(0)
    n, F = 3001, 7
    X = rng.standard_normal((n, F)).astype(np.float32)
    y = (rng.standard_normal(n) * 5 + 3).astype(np.float32)
    era = rng.integers(10, 20, n).astype(np.int32)
    cut = 1200
    return X, y, era, cut


def _shard(a, rank, cut):
    return a[:cut] if rank == 0 else a[cut:]


# ---- worker bodies ------------------------------------------------------
def w_eras_and_mean(rank, world):
    from warpgbm_b200.core import _Comm, exact_mean, global_unique_eras
    X, y, era, cut = _data()
    comm = _Comm(True)
    e = torch.from_numpy(_shard(era, rank, cut))
    if rank == 0:
        e = e[e < 18]                  # rank 0 lacks some eras
    uniq, inv = global_unique_eras(e, comm)
    m = exact_mean(torch.from_numpy(_shard(y, rank, cut)), comm)
    return {"uniq": uniq.numpy(), "inv": inv.numpy(), "e": e.numpy(), "mean": m}


def w_exchange(rank, world):
    from warpgbm_b200.core import _Comm, exchange_columns
    X, y, era, cut = _data()
    cols, per = exchange_columns(torch.from_numpy(_shard(X, rank, cut)), _Comm(True))
    return {"cols": cols.numpy(), "per": per}


def w_hist_allreduce(rank, world):
    import oracle as O
    X, y, era, cut = _data()
    B = 8
    bins = O.bin_matrix(X, np.tile(np.linspace(-1.5, 1.5, B - 1, dtype=np.float32), (X.shape[1], 1)))
    s = O.quant_shift(float(np.abs(y).max()))
    q = O.quantize(y, s)
    rows = np.arange(len(y), dtype=np.int32)
    mine = rows[:cut] if rank == 0 else rows[cut:]
    feats = np.arange(X.shape[1], dtype=np.int32)
    G, C = O.hist_q(bins, q, mine, feats, np.zeros(len(y), np.int32), 1, B)
    Gt, Ct = torch.from_numpy(G), torch.from_numpy(C)
    dist.all_reduce(Gt)
    dist.all_reduce(Ct)
    Gall, Call = O.hist_q(bins, q, rows, feats, np.zeros(len(y), np.int32), 1, B)
    return {"ok": bool(np.array_equal(Gt.numpy(), Gall) and np.array_equal(Ct.numpy(), Call))}


def w_slices(rank, world):
    """One level of a feature-sliced fit: each rank's local histograms of
    all 7 positions in the staging layout [slice][sums ks*(B+1)][counts
    ks*(B+1)][root sum, spare], reduce-scattered; then the ranks' node
    records all-gathered in place."""
    import oracle as O
    from warpgbm_b200.core import _Comm
    X, y, era, cut = _data()
    B, F = 8, X.shape[1]
    bins = O.bin_matrix(X, np.tile(np.linspace(-1.5, 1.5, B - 1, dtype=np.float32), (F, 1)))
    q = O.quantize(y, O.quant_shift(float(np.abs(y).max())))
    rows = np.arange(len(y), dtype=np.int32)
    cuts = np.linspace(0, len(y), world + 1).astype(int)
    mine = rows[cuts[rank]:cuts[rank + 1]]
    feats = np.arange(F, dtype=np.int32)
    G, C = O.hist_q(bins, q, mine, feats, np.zeros(len(y), np.int32), 1, B)
    ks = (F + world - 1) // world
    SE = 2 * ks * (B + 1) + 2
    stage = np.zeros((world, SE), np.int64)
    for r in range(world):
        js = feats[r * ks:(r + 1) * ks]
        stage[r, :len(js) * (B + 1)] = G[0, js].reshape(-1)
        stage[r, ks * (B + 1):ks * (B + 1) + len(js) * (B + 1)] = C[0, js].reshape(-1)
        stage[r, 2 * ks * (B + 1)] = int(q[mine].astype(np.int64).sum())
    comm = _Comm(True)
    out = torch.zeros(SE, dtype=torch.int64)
    comm.reduce_scatter_(out, torch.from_numpy(stage.reshape(-1)))
    cnt = 5
    win = torch.zeros(world * cnt, dtype=torch.int32)
    win[rank * cnt:(rank + 1) * cnt] = torch.arange(cnt, dtype=torch.int32) + 100 * rank
    comm.all_gather_inplace_(win, cnt)
    return {"out": out.numpy(), "win": win.numpy(), "ks": ks}


def w_dead_rank(rank, world):
    if rank == 1:
        raise RuntimeError("rank 1 failed before the collective")
    t = torch.ones(4)
    dist.all_reduce(t)                 # peer never joins: must end with an error
    return {"reduced": t.numpy()}


# ---- tests ---------------------------------------------------------------
def test_global_eras_and_exact_mean_are_shard_invariant():
    import oracle as O
    X, y, era, cut = _data()
    res = _run("w_eras_and_mean")
    allera = np.concatenate([res[0]["e"], res[1]["e"]])
    uniq = np.unique(allera)
    for r in res:
        assert np.array_equal(r["uniq"], uniq)
        assert np.array_equal(uniq[r["inv"]], r["e"])
        assert np.float32(r["mean"]) == O.canonical_mean(y)


def test_column_exchange_gives_full_columns():
    X, y, era, cut = _data()
    res = _run("w_exchange")
    per = res[0]["per"]
    for r, out in enumerate(res):
        want = np.zeros((X.shape[0], per), np.float32)
        cols = X[:, r * per:(r + 1) * per]
        want[:, :cols.shape[1]] = cols
        assert np.array_equal(out["cols"], want)


def test_histogram_allreduce_is_exact():
    res = _run("w_hist_allreduce")
    assert all(r["ok"] for r in res)


@pytest.mark.parametrize("world", [2, 3])
def test_feature_sliced_exchange_is_exact(world):
    import oracle as O
    X, y, era, cut = _data()
    B, F = 8, X.shape[1]
    bins = O.bin_matrix(X, np.tile(np.linspace(-1.5, 1.5, B - 1, dtype=np.float32), (F, 1)))
    q = O.quantize(y, O.quant_shift(float(np.abs(y).max())))
    G, C = O.hist_q(bins, q, np.arange(len(y), dtype=np.int32), np.arange(F, dtype=np.int32),
                    np.zeros(len(y), np.int32), 1, B)
    res = _run("w_slices", world=world)
    for r, got in enumerate(res):
        assert "error" not in got, got
        ks = got["ks"]
        js = np.arange(F)[r * ks:(r + 1) * ks]
        out = got["out"]
        assert np.array_equal(out[:len(js) * (B + 1)], G[0, js].reshape(-1))
        assert np.array_equal(out[ks * (B + 1):ks * (B + 1) + len(js) * (B + 1)], C[0, js].reshape(-1))
        assert not out[len(js) * (B + 1):ks * (B + 1)].any()          # an uneven slice's padding
        assert out[2 * ks * (B + 1)] == int(q.astype(np.int64).sum())  # the root sum
        want = np.concatenate([np.arange(5) + 100 * w for w in range(world)])
        assert np.array_equal(got["win"], want)


def test_dead_rank_is_detected_by_peer():
    res = _run("w_dead_rank", timeout_s=5)
    assert "error" in res[1]
    assert "error" in res[0], "the surviving rank must not hang or succeed"
