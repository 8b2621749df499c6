"""The no-allocation histogram entry point against the regular one and
against the oracle (canonical exact sums on the grid of max |g|).

wgb_compute_histogram3_noalloc is for hosts that may not allocate device
memory while building a histogram (a fixed memory budget handed to the
library, or code where an allocator call must not happen).  It uses a fixed
64 MiB block inside the library instead of the stream-ordered pool.  This
file is collected last so that a run stopping at the first failure has run
every other test; it also passes alone in a fresh process, where its first
call is the one that looks up the block's device address."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from warpgbm_b200 import _lib

pytestmark = pytest.mark.gpu


def _hist(fn, bins, g, samples, feats, era, E, B, dev):
    k = feats.size
    G = torch.zeros((E, k, B), device=dev)
    H = torch.zeros((E, k, B), device=dev)
    d = {n: torch.from_numpy(a).to(dev) for n, a in
         (("bins", bins), ("g", g), ("s", samples), ("f", feats), ("e", era))}
    rc = getattr(_lib.lib(), fn)(
        d["bins"].data_ptr(), bins.shape[0], bins.shape[1], d["g"].data_ptr(), d["s"].data_ptr(),
        samples.size, d["f"].data_ptr(), k, d["e"].data_ptr(), G.data_ptr(), H.data_ptr(), E, B,
        64, 4, torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, fn)
    return G.cpu().numpy(), H.cpu().numpy()


@pytest.mark.parametrize("n,F,k,E,B", [(200_000, 500, 500, 1, 32), (30_000, 61, 40, 7, 10),
                                       (5_000, 8, 8, 1, 2)])
def test_noalloc_matches_regular_entry_point_twice(n, F, k, E, B):
    assert torch.cuda.is_available()
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(n + F)
    bins = rng.integers(-1, B + 1, (n + 3, F)).astype(np.int8)
    g = (rng.standard_normal(n + 3) * 2).astype(np.float32)
    era = rng.integers(0, E, n + 3).astype(np.int32)
    samples = rng.permutation(n + 3)[:n].astype(np.int32)
    feats = rng.permutation(F)[:k].astype(np.int32)
    want = _hist("wgb_compute_histogram3", bins, g, samples, feats, era, E, B, dev)
    s = O.quant_shift(float(np.abs(g[samples]).max()))
    Gq, Cq = O.hist_q(bins, O.quantize(g, s), samples, feats, era, E, B)
    Gf, Hf = O.dequant(Gq, Cq, s)
    for _ in range(2):  # the block keeps the last call's contents: both calls must agree
        got = _hist("wgb_compute_histogram3_noalloc", bins, g, samples, feats, era, E, B, dev)
        assert np.array_equal(got[0], want[0])   # exact: same integer sums
        assert np.array_equal(got[1], want[1])
        assert np.array_equal(got[0], Gf)        # and the oracle's, on their own
        assert np.array_equal(got[1], Hf)


def test_noalloc_rejects_work_beyond_its_block():
    L = _lib.lib()
    # 600 eras x 2000 features x 33 bins x 16 B = 634 MB of cells > 64 MiB;
    # rejected before any pointer is touched
    rc = L.wgb_compute_histogram3_noalloc(None, 1, 2000, None, None, 10, None, 2000, None, None,
                                          None, 600, 32, 64, 4, None)
    assert rc == 1
    assert b"fixed block" in L.wgb_last_error()
