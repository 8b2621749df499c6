"""The reference's own CUDA kernels (compiled from its sources into
oracle/_ref/) under the restated fit loop of oracle/ref_cuda.py reproduce the
golden fixture of config 1, which the reference's core.py produced with a
CPU restatement of the same kernels.  This pins the baseline that bench.py
--impl reference-cuda times."""
import numpy as np
import pytest

import oracle as O
from conftest import load_golden

pytestmark = pytest.mark.gpu


def _ops():
    from oracle.build_ref import built_path, load
    if built_path() is None:
        pytest.skip("reference CUDA extension not built")
    return load()


def _plain(t):
    if "leaf_value" in t:
        return t
    return {"feature": int(t["feature"]), "bin": int(t["bin"]),
            "left": _plain(t["left"]), "right": _plain(t["right"])}


def test_reference_kernels_reproduce_config1_golden(cuda):
    from oracle.ref_cuda import RefCudaFit
    g, params = load_golden("c1_regression")
    m = RefCudaFit(_ops(), num_bins=params["num_bins"], max_depth=params["max_depth"],
                   learning_rate=params["learning_rate"], n_estimators=params["n_estimators"],
                   random_state=params["random_state"]).fit(g["X"], g["y"])
    assert np.array_equal(m.bins.cpu().numpy(), g["bins"])
    D = params["max_depth"]
    flat = np.stack([O.flatten_tree(_plain(t), 2 ** (D + 1)) for t in m.forest])
    ref = g["forest"]
    same = np.isnan(flat) == np.isnan(ref)
    assert same.all()
    structure = ~np.isnan(ref)
    structure[:, :, 5] = False               # leaf values compared with a tolerance
    assert np.array_equal(flat[structure], ref[structure])
    lv = ~np.isnan(ref[:, :, 5])
    assert np.allclose(flat[:, :, 5][lv], ref[:, :, 5][lv], rtol=1e-5, atol=1e-6)
