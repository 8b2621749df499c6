import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")
GOLDEN_CASES = ["c1_regression", "era_des", "prebinned_colsample", "multiclass", "binary",
                "binning_edges", "eval_corr"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libwgb_b200.so")


def load_golden(name):
    import numpy as np
    d = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    params = eval(str(d["params"]))  # repr of a plain dict written by make_golden.py
    return d, params


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)
