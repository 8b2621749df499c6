"""Argument validation of the estimator (no GPU): the same exceptions and
messages as the reference's constructor and fit checks
(warpgbm/core.py:83-143 and 216-291), raised before any device work."""
import re

import numpy as np
import pytest

from warpgbm_b200 import WarpGBM


@pytest.mark.parametrize("kw,exc,msg", [
    (dict(objective="ranking"), ValueError,
     "objective must be 'regression', 'binary', or 'multiclass', got ranking."),
    (dict(num_bins=32.0), TypeError, "num_bins must be an integer, got <class 'float'>."),
    (dict(max_depth="3"), TypeError, "max_depth must be an integer, got <class 'str'>."),
    (dict(learning_rate="0.1"), TypeError, "learning_rate must be a float, got <class 'str'>."),
    (dict(num_bins=1), ValueError, "num_bins must be between 2 and 127 inclusive."),
    (dict(num_bins=128), ValueError, "num_bins must be between 2 and 127 inclusive."),
    (dict(max_depth=0), ValueError, "max_depth must be at least 1."),
    (dict(learning_rate=0.0), ValueError, "learning_rate must be in (0.0, 1.0]."),
    (dict(learning_rate=1.5), ValueError, "learning_rate must be in (0.0, 1.0]."),
    (dict(n_estimators=0), ValueError, "n_estimators must be positive."),
    (dict(min_child_weight=0), ValueError, "min_child_weight must be a positive integer."),
    (dict(min_split_gain=-1.0), ValueError, "min_split_gain must be non-negative."),
    (dict(threads_per_block=48), ValueError,
     "threads_per_block should be a positive multiple of 32 (warp size)."),
    (dict(rows_per_thread=17), ValueError, "rows_per_thread must be positive between 1 and 16 inclusive."),
    (dict(L2_reg=-1e-3), ValueError, "L2_reg must be non-negative."),
    (dict(colsample_bytree=0.0), ValueError,
     "Invalid colsample_bytree: 0.0. Must be a float value > 0 and <= 1."),
    (dict(colsample_bytree=1.5), ValueError,
     "Invalid colsample_bytree: 1.5. Must be a float value > 0 and <= 1."),
])
def test_constructor_rejects(kw, exc, msg):
    with pytest.raises(exc, match="^" + re.escape(msg) + "$"):
        WarpGBM(**kw)


def test_constructor_accepts_int_for_float_parameters():
    m = WarpGBM(learning_rate=1, L2_reg=0, min_split_gain=0, colsample_bytree=1)
    assert m.learning_rate == 1


X, y = np.zeros((6, 3), np.float32), np.zeros(6, np.float32)
Xe, ye = np.zeros((4, 3), np.float32), np.zeros(4, np.float32)


@pytest.mark.parametrize("args,exc,msg", [
    ((X.tolist(), y, None, None, None, None, None, "mse"), TypeError, "X and y must be numpy arrays."),
    ((X[0], y, None, None, None, None, None, "mse"), ValueError, "X must be 2-dimensional, got shape (3,)"),
    ((X, X, None, None, None, None, None, "mse"), ValueError, "y must be 1-dimensional, got shape (6, 3)"),
    ((X, y[:5], None, None, None, None, None, "mse"), ValueError,
     "X and y must have the same number of rows. Got 6 and 5."),
    ((X, y, [0] * 6, None, None, None, None, "mse"), TypeError, "era_id must be a numpy array."),
    ((X, y, np.zeros((6, 1)), None, None, None, None, "mse"), ValueError,
     "era_id must be 1-dimensional, got shape (6, 1)"),
    ((X, y, np.zeros(5), None, None, None, None, "mse"), ValueError,
     "era_id must have same length as y. Got 5 and 6."),
    ((X, y, None, Xe, None, None, None, "mse"), ValueError,
     "If using eval set, X_eval, y_eval, and eval_every_n_trees must all be defined."),
    ((X, y, None, Xe.tolist(), ye, 2, None, "mse"), TypeError, "X_eval and y_eval must be numpy arrays."),
    ((X, y, None, Xe[0], ye, 2, None, "mse"), ValueError, "X_eval must be 2-dimensional, got shape (3,)"),
    ((X, y, None, Xe, Xe, 2, None, "mse"), ValueError, "y_eval must be 1-dimensional, got shape (4, 3)"),
    ((X, y, None, Xe, ye[:3], 2, None, "mse"), ValueError,
     "X_eval and y_eval must have same number of rows. Got 4 and 3."),
    ((X, y, None, Xe, ye, 0, None, "mse"), ValueError, "eval_every_n_trees must be a positive integer, got 0."),
    ((X, y, None, Xe, ye, 2, 0, "mse"), ValueError, "early_stopping_rounds must be a positive integer, got 0."),
    ((X, y, None, Xe, ye, 2, None, "auc"), ValueError,
     "Invalid eval_metric: auc. Choose from ['mse', 'corr', 'rmsle', 'logloss', 'accuracy']."),
])
def test_fit_params_rejected(args, exc, msg):
    with pytest.raises(exc, match="^" + re.escape(msg) + "$"):
        WarpGBM(n_estimators=5).validate_fit_params(*args)


def test_fit_params_early_stopping_default():
    m = WarpGBM(n_estimators=5)
    # with an eval set and no early stopping, "never stop" is n_estimators + 1
    assert m.validate_fit_params(X, y, None, Xe, ye, 2, None, "mse") == 6
    assert m.validate_fit_params(X, y, None, Xe, ye, 2, 3, "corr") == 3
    # without an eval set the value passes through
    assert m.validate_fit_params(X, y, None, None, None, None, None, "mse") is None


def test_fit_rejects_before_device_work():
    with pytest.raises(ValueError, match="X and y must have the same number of rows"):
        WarpGBM(n_estimators=2).fit(X, y[:4])
