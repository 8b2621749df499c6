"""The era criterion plan of the C ABI (wgb_era_mean_plan) against the
oracle's restatement of torch's CUDA mean order, on the CPU: the plan is run
by a small numpy interpreter here and must give the same fp32 bits as
oracle.cuda_era_mean, whose order is pinned against torch on the B200
(tests/test_gpu_ops.py)."""
import numpy as np
import pytest

import oracle as O
from warpgbm_b200 import _lib

B200 = dict(num_sms=148, max_threads_per_sm=2048)


def run_plan(x, sched, ops):
    """Interpret the plan: 0 push (restart at 0), 1 add popped, 2 add next era."""
    E = x.shape[0]
    flat = x.reshape(E, -1)
    acc = np.zeros(flat.shape[1], np.float32)
    stack = []
    nxt = 0
    for op in ops.tolist():
        if op == 0:
            stack.append(acc)
            acc = np.zeros_like(acc)
        elif op == 1:
            acc = stack.pop() + acc
        else:
            acc = acc + flat[sched[nxt]]
            nxt += 1
    assert nxt == E
    return acc


SHAPES = [(2, 10, 4), (3, 40, 4), (30, 40, 4), (60, 50, 4), (100, 300, 9), (600, 1188, 4),
          (600, 128, 4), (12, 30, 32), (200, 7, 3), (64, 2, 2), (40, 16, 4), (257, 33, 31),
          (300, 5, 4), (999, 1, 2),
          # eras split over several blocks (global reduction)
          (1100, 64, 4), (2000, 1188, 4), (5000, 10, 4), (1024, 300, 31), (4096, 3, 1), (3000, 1, 126)]


@pytest.mark.parametrize("E,k,nb", SHAPES)
def test_plan_reproduces_oracle_order(E, k, nb):
    M = k * nb
    sched, ops, depth = _lib.era_mean_plan(E, M, **B200)
    assert sorted(sched.tolist()) == list(range(E))
    assert depth >= 1
    rng = np.random.default_rng(E * 7 + k)
    x = (rng.standard_normal((E, k, nb)) * 10).astype(np.float32)
    got = run_plan(x, sched, ops) * O.cuda_mean_factor(E, k, nb)
    want = O.cuda_era_mean(x, **B200).reshape(-1)
    assert np.array_equal(got.astype(np.float32).view(np.int32), want.view(np.int32))


def test_plan_orders_differ_from_sequential():
    """From tens of eras the order is not a sequential sum (else this
    machinery would be pointless): the sums differ in the last bits."""
    E, k, nb = 600, 1188, 4
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((E, k, nb)) * 10).astype(np.float32)
    seq = np.zeros(k * nb, np.float32)
    for e in range(E):
        seq = seq + x[e].reshape(-1)
    sched, ops, _ = _lib.era_mean_plan(E, k * nb, **B200)
    assert (run_plan(x, sched, ops) != seq).sum() > 1000


def test_single_output_is_sequential():
    sched, ops, depth = _lib.era_mean_plan(7, 1, **B200)
    assert sched.tolist() == list(range(7)) and ops.tolist() == [0] + [2] * 7 and depth == 1


def test_plan_rejects_bad_sizes():
    with pytest.raises(_lib.WgbError):
        _lib.era_mean_plan(0, 10, **B200)
