"""CPU: pin the oracle.

1. oracle.ops against the golden fixtures (the reference arm's recorded
   torch-eager CPU outputs) for every problem;
2. oracle.ops against the torch-eager problem models on fresh seeded inputs;
3. known answers the reference's kernels imply (argmax tie rule, NaN,
   max-pool windows with stride, biased BN variance, empty reductions).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import ops as O
from oracle import problems
from tests.opmap import EXACT, ORACLE, assert_close, load_golden

NAMES = problems.SUBSET


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_golden(name):
    ins, out, _ = load_golden(name)
    fn, tol = ORACLE[name]
    assert_close(fn(*ins), out, tol, name)


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("seed", [1, 2])
def test_oracle_matches_problem_model(name, seed):
    Model, get_inputs, get_init_inputs, _ = problems.load_problem(name, "small")
    torch.manual_seed(seed)
    inputs = get_inputs()
    with torch.no_grad():
        ref = Model(*get_init_inputs())(*inputs).numpy()
    fn, tol = ORACLE[name]
    assert_close(fn(*[t.numpy() for t in inputs]), ref, tol, name)


def test_golden_fixtures_cover_every_problem():
    from tests.golden.make_golden import GOLDEN_SHAPES

    assert set(GOLDEN_SHAPES) == set(problems.SUBSET)


# ---------------------------------------------------------------- known answers
def test_argmax_ties_pick_lowest_index():
    x = np.zeros((1, 5, 3), dtype=np.float32)
    x[0, 1, 0] = x[0, 3, 0] = 2.0          # tie between rows 1 and 3
    x[0, :, 1] = 7.0                        # all equal -> 0
    x[0, 4, 2] = np.nan
    x[0, 2, 2] = np.nan                     # first NaN wins
    np.testing.assert_array_equal(O.argmax_dim(x, 1), [[1, 0, 2]])
    t = torch.from_numpy(x)
    np.testing.assert_array_equal(torch.argmax(t, 1).numpy(), [[1, 0, 2]])


def test_argmax_all_neg_inf():
    x = np.full((1, 4, 2), -np.inf, dtype=np.float32)
    np.testing.assert_array_equal(O.argmax_dim(x, 1), [[0, 0]])


def test_relu_nan_and_signed_zero():
    x = np.array([-0.0, 0.0, np.nan, -1.0, 3.0], dtype=np.float32)
    y = O.relu(x)
    ref = torch.relu(torch.from_numpy(x)).numpy()
    assert np.array_equal(np.signbit(y), np.signbit(ref))
    assert_close(y, ref, EXACT)


def test_maxpool_stride_and_padding_window():
    x = np.arange(36, dtype=np.float32).reshape(1, 1, 6, 6)
    y = O.max_pool2d(x, 3, 2, 1, 1)
    # output (3, 3): window rows {2oh-1..2oh+1}, cols likewise, clipped
    want = np.array([[7, 9, 11], [19, 21, 23], [31, 33, 35]], dtype=np.float32)
    np.testing.assert_array_equal(y[0, 0], want)
    ref = torch.nn.functional.max_pool2d(torch.from_numpy(x), 3, 2, 1).numpy()
    np.testing.assert_array_equal(y, ref)


def test_maxpool_nan_propagates():
    x = np.zeros((1, 1, 4, 4), dtype=np.float32)
    x[0, 0, 1, 1] = np.nan
    y = O.max_pool2d(x, 2, 2, 0, 1)
    ref = torch.nn.functional.max_pool2d(torch.from_numpy(x), 2, 2).numpy()
    assert_close(y, ref, EXACT)
    assert np.isnan(y[0, 0, 0, 0]) and not np.isnan(y[0, 0, 1, 1])


def test_maxpool_dilation_matches_torch():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 3, 17, 19)).astype(np.float32)
    for k, s, p, d in [(3, 2, 1, 2), (2, 1, 0, 3), (4, 3, 2, 1), (5, 1, 2, 1)]:
        ref = torch.nn.functional.max_pool2d(torch.from_numpy(x), k, s, p, d).numpy()
        assert_close(O.max_pool2d(x, k, s, p, d), ref, EXACT, f"k{k}s{s}p{p}d{d}")


def test_batchnorm_uses_biased_variance_and_updates_running_stats():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((4, 3, 5, 5)).astype(np.float32) * 3 + 1
    y = O.batch_norm_train(x)
    per_c = y.transpose(1, 0, 2, 3).reshape(3, -1)
    np.testing.assert_allclose(per_c.mean(1), 0, atol=1e-5)
    np.testing.assert_allclose(per_c.var(1), 1, atol=1e-3)   # biased: exactly 1 - eps effect
    rm, rv = O.batch_norm_running_update(x, np.zeros(3), np.ones(3))
    bn = torch.nn.BatchNorm2d(3)
    bn.train()
    with torch.no_grad():
        bn(torch.from_numpy(x))
    np.testing.assert_allclose(rm, bn.running_mean.numpy(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(rv, bn.running_var.numpy(), rtol=1e-5, atol=1e-6)


def test_empty_reductions():
    assert math.isnan(float(O.mse_loss(np.zeros(0, np.float32), np.zeros(0, np.float32))))
    assert math.isnan(float(torch.mean((torch.zeros(0) - torch.zeros(0)) ** 2)))
    x = np.zeros((2, 0, 3), dtype=np.float32)
    np.testing.assert_array_equal(O.sum_dim(x, 1), np.zeros((2, 3), np.float32))


def test_softmax_rows_sum_to_one_and_logsoftmax_consistent():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((3, 777)) * 2).astype(np.float32)
    s = O.softmax(x)
    np.testing.assert_allclose(s.sum(-1), 1.0, rtol=1e-6)
    np.testing.assert_allclose(np.exp(O.log_softmax(x).astype(np.float64)), s, rtol=1e-5, atol=1e-9)


def test_gelu_tanh_formula_points():
    x = np.array([0.0, 1.0, -1.0, 3.0], dtype=np.float32)
    c = math.sqrt(2 / math.pi)
    want = [0.5 * v * (1 + math.tanh(c * (v + 0.044715 * v ** 3))) for v in x.astype(float)]
    np.testing.assert_allclose(O.gelu_tanh(x), want, rtol=1e-7)


def test_matmul_oracle_is_fp64_accurate():
    rng = np.random.default_rng(2)
    a = rng.standard_normal((17, 300)).astype(np.float32)
    b = rng.standard_normal((300, 9)).astype(np.float32)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    np.testing.assert_allclose(O.matmul(a, b), exact, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(O.matmul(a.T.copy(), b, trans_a=True), exact, rtol=1e-6, atol=1e-6)
