"""Per-problem test table: oracle function, CUDA op, tolerance.

Tolerances are the ones the operator library promises against the
torch-eager fp32 reference: atol = rtol = 1e-5 for elementwise and
normalisation outputs, 1e-3 for reductions and contractions, bit-exact for
argmax indices and max-pooling (whose outputs are input values).  Of the
problems the reference never attempted, average pooling and cross-entropy
hold 1e-5 and cumsum 1e-4 (a prefix of 32768 N(0,1) terms reaches |y| ~ 500,
where one fp32 ulp is 3e-5).
"""
from __future__ import annotations

import numpy as np

from oracle import ops as O

EXACT = "exact"

# name -> (oracle(*numpy inputs) -> numpy, tolerance)
ORACLE = {
    "88_MinGPTNewGelu": (lambda x: O.gelu_tanh(x), 1e-5),
    "26_GELU_": (lambda x: O.gelu_erf(x), 1e-5),
    "25_Swish": (lambda x: O.swish(x), 1e-5),
    "19_ReLU": (lambda x: O.relu(x), EXACT),
    "40_LayerNorm": (lambda x, w, b: O.layer_norm(x, w, b, 1e-5), 1e-5),
    "36_RMSNorm_": (lambda x, w: O.rms_norm(x, w, 1e-5), 1e-5),
    "23_Softmax": (lambda x: O.softmax(x), 1e-5),
    "24_LogSoftmax": (lambda x: O.log_softmax(x), 1e-5),
    "47_Sum_reduction_over_a_dimension": (lambda x: O.sum_dim(x, 1, keepdim=True), 1e-3),
    "48_Mean_reduction_over_a_dimension": (lambda x: O.mean_dim(x, 1), 1e-3),
    "51_Argmax_over_a_dimension": (lambda x: O.argmax_dim(x, 1), EXACT),
    "94_MSELoss": (lambda a, b: O.mse_loss(a, b), 1e-3),
    "37_FrobeniusNorm_": (lambda x: O.frobenius_normalize(x), 1e-5),
    "42_Max_Pooling_2D": (lambda x: O.max_pool2d(x, 3, 2, 1, 1), EXACT),
    "33_BatchNorm": (lambda x, w, b: O.batch_norm_train(x, w, b, 1e-5), 1e-5),
    "1_Square_matrix_multiplication_": (lambda a, b: O.matmul(a, b), 1e-3),
    "3_Batched_matrix_multiplication": (lambda a, b: O.bmm(a, b), 1e-3),
    "6_Matmul_with_large_K_dimension_": (lambda a, b: O.matmul_splitk(a, b), 1e-3),
    "4_Matrix_vector_multiplication_": (lambda a, x: O.gemv(a, x), 1e-3),
    "16_Matmul_with_transposed_A": (lambda a, b: O.matmul_transposed_a(a, b), 1e-3),
    "13_Matmul_for_symmetric_matrices": (lambda a, b: O.matmul(a, b), 1e-3),
    "12_Matmul_with_diagonal_matrices_": (lambda a, b: O.diag_matmul(a, b), 1e-5),
    "7_Matmul_with_small_K_dimension_": (lambda a, b: O.matmul(a, b), 1e-3),
    "45_Average_Pooling_2D": (lambda x: O.avg_pool2d(x, 3, 2, 1), 1e-5),
    "89_cumsum": (lambda x: O.cumsum(x, 1), 1e-4),
    "95_CrossEntropyLoss": (lambda p, t: O.cross_entropy(p, t), 1e-5),
}


def gpu_call(name: str):
    """The tensor-level CUDA op for problem `name` (imports kbb200 lazily)."""
    from kbb200 import ops as K

    table = {
        "88_MinGPTNewGelu": lambda x: K.gelu_tanh(x),
        "26_GELU_": lambda x: K.gelu_erf(x),
        "25_Swish": lambda x: K.swish(x),
        "19_ReLU": lambda x: K.relu(x),
        "40_LayerNorm": lambda x, w, b: K.layer_norm(x, w, b, 1e-5),
        "36_RMSNorm_": lambda x, w: K.rms_norm(x, w, 1e-5),
        "23_Softmax": lambda x: K.softmax(x),
        "24_LogSoftmax": lambda x: K.log_softmax(x),
        "47_Sum_reduction_over_a_dimension": lambda x: K.sum_dim(x, 1, keepdim=True),
        "48_Mean_reduction_over_a_dimension": lambda x: K.mean_dim(x, 1),
        "51_Argmax_over_a_dimension": lambda x: K.argmax_dim(x, 1),
        "94_MSELoss": lambda a, b: K.mse_loss(a, b),
        "37_FrobeniusNorm_": lambda x: K.frobenius_normalize(x),
        "42_Max_Pooling_2D": lambda x: K.max_pool2d(x, 3, 2, 1, 1),
        "33_BatchNorm": lambda x, w, b: K.batch_norm_train(x, w, b, 1e-5),
        "1_Square_matrix_multiplication_": lambda a, b: K.matmul(a, b),
        "3_Batched_matrix_multiplication": lambda a, b: K.bmm(a, b),
        "6_Matmul_with_large_K_dimension_": lambda a, b: K.matmul_splitk(a, b),
        "4_Matrix_vector_multiplication_": lambda a, x: K.gemv(a, x),
        "16_Matmul_with_transposed_A": lambda a, b: K.matmul(a, b, trans_a=True),
        "13_Matmul_for_symmetric_matrices": lambda a, b: K.matmul(a, b),
        "12_Matmul_with_diagonal_matrices_": lambda a, b: K.diag_matmul(a, b),
        "7_Matmul_with_small_K_dimension_": lambda a, b: K.matmul(a, b),
        "45_Average_Pooling_2D": lambda x: K.avg_pool2d(x, 3, 2, 1),
        "89_cumsum": lambda x: K.cumsum(x, 1),
        "95_CrossEntropyLoss": lambda p, t: K.cross_entropy(p, t),
    }
    return table[name]


def assert_close(got, want, tol, what: str = "") -> None:
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    if tol == EXACT:
        ok = np.array_equal(got, want, equal_nan=True)
        if not ok:
            bad = np.argwhere(~((got == want) | (np.isnan(got) & np.isnan(want))))
            raise AssertionError(f"{what}: {len(bad)} mismatches, first at {bad[:3].tolist()}")
        return
    g = got.astype(np.float64)
    w = want.astype(np.float64)
    nan_ok = np.isnan(g) == np.isnan(w)
    assert nan_ok.all(), f"{what}: NaN pattern differs"
    m = ~np.isnan(w) & ~(np.isinf(w) & (g == w))   # equal infinities match
    err = np.abs(g[m] - w[m])
    lim = tol + tol * np.abs(w[m])
    if not (err <= lim).all():
        i = int(np.argmax(err - lim))
        raise AssertionError(
            f"{what}: max |diff| {err.max():.3e} exceeds atol=rtol={tol} "
            f"(worst: got {g[m][i]!r} want {w[m][i]!r})")


def load_golden(name: str):
    from pathlib import Path

    p = Path(__file__).resolve().parent / "golden" / f"{name}.npz"
    z = np.load(p)
    ins = [z[f"in{i}"] for i in range(len([k for k in z.files if k.startswith("in")]))]
    return ins, z["out"], z
