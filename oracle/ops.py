"""numpy restatement of the operator library (test oracle; see oracle/__init__).

Every function takes and returns numpy arrays.  Arithmetic runs in float64
and the result is rounded to float32 once, so the oracle is at least as
accurate as any fp32 implementation; int64 results (argmax) are exact.
Each function names the reference kernel whose semantics it restates.
"""
from __future__ import annotations

import math

import numpy as np

try:
    from scipy.special import erf as _erf
except ImportError:  # pragma: no cover
    _erf = np.vectorize(math.erf)


def _f64(x):
    return np.asarray(x, dtype=np.float64)


def _out(v):
    return np.asarray(v, dtype=np.float32)


# -------------------------------------------------------------- elementwise
def gelu_tanh(x):
    """candidates/88_MinGPTNewGelu/v1.py:16-17: 0.5 x (1 + tanh(sqrt(2/pi)(x + 0.044715 x^3)))."""
    x = _f64(x)
    return _out(0.5 * x * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3))))


def gelu_erf(x):
    """candidates/26_GELU_/v1.py:14: 0.5 x (1 + erf(x / sqrt 2))."""
    x = _f64(x)
    return _out(0.5 * x * (1.0 + _erf(x / math.sqrt(2.0))))


def swish(x):
    """candidates/25_Swish/v1.py:14: x / (1 + exp(-x))."""
    x = _f64(x)
    with np.errstate(over="ignore"):
        return _out(x / (1.0 + np.exp(-x)))


def relu(x):
    """candidates/19_ReLU/v1.py:12, with torch.relu's NaN / -0.0 behaviour."""
    x = np.asarray(x, dtype=np.float32)
    return np.where(x < 0, np.float32(0), x).astype(np.float32)


# -------------------------------------------------------------- row ops
def layer_norm(x, weight=None, bias=None, eps=1e-5):
    """candidates/40_LayerNorm/v1.py:12-60 semantics (F.layer_norm over the last
    dim, biased variance, eps inside the sqrt), with optional affine."""
    x = _f64(x)
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    y = (x - mean) / np.sqrt(var + eps)
    if weight is not None:
        y = y * _f64(weight)
    if bias is not None:
        y = y + _f64(bias)
    return _out(y)


def rms_norm(x, weight=None, eps=1e-5, axis=-1):
    """candidates/36_RMSNorm_/v3.py:25-35: x / sqrt(mean(x^2) + eps) over `axis`."""
    x = _f64(x)
    ms = (x * x).mean(axis=axis, keepdims=True)
    y = x / np.sqrt(ms + eps)
    if weight is not None:
        shape = [1] * x.ndim
        shape[axis] = -1
        y = y * _f64(weight).reshape(shape)
    return _out(y)


def softmax(x):
    """candidates/23_Softmax/v1.py:12-45: exp(x - max) / sum(exp(x - max)), last dim."""
    x = _f64(x)
    m = x.max(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore"):
        e = np.exp(x - m)
        return _out(e / e.sum(axis=-1, keepdims=True))


def log_softmax(x):
    """candidates/24_LogSoftmax/v1.py:11-44: (x - max) - log(sum(exp(x - max)))."""
    x = _f64(x)
    m = x.max(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore", divide="ignore"):
        return _out((x - m) - np.log(np.exp(x - m).sum(axis=-1, keepdims=True)))


# -------------------------------------------------------------- dim reductions
def sum_dim(x, dim=1, keepdim=False):
    """candidates/47_Sum_reduction_over_a_dimension/v1.py:13-26."""
    return _out(_f64(x).sum(axis=dim, keepdims=keepdim))


def mean_dim(x, dim=1, keepdim=False):
    """candidates/48_Mean_reduction_over_a_dimension/v1.py:10-23."""
    x = _f64(x)
    with np.errstate(invalid="ignore", divide="ignore"):
        return _out(x.sum(axis=dim, keepdims=keepdim) / x.shape[dim])


def argmax_dim(x, dim=1, keepdim=False):
    """candidates/51_Argmax_over_a_dimension/v1.py:11-25: first index of the
    maximum (strict > while scanning upward); a NaN is the maximum and the
    first NaN wins, as torch.argmax."""
    x = np.asarray(x, dtype=np.float32)
    xm = np.moveaxis(x, dim, -1)
    nan = np.isnan(xm)
    idx = np.argmax(xm, axis=-1)  # numpy: first occurrence of the maximum
    has_nan = nan.any(axis=-1)
    first_nan = np.argmax(nan, axis=-1)
    idx = np.where(has_nan, first_nan, idx).astype(np.int64)
    if keepdim:
        idx = np.expand_dims(idx, dim)
    return idx


# -------------------------------------------------------------- global reductions
def mse_loss(a, b):
    """candidates/94_MSELoss/v1.py:13-45: mean((a - b)^2) -> 0-d."""
    d = _f64(a) - _f64(b)
    with np.errstate(invalid="ignore"):
        return _out(np.mean(d * d) if d.size else np.nan)


def frobenius_normalize(x):
    """candidates/37_FrobeniusNorm_/v1.py:12-46: x / ||x||_F."""
    x = _f64(x)
    return _out(x / np.sqrt((x * x).sum()))


# -------------------------------------------------------------- spatial
def max_pool2d(x, kernel_size, stride=None, padding=0, dilation=1):
    """torch.max_pool2d (floor mode) on NCHW; the reference kernel
    candidates/42_Max_Pooling_2D/v1.py:12-35 ignored stride and dilation.
    Padding is -inf; NaN in a window propagates."""
    x = np.asarray(x, dtype=np.float32)
    k, s = kernel_size, (stride or kernel_size)
    p, d = padding, dilation
    N, C, H, W = x.shape
    OH = (H + 2 * p - d * (k - 1) - 1) // s + 1
    OW = (W + 2 * p - d * (k - 1) - 1) // s + 1
    xp = np.full((N, C, H + 2 * p, W + 2 * p), -np.inf, dtype=np.float32)
    xp[:, :, p:p + H, p:p + W] = x
    out = np.full((N, C, OH, OW), -np.inf, dtype=np.float32)
    anynan = np.zeros((N, C, OH, OW), dtype=bool)
    for u in range(k):
        for v in range(k):
            win = xp[:, :, u * d: u * d + s * (OH - 1) + 1: s, v * d: v * d + s * (OW - 1) + 1: s]
            anynan |= np.isnan(win)
            out = np.fmax(out, win)
    out[anynan] = np.nan
    return out


def batch_norm_train(x, weight=None, bias=None, eps=1e-5):
    """candidates/33_BatchNorm/v1.py:18-51 semantics: training-mode BatchNorm
    with batch statistics over (N, H, W) per channel, biased variance."""
    x = _f64(x)
    axes = (0,) + tuple(range(2, x.ndim))
    mean = x.mean(axis=axes, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=axes, keepdims=True)
    y = (x - mean) / np.sqrt(var + eps)
    shape = [1, -1] + [1] * (x.ndim - 2)
    if weight is not None:
        y = y * _f64(weight).reshape(shape)
    if bias is not None:
        y = y + _f64(bias).reshape(shape)
    return _out(y)


def batch_norm_running_update(x, running_mean, running_var, momentum=0.1):
    """running statistics after one training-mode step (unbiased variance)."""
    x = _f64(x)
    axes = (0,) + tuple(range(2, x.ndim))
    n = x.size // x.shape[1]
    mean = x.mean(axis=axes)
    var_u = x.var(axis=axes) * n / max(n - 1, 1)
    rm = (1 - momentum) * _f64(running_mean) + momentum * mean
    rv = (1 - momentum) * _f64(running_var) + momentum * var_u
    return _out(rm), _out(rv)


# -------------------------------------------------------------- contractions
def matmul(a, b, trans_a=False):
    """candidates/1_Square_matrix_multiplication_/v1.py:19-80: op(A) @ B."""
    a = _f64(a)
    if trans_a:
        a = a.T
    return _out(a @ _f64(b))


def bmm(a, b):
    """candidates/3_Batched_matrix_multiplication/v1.py:19-80."""
    return _out(np.matmul(_f64(a), _f64(b)))


def matmul_splitk(a, b):
    """candidates/6_Matmul_with_large_K_dimension_/v1.py:17-65."""
    return _out(_f64(a) @ _f64(b))


def gemv(a, x):
    """candidates/4_Matrix_vector_multiplication_/v1.py:14-34."""
    return _out(_f64(a) @ _f64(x))


def diag_matmul(a, b):
    """candidates/12_Matmul_with_diagonal_matrices_/v1.py:10-17: diag(a) @ B
    evaluated as the row scale a[i] * b[i, j]."""
    return _out(_f64(a)[:, None] * _f64(b))


def matmul_transposed_a(a_t, b):
    """candidates/16_Matmul_with_transposed_A/v1.py (TRANS_A): A stored [K, M], C = A^T @ B."""
    return _out(_f64(a_t).T @ _f64(b))


# ------------------------------ problems the reference lists but never attempted
# (harness/problems.py:45-56; scripts/milestone_table.py:16-24): restated from
# the torch functions they name.
def avg_pool2d(x, kernel_size, stride=None, padding=0, count_include_pad=True, divisor_override=None):
    """torch.nn.functional.avg_pool2d (floor mode) on NCHW: window sum over
    the real input (padding counts as 0) divided by the window size clipped to
    the padded input (count_include_pad), to the real input (otherwise), or
    by divisor_override."""
    x = _f64(x)
    k, s, p = kernel_size, (stride or kernel_size), padding
    N, C, H, W = x.shape
    OH = (H + 2 * p - k) // s + 1
    OW = (W + 2 * p - k) // s + 1
    xp = np.zeros((N, C, H + 2 * p, W + 2 * p))
    xp[:, :, p:p + H, p:p + W] = x
    tot = np.zeros((N, C, OH, OW))
    for u in range(k):
        for v in range(k):
            tot += xp[:, :, u: u + s * (OH - 1) + 1: s, v: v + s * (OW - 1) + 1: s]
    hs = np.arange(OH) * s - p
    ws = np.arange(OW) * s - p
    he, we = np.minimum(hs + k, H + p), np.minimum(ws + k, W + p)
    if divisor_override:
        div = np.full((OH, OW), float(divisor_override))
    elif count_include_pad:
        div = np.outer(he - hs, we - ws).astype(np.float64)
    else:
        div = np.outer(np.minimum(he, H) - np.maximum(hs, 0), np.minimum(we, W) - np.maximum(ws, 0)).astype(np.float64)
    return _out(tot / div)


def cumsum(x, dim):
    """torch.cumsum(x, dim): inclusive prefix sum, float64 accumulation."""
    return _out(np.cumsum(_f64(x), axis=dim))


def cross_entropy(logits, targets, ignore_index=-100):
    """torch.nn.functional.cross_entropy(logits[N, C], targets[N]),
    reduction 'mean': mean over rows with target != ignore_index of
    logsumexp(logits[i]) - logits[i, t_i]; a target outside [0, C) gives NaN;
    no valid row gives NaN."""
    x = _f64(logits)
    t = np.asarray(targets, dtype=np.int64)
    m = x.max(axis=1, keepdims=True)
    lse = (m + np.log(np.exp(x - m).sum(axis=1, keepdims=True)))[:, 0]
    keep = t != ignore_index
    ok = keep & (t >= 0) & (t < x.shape[1])
    picked = np.where(ok, x[np.arange(x.shape[0]), np.clip(t, 0, x.shape[1] - 1)], np.nan)
    loss = lse - picked
    with np.errstate(invalid="ignore", divide="ignore"):
        return _out(loss[keep].sum() / keep.sum())
