"""Tensor-level host API over the C ABI (include/kbb200.h).

Every function validates its tensors (CUDA, fp32, contiguous, matching
shapes), allocates outputs and scratch through torch's caching allocator,
and launches the CUDA kernel through the C ABI on torch's current stream of
the tensor's device.  Launches are asynchronous, like the reference's
candidate entries (e.g. candidates/26_GELU_/v1.py:18-23).  A C-ABI error
raises KbError; nothing falls back to another implementation.
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from ._lib import LIB, check

__all__ = [
    "gelu_tanh", "gelu_erf", "swish", "relu", "layer_norm", "rms_norm", "softmax",
    "log_softmax", "sum_dim", "mean_dim", "argmax_dim", "mse_loss", "frobenius_normalize",
    "max_pool2d", "batch_norm_train", "matmul", "bmm", "matmul_splitk", "gemv", "diag_matmul",
    "mse_partial", "mse_finalize", "sumsq_partial", "scale_by_inv_norm", "batch_norm_stats",
    "batch_norm_apply",
]

_get_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(t: torch.Tensor) -> int:
    idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
    if _get_raw_stream is not None:
        return _get_raw_stream(idx)
    return torch.cuda.current_stream(idx).cuda_stream


def _check_f32(name: str, *ts: torch.Tensor) -> None:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name}: expected a tensor, got {type(t).__name__}")
        if not t.is_cuda:
            raise RuntimeError(f"{name}: tensors must be on a CUDA device (got {t.device})")
        if t.dtype != torch.float32:
            raise RuntimeError(f"{name}: expected float32, got {t.dtype}")
        if not t.is_contiguous():
            raise RuntimeError(f"{name}: tensors must be contiguous")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{name}: tensors on different devices ({dev} vs {t.device})")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _out_like(x: torch.Tensor, out: torch.Tensor | None, name: str, shape=None, dtype=torch.float32):
    shape = tuple(x.shape) if shape is None else tuple(shape)
    if out is None:
        return torch.empty(shape, device=x.device, dtype=dtype)
    if tuple(out.shape) != shape and out.numel() != math.prod(shape):
        raise RuntimeError(f"{name}: out has shape {tuple(out.shape)}, expected {shape}")
    if out.dtype != dtype or not out.is_contiguous() or out.device != x.device:
        raise RuntimeError(f"{name}: out must be a contiguous {dtype} tensor on {x.device}")
    return out


def _workspace(x: torch.Tensor, nbytes: int) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 16), device=x.device, dtype=torch.uint8)


# ---------------------------------------------------------------- elementwise
def _elementwise(fn: str, x: torch.Tensor, out: torch.Tensor | None) -> torch.Tensor:
    _check_f32(fn, x)
    y = _out_like(x, out, fn)
    check(fn, getattr(LIB, fn)(x.data_ptr(), y.data_ptr(), x.numel(), _stream(x)))
    return y


def gelu_tanh(x, out=None):
    """0.5 x (1 + tanh(sqrt(2/pi)(x + 0.044715 x^3))) — candidates/88_MinGPTNewGelu/v1.py:12-19."""
    return _elementwise("kb_gelu_tanh_f32", x, out)


def gelu_erf(x, out=None):
    """x/2 (1 + erf(x / sqrt 2)) — candidates/26_GELU_/v1.py:10-16."""
    return _elementwise("kb_gelu_erf_f32", x, out)


def swish(x, out=None):
    """x sigmoid(x) — candidates/25_Swish/v1.py:10-16."""
    return _elementwise("kb_swish_f32", x, out)


def relu(x, out=None):
    """max(x, 0), NaN propagated — candidates/19_ReLU/v1.py:10-13."""
    return _elementwise("kb_relu_f32", x, out)


def diag_matmul(a, b, out=None):
    """diag(a) @ B as a broadcast row scale, y[i, j] = a[i] * b[i, j] —
    replaces candidates/12_Matmul_with_diagonal_matrices_/v1.py:10-27."""
    fn = "kb_diag_matmul_f32"
    _check_f32(fn, a, b)
    if a.dim() != 1 or b.dim() != 2 or b.shape[0] != a.shape[0]:
        raise RuntimeError(f"{fn}: expected a[N], b[N, M], got {tuple(a.shape)} and {tuple(b.shape)}")
    y = _out_like(b, out, fn)
    check(fn, LIB.kb_diag_matmul_f32(a.data_ptr(), b.data_ptr(), y.data_ptr(), b.shape[0], b.shape[1],
                                     _stream(b)))
    return y


# ---------------------------------------------------------------- row ops
def _rows_cols(x: torch.Tensor, cols: int, name: str) -> tuple[int, int]:
    if cols <= 0 and x.numel() > 0:
        raise RuntimeError(f"{name}: empty normalized dimension")
    if cols > 0 and x.numel() % cols:
        raise RuntimeError(f"{name}: {x.numel()} elements do not split into rows of {cols}")
    return (x.numel() // cols if cols else 0), cols


def layer_norm(x, weight=None, bias=None, eps: float = 1e-5, normalized_size: int | None = None,
               out=None):
    """LayerNorm over the trailing `normalized_size` elements (default: weight.numel() or the
    last dim) — replaces candidates/40_LayerNorm/v1.py:62-80 (which had identity affine)."""
    fn = "kb_layernorm_f32"
    _check_f32(fn, x, weight, bias)
    if normalized_size is None:
        normalized_size = weight.numel() if weight is not None else x.shape[-1]
    for p in (weight, bias):
        if p is not None and p.numel() != normalized_size:
            raise RuntimeError(f"{fn}: affine parameter has {p.numel()} elements, expected {normalized_size}")
    rows, cols = _rows_cols(x, normalized_size, fn)
    y = _out_like(x, out, fn)
    check(fn, LIB.kb_layernorm_f32(x.data_ptr(), _ptr(weight), _ptr(bias), y.data_ptr(), rows, cols,
                                   float(eps), _stream(x)))
    return y


def rms_norm(x, weight=None, eps: float = 1e-5, dim: int = -1, out=None):
    """x / sqrt(mean(x^2 over `dim`) + eps) (* weight) — replaces
    candidates/36_RMSNorm_/v3.py:42-51.  dim = -1 (last-dim rows) or any other
    dim of a contiguous tensor (channel form, e.g. dim 1 of NCHW)."""
    fn = "kb_rmsnorm_f32"
    _check_f32(fn, x, weight)
    d = dim % x.dim() if x.dim() else 0
    F = x.shape[d] if x.dim() else 1
    outer = math.prod(x.shape[:d])
    inner = math.prod(x.shape[d + 1:])
    if weight is not None and weight.numel() != F:
        raise RuntimeError(f"{fn}: weight has {weight.numel()} elements, expected {F}")
    y = _out_like(x, out, fn)
    check(fn, LIB.kb_rmsnorm_f32(x.data_ptr(), _ptr(weight), y.data_ptr(), outer, F, inner,
                                 float(eps), _stream(x)))
    return y


def _softmax_like(fn: str, x, out):
    _check_f32(fn, x)
    cols = x.shape[-1] if x.dim() else 1
    rows, cols = _rows_cols(x, cols, fn)
    y = _out_like(x, out, fn)
    check(fn, getattr(LIB, fn)(x.data_ptr(), y.data_ptr(), rows, cols, _stream(x)))
    return y


def softmax(x, out=None):
    """softmax over the last dim — replaces candidates/23_Softmax/v1.py:47-52."""
    return _softmax_like("kb_softmax_f32", x, out)


def log_softmax(x, out=None):
    """log-softmax over the last dim — replaces candidates/24_LogSoftmax/v1.py:46-51."""
    return _softmax_like("kb_logsoftmax_f32", x, out)


# ---------------------------------------------------------------- dim reductions
def _bij(x: torch.Tensor, dim: int) -> tuple[int, int, int]:
    d = dim % x.dim()
    return math.prod(x.shape[:d]), x.shape[d], math.prod(x.shape[d + 1:])


def _reduced_shape(x, dim, keepdim):
    d = dim % x.dim()
    s = list(x.shape)
    if keepdim:
        s[d] = 1
    else:
        s.pop(d)
    return s


def sum_dim(x, dim: int = 1, keepdim: bool = False, out=None):
    """torch.sum(x, dim) — replaces candidates/47_Sum_reduction_over_a_dimension/v1.py:28-35."""
    fn = "kb_sum_dim1_f32"
    _check_f32(fn, x)
    B, I, J = _bij(x, dim)
    y = _out_like(x, out, fn, _reduced_shape(x, dim, keepdim))
    check(fn, LIB.kb_sum_dim1_f32(x.data_ptr(), y.data_ptr(), B, I, J, _stream(x)))
    return y


def mean_dim(x, dim: int = 1, keepdim: bool = False, out=None):
    """torch.mean(x, dim) — replaces candidates/48_Mean_reduction_over_a_dimension/v1.py:25-32."""
    fn = "kb_mean_dim1_f32"
    _check_f32(fn, x)
    B, I, J = _bij(x, dim)
    y = _out_like(x, out, fn, _reduced_shape(x, dim, keepdim))
    check(fn, LIB.kb_mean_dim1_f32(x.data_ptr(), y.data_ptr(), B, I, J, _stream(x)))
    return y


def argmax_dim(x, dim: int = 1, keepdim: bool = False, out=None):
    """torch.argmax(x, dim), int64, lowest index on ties, NaN is the maximum —
    replaces candidates/51_Argmax_over_a_dimension/v1.py:27-31."""
    fn = "kb_argmax_dim1_f32"
    _check_f32(fn, x)
    B, I, J = _bij(x, dim)
    y = _out_like(x, out, fn, _reduced_shape(x, dim, keepdim), dtype=torch.int64)
    check(fn, LIB.kb_argmax_dim1_f32(x.data_ptr(), y.data_ptr(), B, I, J, _stream(x)))
    return y


# ---------------------------------------------------------------- global reductions
def mse_loss(a, b, out=None):
    """mean((a - b)^2) as a 0-d tensor — replaces candidates/94_MSELoss/v1.py:35-45."""
    fn = "kb_mse_f32"
    _check_f32(fn, a, b)
    if a.shape != b.shape:
        raise RuntimeError(f"{fn}: shape mismatch {tuple(a.shape)} vs {tuple(b.shape)}")
    y = _out_like(a, out, fn, ())
    n = a.numel()
    ws_bytes = LIB.kb_mse_workspace_size(n)
    ws = _workspace(a, ws_bytes)
    check(fn, LIB.kb_mse_f32(a.data_ptr(), b.data_ptr(), y.data_ptr(), n, ws.data_ptr(), ws.numel(),
                             _stream(a)))
    return y


def frobenius_normalize(x, out=None):
    """x / ||x||_F — replaces candidates/37_FrobeniusNorm_/v1.py:48-58."""
    fn = "kb_frobenius_normalize_f32"
    _check_f32(fn, x)
    y = _out_like(x, out, fn)
    n = x.numel()
    ws = _workspace(x, LIB.kb_frobenius_workspace_size(n))
    check(fn, LIB.kb_frobenius_normalize_f32(x.data_ptr(), y.data_ptr(), n, ws.data_ptr(), ws.numel(),
                                             _stream(x)))
    return y


def _f64_buffer(fn, buf, n, device):
    """A caller's fp64 buffer of at least n contiguous elements, or a new one."""
    if buf is None:
        return torch.empty(n, device=device, dtype=torch.float64)
    if buf.dtype != torch.float64 or not buf.is_contiguous() or buf.numel() < n or buf.device != device:
        raise RuntimeError(f"{fn}: expected a contiguous float64 buffer of {n} elements on {device}")
    return buf


def mse_partial(a, b, partial=None):
    """fp64 [sum((a - b)^2), element count] of this shard: one cross-GPU sum
    of it gives mse_finalize both the total and the global count."""
    fn = "kb_mse_partial_f64"
    _check_f32(fn, a, b)
    p = _f64_buffer(fn, partial, 2, a.device)
    n = a.numel()
    ws = _workspace(a, LIB.kb_mse_workspace_size(n))
    check(fn, LIB.kb_mse_partial_f64(a.data_ptr(), b.data_ptr(), p.data_ptr(), n, ws.data_ptr(),
                                     ws.numel(), _stream(a)))
    return p


def mse_finalize(total: torch.Tensor, total_n: int = 0, out=None):
    """total[0] / total_n; total_n 0: divide by the summed count total[1]."""
    fn = "kb_mse_finalize_f32"
    y = out if out is not None else torch.empty((), device=total.device, dtype=torch.float32)
    check(fn, LIB.kb_mse_finalize_f32(total.data_ptr(), y.data_ptr(), int(total_n), _stream(total)))
    return y


def sumsq_partial(x, partial=None):
    fn = "kb_sumsq_partial_f64"
    _check_f32(fn, x)
    p = partial if partial is not None else torch.empty((), device=x.device, dtype=torch.float64)
    n = x.numel()
    ws = _workspace(x, LIB.kb_frobenius_workspace_size(n))
    check(fn, LIB.kb_sumsq_partial_f64(x.data_ptr(), p.data_ptr(), n, ws.data_ptr(), ws.numel(),
                                       _stream(x)))
    return p


def scale_by_inv_norm(x, total_sumsq: torch.Tensor, out=None):
    fn = "kb_scale_by_inv_norm_f32"
    _check_f32(fn, x)
    y = _out_like(x, out, fn)
    check(fn, LIB.kb_scale_by_inv_norm_f32(x.data_ptr(), y.data_ptr(), x.numel(),
                                           total_sumsq.data_ptr(), _stream(x)))
    return y


# ---------------------------------------------------------------- spatial
def max_pool2d(x, kernel_size: int, stride: int | None = None, padding: int = 0, dilation: int = 1,
               out=None):
    """torch.nn.functional.max_pool2d (floor mode) on NCHW — replaces
    candidates/42_Max_Pooling_2D/v1.py:37-44 with stride and dilation honoured."""
    fn = "kb_maxpool2d_f32"
    _check_f32(fn, x)
    if x.dim() != 4:
        raise RuntimeError(f"{fn}: expected NCHW input")
    k, s = int(kernel_size), int(stride if stride is not None else kernel_size)
    p, d = int(padding), int(dilation)
    N, Cc, H, W = x.shape
    OH = (H + 2 * p - d * (k - 1) - 1) // s + 1
    OW = (W + 2 * p - d * (k - 1) - 1) // s + 1
    y = _out_like(x, out, fn, (N, Cc, max(OH, 0), max(OW, 0)))
    check(fn, LIB.kb_maxpool2d_f32(x.data_ptr(), y.data_ptr(), N, Cc, H, W, OH, OW, k, s, p, d,
                                   _stream(x)))
    return y


def batch_norm_train(x, weight=None, bias=None, eps: float = 1e-5, momentum: float = 0.1,
                     running_mean=None, running_var=None, out=None):
    """Training-mode BatchNorm over dim 1 of NC* input — replaces
    candidates/33_BatchNorm/v1.py:53-68 (which had identity affine)."""
    fn = "kb_batchnorm_train_f32"
    _check_f32(fn, x, weight, bias, running_mean, running_var)
    N, Cc = x.shape[0], x.shape[1]
    HW = math.prod(x.shape[2:])
    y = _out_like(x, out, fn)
    ws = _workspace(x, LIB.kb_batchnorm_workspace_size(N, Cc, HW))
    check(fn, LIB.kb_batchnorm_train_f32(x.data_ptr(), _ptr(weight), _ptr(bias), y.data_ptr(), N, Cc,
                                         HW, float(eps), float(momentum), _ptr(running_mean),
                                         _ptr(running_var), ws.data_ptr(), ws.numel(), _stream(x)))
    return y


def batch_norm_stats(x, stats=None):
    """fp64 [2C + 1] of this shard: per-channel sums, per-channel sums of
    squares, elements per channel; one cross-GPU sum of it gives
    batch_norm_apply the global statistics and count."""
    fn = "kb_batchnorm_stats_f64"
    _check_f32(fn, x)
    N, Cc = x.shape[0], x.shape[1]
    HW = math.prod(x.shape[2:])
    st = _f64_buffer(fn, stats, 2 * Cc + 1, x.device)
    ws = _workspace(x, LIB.kb_batchnorm_workspace_size(N, Cc, HW))
    check(fn, LIB.kb_batchnorm_stats_f64(x.data_ptr(), st.data_ptr(), N, Cc, HW, ws.data_ptr(),
                                         ws.numel(), _stream(x)))
    return st


def batch_norm_apply(x, stats, total_count: int = 0, weight=None, bias=None, eps: float = 1e-5,
                     momentum: float = 0.1, running_mean=None, running_var=None, out=None):
    """Normalise with the (summed) stats of batch_norm_stats; total_count 0:
    the element count stats[2C]."""
    fn = "kb_batchnorm_apply_f32"
    _check_f32(fn, x, weight, bias, running_mean, running_var)
    N, Cc = x.shape[0], x.shape[1]
    HW = math.prod(x.shape[2:])
    y = _out_like(x, out, fn)
    check(fn, LIB.kb_batchnorm_apply_f32(x.data_ptr(), _ptr(weight), _ptr(bias), y.data_ptr(),
                                         stats.data_ptr(), N, Cc, HW, int(total_count), float(eps),
                                         float(momentum), _ptr(running_mean), _ptr(running_var),
                                         _stream(x)))
    return y


# ---------------------------------------------------------------- contractions
def matmul(A, B, trans_a: bool = False, out=None):
    """C = op(A) @ B, 3xTF32 on tcgen05 — replaces
    candidates/1_Square_matrix_multiplication_/v1.py:83-102."""
    fn = "kb_sgemm_3xtf32"
    _check_f32(fn, A, B)
    if A.dim() != 2 or B.dim() != 2:
        raise RuntimeError(f"{fn}: expected 2-D operands")
    M, K = (A.shape[1], A.shape[0]) if trans_a else (A.shape[0], A.shape[1])
    if B.shape[0] != K:
        raise RuntimeError(f"{fn}: inner dimensions differ ({K} vs {B.shape[0]})")
    N = B.shape[1]
    y = _out_like(A, out, fn, (M, N))
    ws_bytes = LIB.kb_sgemm_workspace_size(M, N, K, 1 if trans_a else 0)
    if ws_bytes:  # K split into partial tiles for a better-filled grid (deterministic sum)
        fn = "kb_sgemm_3xtf32_ws"
        ws = _workspace(A, ws_bytes)
        check(fn, LIB.kb_sgemm_3xtf32_ws(A.data_ptr(), B.data_ptr(), y.data_ptr(), M, N, K, A.stride(0),
                                         B.stride(0), N, 1 if trans_a else 0, ws.data_ptr(), ws.numel(),
                                         _stream(A)))
        return y
    check(fn, LIB.kb_sgemm_3xtf32(A.data_ptr(), B.data_ptr(), y.data_ptr(), M, N, K, A.stride(0),
                                  B.stride(0), N, 1 if trans_a else 0, _stream(A)))
    return y


def bmm(A, B, out=None):
    """C[b] = A[b] @ B[b] — replaces candidates/3_Batched_matrix_multiplication/v1.py:83-102."""
    fn = "kb_bgemm_3xtf32"
    _check_f32(fn, A, B)
    if A.dim() != 3 or B.dim() != 3 or A.shape[0] != B.shape[0] or A.shape[2] != B.shape[1]:
        raise RuntimeError(f"{fn}: bad shapes {tuple(A.shape)} @ {tuple(B.shape)}")
    bt, M, K = A.shape
    N = B.shape[2]
    y = _out_like(A, out, fn, (bt, M, N))
    check(fn, LIB.kb_bgemm_3xtf32(A.data_ptr(), B.data_ptr(), y.data_ptr(), bt, M, N, K, _stream(A)))
    return y


def matmul_splitk(A, B, out=None):
    """C = A @ B for small M, N and huge K — replaces
    candidates/6_Matmul_with_large_K_dimension_/v1.py:67-78."""
    fn = "kb_gemm_splitk_3xtf32"
    _check_f32(fn, A, B)
    M, K = A.shape
    if B.shape[0] != K:
        raise RuntimeError(f"{fn}: inner dimensions differ")
    N = B.shape[1]
    y = _out_like(A, out, fn, (M, N))
    ws = _workspace(A, LIB.kb_gemm_splitk_workspace_size(M, N, K))
    check(fn, LIB.kb_gemm_splitk_3xtf32(A.data_ptr(), B.data_ptr(), y.data_ptr(), M, N, K,
                                        ws.data_ptr(), ws.numel(), _stream(A)))
    return y


def gemv(A, x, out=None):
    """y = A @ x for A[M, K], x[K] or x[K, 1] — replaces
    candidates/4_Matrix_vector_multiplication_/v1.py:36-43."""
    fn = "kb_gemv_f32"
    _check_f32(fn, A, x)
    M, K = A.shape
    if x.numel() != K:
        raise RuntimeError(f"{fn}: x has {x.numel()} elements, expected {K}")
    shape = (M,) if x.dim() == 1 else (M, 1)
    y = _out_like(A, out, fn, shape)
    check(fn, LIB.kb_gemv_f32(A.data_ptr(), x.data_ptr(), y.data_ptr(), M, K, _stream(A)))
    return y


# ------------------------------------------- listed but unattempted by the reference
# harness/problems.py:45-56 lists 45_Average_Pooling_2D, 89_cumsum and
# 95_CrossEntropyLoss; scripts/milestone_table.py:16-24 marks them not
# attempted.  These follow the torch functions they are named after.
def avg_pool2d(x, kernel_size: int, stride: int | None = None, padding: int = 0,
               count_include_pad: bool = True, divisor_override: int | None = None, out=None):
    """torch.nn.functional.avg_pool2d (floor mode) on NCHW."""
    fn = "kb_avgpool2d_f32"
    _check_f32(fn, x)
    if x.dim() != 4:
        raise RuntimeError(f"{fn}: expected NCHW input")
    k, s, p = int(kernel_size), int(stride if stride is not None else kernel_size), int(padding)
    div = int(divisor_override or 0)
    N, Cc, H, W = x.shape
    OH = (H + 2 * p - k) // s + 1
    OW = (W + 2 * p - k) // s + 1
    y = _out_like(x, out, fn, (N, Cc, max(OH, 0), max(OW, 0)))
    check(fn, LIB.kb_avgpool2d_f32(x.data_ptr(), y.data_ptr(), N, Cc, H, W, OH, OW, k, s, p,
                                   1 if count_include_pad else 0, div, _stream(x)))
    return y


def cumsum(x, dim: int, out=None):
    """torch.cumsum(x, dim) (inclusive prefix sum) on fp32."""
    fn = "kb_cumsum_f32"
    _check_f32(fn, x)
    if x.dim() == 0:
        outer, n, inner = 1, 1, 1
    else:
        outer, n, inner = _bij(x, dim)
    y = _out_like(x, out, fn)
    check(fn, LIB.kb_cumsum_f32(x.data_ptr(), y.data_ptr(), outer, n, inner, _stream(x)))
    return y


def _ce_args(fn, logits, targets):
    _check_f32(fn, logits)
    if logits.dim() != 2:
        raise RuntimeError(f"{fn}: expected logits [N, C], got {tuple(logits.shape)}")
    if not isinstance(targets, torch.Tensor) or targets.dtype != torch.int64:
        raise RuntimeError(f"{fn}: targets must be an int64 tensor")
    if targets.device != logits.device or not targets.is_contiguous():
        raise RuntimeError(f"{fn}: targets must be contiguous and on {logits.device}")
    if targets.numel() != logits.shape[0]:
        raise RuntimeError(f"{fn}: {targets.numel()} targets for {logits.shape[0]} rows")
    return logits.shape


def cross_entropy_partial(logits, targets, ignore_index: int = -100, partial=None):
    """fp64 (sum of row losses, rows not ignored) of this shard, for a
    cross-GPU sum before cross_entropy_finalize."""
    fn = "kb_cross_entropy_partial_f64"
    N, Cc = _ce_args(fn, logits, targets)
    p = partial if partial is not None else torch.empty(2, device=logits.device, dtype=torch.float64)
    ws = _workspace(logits, LIB.kb_cross_entropy_workspace_size(N))
    check(fn, LIB.kb_cross_entropy_partial_f64(logits.data_ptr(), targets.data_ptr(), p.data_ptr(), N, Cc,
                                               int(ignore_index), ws.data_ptr(), ws.numel(), _stream(logits)))
    return p


def cross_entropy_finalize(total: torch.Tensor, out=None):
    fn = "kb_cross_entropy_finalize_f32"
    y = out if out is not None else torch.empty((), device=total.device, dtype=torch.float32)
    check(fn, LIB.kb_cross_entropy_finalize_f32(total.data_ptr(), y.data_ptr(), _stream(total)))
    return y


def cross_entropy(logits, targets, ignore_index: int = -100, out=None):
    """torch.nn.functional.cross_entropy(logits[N, C], targets[N] int64),
    reduction 'mean', no class weights, no label smoothing; a 0-d result."""
    fn = "kb_cross_entropy_f32"
    N, Cc = _ce_args(fn, logits, targets)
    y = _out_like(logits, out, fn, ())
    ws = _workspace(logits, LIB.kb_cross_entropy_workspace_size(N))
    check(fn, LIB.kb_cross_entropy_f32(logits.data_ptr(), targets.data_ptr(), y.data_ptr(), N, Cc,
                                       int(ignore_index), ws.data_ptr(), ws.numel(), _stream(logits)))
    return y


def matmul_splitk_partials(A, B):
    """The K-split partial tiles of A @ B without their reduction:
    (partials [splits, M, N], splits), for a fused cross-GPU reduction."""
    fn = "kb_gemm_splitk_partials_3xtf32"
    _check_f32(fn, A, B)
    M, K = A.shape
    if B.shape[0] != K:
        raise RuntimeError(f"{fn}: inner dimensions differ")
    N = B.shape[1]
    ws = _workspace(A, LIB.kb_gemm_splitk_partials_workspace_size(M, N, K))
    sp = C.c_int(1)
    check(fn, LIB.kb_gemm_splitk_partials_3xtf32(A.data_ptr(), B.data_ptr(), M, N, K, ws.data_ptr(),
                                                 ws.numel(), C.byref(sp), _stream(A)))
    splits = sp.value
    return ws.view(torch.float32)[: splits * M * N].view(splits, M, N), splits
