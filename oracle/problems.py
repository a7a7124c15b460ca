"""Torch-eager fp32 reference models at the benchmark shapes (test oracle).

The reference's protected eval builds the reference model from a problem
definition — `Model`, `get_inputs()`, `get_init_inputs()`
(harness/problems.py:3-5, :62-74) — and compares each candidate against
`Model_ref(*init)(*get_inputs())` on seeds 0-4 (harness/eval_protected.py:
338-399).  The KernelBench problem files it loads are not vendored, so this
module restates each op from its torch semantics, with the benchmark shapes
and input distributions, behind the same three-name interface:

    Model, get_inputs, get_init_inputs, src = load_problem("40_LayerNorm")

`get_inputs()` draws from torch's global CPU generator, so callers seed it
first (torch.manual_seed(seed)), as eval_protected.make_inputs does.  Affine
parameters are inputs, not module parameters, so that a reference model and
a candidate built back to back without reseeding (eval_protected.py:346-347)
see identical values.  `load_problem(name, shapes=...)` overrides shapes for
small CPU-checkable cases.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


# ------------------------------------------------------------------ models
class GeluTanh(nn.Module):
    """y = 0.5 x (1 + tanh(sqrt(2/pi)(x + 0.044715 x^3))), evaluated as the
    eager op chain (mul / add / pow / tanh)."""

    def forward(self, x):
        inner = math.sqrt(2.0 / math.pi) * (x + 0.044715 * torch.pow(x, 3.0))
        return 0.5 * x * (1.0 + torch.tanh(inner))


class GeluErf(nn.Module):
    def forward(self, x):
        return F.gelu(x)


class Swish(nn.Module):
    def forward(self, x):
        return x * torch.sigmoid(x)


class Relu(nn.Module):
    def forward(self, x):
        return torch.relu(x)


class LayerNormLast(nn.Module):
    def __init__(self, eps: float = 1e-5):
        super().__init__()
        self.eps = eps

    def forward(self, x, weight, bias):
        return F.layer_norm(x, (weight.numel(),), weight, bias, self.eps)


class RmsNormLast(nn.Module):
    def __init__(self, eps: float = 1e-5):
        super().__init__()
        self.eps = eps

    def forward(self, x, weight):
        return x / torch.sqrt(torch.mean(x * x, dim=-1, keepdim=True) + self.eps) * weight


class Softmax(nn.Module):
    def forward(self, x):
        return torch.softmax(x, dim=-1)


class LogSoftmax(nn.Module):
    def forward(self, x):
        return torch.log_softmax(x, dim=-1)


class SumDim(nn.Module):
    def __init__(self, dim: int = 1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        return torch.sum(x, dim=self.dim, keepdim=True)


class MeanDim(nn.Module):
    def __init__(self, dim: int = 1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        return torch.mean(x, dim=self.dim)


class ArgmaxDim(nn.Module):
    def __init__(self, dim: int = 1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        return torch.argmax(x, dim=self.dim)


class MseLoss(nn.Module):
    def forward(self, predictions, targets):
        return torch.mean((predictions - targets) ** 2)


class FrobeniusNormalize(nn.Module):
    def forward(self, x):
        return x / torch.norm(x, p="fro")


class MaxPool(nn.Module):
    def __init__(self, kernel_size: int = 3, stride: int = 2, padding: int = 1, dilation: int = 1):
        super().__init__()
        self.pool = nn.MaxPool2d(kernel_size, stride, padding, dilation)

    def forward(self, x):
        return self.pool(x)


class BatchNormTrain(nn.Module):
    """Training-mode BatchNorm2d with batch statistics; running buffers start
    at (0, 1) and are updated as nn.BatchNorm2d does."""

    def __init__(self, num_features: int = 128, eps: float = 1e-5, momentum: float = 0.1):
        super().__init__()
        self.eps, self.momentum = eps, momentum
        self.register_buffer("running_mean", torch.zeros(num_features))
        self.register_buffer("running_var", torch.ones(num_features))

    def forward(self, x, weight, bias):
        return F.batch_norm(x, self.running_mean, self.running_var, weight, bias, True,
                            self.momentum, self.eps)


class Matmul(nn.Module):
    def forward(self, A, B):
        return torch.matmul(A, B)


class MatmulTransposedA(nn.Module):
    """C = A^T @ B with A stored [K, M]."""

    def forward(self, A, B):
        return torch.matmul(A.T, B)


class DiagMatmul(nn.Module):
    """diag(A) @ B, evaluated as the broadcast row scale A[:, None] * B."""

    def forward(self, A, B):
        return A.unsqueeze(1) * B


class Bmm(nn.Module):
    def forward(self, A, B):
        return torch.bmm(A, B)


class AvgPool(nn.Module):
    def __init__(self, kernel_size: int = 3, stride: int = 2, padding: int = 1):
        super().__init__()
        self.pool = nn.AvgPool2d(kernel_size, stride, padding)

    def forward(self, x):
        return self.pool(x)


class Cumsum(nn.Module):
    def __init__(self, dim: int = 1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        return torch.cumsum(x, dim=self.dim)


class CrossEntropy(nn.Module):
    def forward(self, predictions, targets):
        return F.cross_entropy(predictions, targets)


# ------------------------------------------------------------------ registry
# name -> (model class, init inputs, ((input name, shape, dist), ...), small shapes)
_N_EW = (4096, 16384)
PROBLEMS: dict[str, tuple] = {
    "88_MinGPTNewGelu": (GeluTanh, [], (("x", _N_EW, "normal"),), {"x": (37, 301)}),
    "26_GELU_": (GeluErf, [], (("x", _N_EW, "normal"),), {"x": (37, 301)}),
    "25_Swish": (Swish, [], (("x", _N_EW, "normal"),), {"x": (37, 301)}),
    "19_ReLU": (Relu, [], (("x", _N_EW, "normal"),), {"x": (37, 301)}),
    "40_LayerNorm": (LayerNormLast, [],
                     (("x", (65536, 8192), "normal"), ("weight", (8192,), "gamma"),
                      ("bias", (8192,), "beta")),
                     {"x": (33, 8192), "weight": (8192,), "bias": (8192,)}),
    "36_RMSNorm_": (RmsNormLast, [],
                    (("x", (65536, 8192), "normal"), ("weight", (8192,), "gamma")),
                    {"x": (33, 8192), "weight": (8192,)}),
    "23_Softmax": (Softmax, [], (("x", (8192, 32768), "normal_std2"),), {"x": (5, 32768)}),
    "24_LogSoftmax": (LogSoftmax, [], (("x", (8192, 32768), "normal_std2"),), {"x": (5, 32768)}),
    "47_Sum_reduction_over_a_dimension": (SumDim, [1], (("x", (128, 4096, 4096), "uniform"),),
                                          {"x": (3, 257, 260)}),
    "48_Mean_reduction_over_a_dimension": (MeanDim, [1], (("x", (128, 4096, 4096), "uniform"),),
                                           {"x": (3, 257, 260)}),
    "51_Argmax_over_a_dimension": (ArgmaxDim, [1], (("x", (128, 4096, 4096), "uniform"),),
                                   {"x": (3, 257, 260)}),
    "94_MSELoss": (MseLoss, [], (("predictions", (1 << 28,), "normal"),
                                 ("targets", (1 << 28,), "normal")),
                   {"predictions": (100003,), "targets": (100003,)}),
    "37_FrobeniusNorm_": (FrobeniusNormalize, [], (("x", (256, 1024, 1024), "normal"),),
                          {"x": (3, 64, 129)}),
    "42_Max_Pooling_2D": (MaxPool, [3, 2, 1, 1], (("x", (32, 64, 512, 512), "normal"),),
                          {"x": (2, 3, 128, 128)}),
    "33_BatchNorm": (BatchNormTrain, [128], (("x", (64, 128, 256, 256), "normal"),
                                             ("weight", (128,), "gamma"), ("bias", (128,), "beta")),
                     {"x": (4, 128, 16, 20), "weight": (128,), "bias": (128,)}),
    "1_Square_matrix_multiplication_": (Matmul, [], (("A", (8192, 8192), "gemm"),
                                                     ("B", (8192, 8192), "gemm")),
                                        {"A": (256, 192), "B": (192, 320)}),
    "3_Batched_matrix_multiplication": (Bmm, [], (("A", (256, 512, 1024), "gemm"),
                                                  ("B", (256, 1024, 512), "gemm")),
                                        {"A": (3, 128, 96), "B": (3, 96, 256)}),
    "6_Matmul_with_large_K_dimension_": (Matmul, [], (("A", (256, 4194304), "gemm"),
                                                      ("B", (4194304, 256), "gemm")),
                                         {"A": (256, 65536), "B": (65536, 256)}),
    "4_Matrix_vector_multiplication_": (Matmul, [], (("A", (4096, 1048576), "normal"),
                                                     ("x", (1048576,), "normal")),
                                        {"A": (64, 4099), "x": (4099,)}),
}

# the remaining candidates of the reference (structured and shaped matmuls)
PROBLEMS.update({
    "16_Matmul_with_transposed_A": (MatmulTransposedA, [], (("A", (8192, 8192), "gemm_t"),
                                                           ("B", (8192, 8192), "gemm")),
                                    {"A": (160, 96), "B": (160, 200)}),
    "13_Matmul_for_symmetric_matrices": (Matmul, [], (("A", (8192, 8192), "gemm_sym"),
                                                      ("B", (8192, 8192), "gemm_sym")),
                                         {"A": (192, 192), "B": (192, 192)}),
    "12_Matmul_with_diagonal_matrices_": (DiagMatmul, [], (("A", (4096,), "normal"),
                                                           ("B", (4096, 4096), "normal")),
                                          {"A": (67,), "B": (67, 300)}),
    "7_Matmul_with_small_K_dimension_": (Matmul, [], (("A", (32768, 64), "gemm"),
                                                      ("B", (64, 32768), "gemm")),
                                         {"A": (300, 64), "B": (64, 520)}),
})

# problems the reference lists but never attempted (harness/problems.py:45-56,
# scripts/milestone_table.py:16-24).  Shapes: cross-entropy as the
# reference's recorded baseline (results/baselines.json: logits [32768,
# 4096]); average pooling on the max-pooling input with the same window;
# cumsum along the rows of a 1 GiB matrix, the softmax shape.
PROBLEMS.update({
    "45_Average_Pooling_2D": (AvgPool, [3, 2, 1], (("x", (32, 64, 512, 512), "normal"),),
                              {"x": (2, 3, 128, 128)}),
    "89_cumsum": (Cumsum, [1], (("x", (8192, 32768), "normal"),), {"x": (5, 9000)}),
    "95_CrossEntropyLoss": (CrossEntropy, [], (("predictions", (32768, 4096), "normal"),
                                               ("targets", (32768,), "labels")),
                            {"predictions": (300, 1000), "targets": (300,)}),
})

SUBSET = list(PROBLEMS)


def draw(shape, dist: str, fan_in: int = 1) -> torch.Tensor:
    """One input tensor from torch's global CPU generator."""
    if dist == "normal":
        return torch.randn(shape)
    if dist == "normal_std2":
        return torch.randn(shape) * 2.0
    if dist == "uniform":
        return torch.rand(shape) * 2.0 - 1.0
    if dist == "gamma":
        return 1.0 + 0.02 * torch.randn(shape)
    if dist == "beta":
        return 0.02 * torch.randn(shape)
    if dist == "gemm":
        return torch.randn(shape) / math.sqrt(fan_in)
    if dist == "gemm_t":  # A stored [K, M]: scaled by 1/sqrt(K) with K the leading dim
        return torch.randn(shape) / math.sqrt(shape[0])
    if dist == "gemm_sym":  # symmetric, entries ~ N(0, 1/K)
        r = torch.randn(shape) / math.sqrt(shape[-1])
        return (r + r.T) * (0.5 ** 0.5)
    if dist == "labels":  # class indices in [0, fan_in)
        return torch.randint(0, fan_in, shape, dtype=torch.int64)
    raise ValueError(dist)


def input_spec(name: str, shapes: dict | str | None = None):
    _, _, spec, small = PROBLEMS[name]
    if shapes == "small":
        shapes = small
    shapes = shapes or {}
    out = []
    for nm, shape, dist in spec:
        shape = tuple(shapes.get(nm, shape))
        if dist in ("gemm", "gemm_sym"):
            fan_in = shape[-2] if nm == "B" else shape[-1]
        elif dist == "labels":  # number of classes: the last dim of the first input
            fan_in = out[0][1][-1]
        else:
            fan_in = 1
        out.append((nm, shape, dist, fan_in))
    return out


def load_problem(name: str, shapes: dict | str | None = None):
    """(Model, get_inputs, get_init_inputs, src) as harness/problems.py:62-74."""
    if name not in PROBLEMS:
        raise FileNotFoundError(f"problem not found: {name}")
    cls, init, _, _ = PROBLEMS[name]
    spec = input_spec(name, shapes)

    def get_inputs():
        return [draw(shape, dist, fan_in) for _, shape, dist, fan_in in spec]

    def get_init_inputs():
        return list(init)

    return cls, get_inputs, get_init_inputs, None


def subset_names(only: list[str] | None = None) -> list[str]:
    return list(only) if only else list(SUBSET)
