"""Workload table: the op families at their benchmark shapes, with the input
distributions and the algorithmic bytes / FLOPs each launch must move.

Algorithmic bytes count every input element read once and every output
element written once (fp32 = 4 B, int64 = 8 B).  Two ops cannot be done in one
read: Frobenius normalisation needs the global norm before any write and
BatchNorm needs the channel statistics before any write, and neither input
fits on chip, so their figures count x twice ("two-read"); the compulsory
single-read figure is given beside it.

Inputs are synthetic and seeded; distributions follow the benchmark
statement: N(0,1); U(-1,1) = 2 * rand - 1; softmax logits N(0, 4) read as
standard deviation 2; GEMM operands with standard deviation 1/sqrt(K);
affine weight 1 + 0.02 N(0,1), bias 0.02 N(0,1).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

F32 = 4


@dataclass(frozen=True)
class Workload:
    name: str                  # op name (kbb200.ops function family)
    problem: str               # candidate / problem id
    family: str                # gelu | rownorm | reductions | spatial | gemm | structured | adjacent
    inputs: tuple              # ((name, shape, dist), ...)
    algo_bytes: int            # bytes per launch (see module doc)
    flops: int = 0             # useful FLOPs per launch (contractions)
    bound: str = "hbm"         # hbm | tensor
    compulsory_bytes: int | None = None
    extra: dict = field(default_factory=dict)

    def numel(self, i: int = 0) -> int:
        return math.prod(self.inputs[i][1])


def _ew(name, problem):
    n = 4096 * 16384
    return Workload(name, problem, "gelu", (("x", (4096, 16384), "normal"),), 2 * F32 * n)


_LN_ROWS, _LN_COLS = 65536, 8192
_SM_ROWS, _SM_COLS = 8192, 32768
_R_B, _R_I, _R_J = 128, 4096, 4096
_MSE_N = 1 << 28
_FRO = (256, 1024, 1024)
_POOL = (32, 64, 512, 512)
_BN = (64, 128, 256, 256)
_CE_ROWS, _CE_CLASSES = 32768, 4096

WORKLOADS: dict[str, Workload] = {w.name: w for w in [
    _ew("gelu_tanh", "88_MinGPTNewGelu"),
    _ew("gelu_erf", "26_GELU_"),
    _ew("swish", "25_Swish"),
    _ew("relu", "19_ReLU"),
    Workload("layer_norm", "40_LayerNorm", "rownorm",
             (("x", (_LN_ROWS, _LN_COLS), "normal"), ("weight", (_LN_COLS,), "gamma"),
              ("bias", (_LN_COLS,), "beta")),
             2 * F32 * _LN_ROWS * _LN_COLS + 2 * F32 * _LN_COLS),
    Workload("rms_norm", "36_RMSNorm_", "rownorm",
             (("x", (_LN_ROWS, _LN_COLS), "normal"), ("weight", (_LN_COLS,), "gamma")),
             2 * F32 * _LN_ROWS * _LN_COLS + F32 * _LN_COLS),
    Workload("softmax", "23_Softmax", "rownorm", (("x", (_SM_ROWS, _SM_COLS), "normal_std2"),),
             2 * F32 * _SM_ROWS * _SM_COLS),
    Workload("log_softmax", "24_LogSoftmax", "rownorm", (("x", (_SM_ROWS, _SM_COLS), "normal_std2"),),
             2 * F32 * _SM_ROWS * _SM_COLS),
    Workload("sum_dim", "47_Sum_reduction_over_a_dimension", "reductions",
             (("x", (_R_B, _R_I, _R_J), "uniform"),), F32 * (_R_B * _R_I * _R_J + _R_B * _R_J)),
    Workload("mean_dim", "48_Mean_reduction_over_a_dimension", "reductions",
             (("x", (_R_B, _R_I, _R_J), "uniform"),), F32 * (_R_B * _R_I * _R_J + _R_B * _R_J)),
    Workload("argmax_dim", "51_Argmax_over_a_dimension", "reductions",
             (("x", (_R_B, _R_I, _R_J), "uniform"),), F32 * _R_B * _R_I * _R_J + 8 * _R_B * _R_J),
    Workload("mse_loss", "94_MSELoss", "reductions",
             (("predictions", (_MSE_N,), "normal"), ("targets", (_MSE_N,), "normal")),
             2 * F32 * _MSE_N + F32),
    Workload("frobenius_normalize", "37_FrobeniusNorm_", "reductions", (("x", _FRO, "normal"),),
             3 * F32 * math.prod(_FRO), compulsory_bytes=2 * F32 * math.prod(_FRO)),
    Workload("max_pool2d", "42_Max_Pooling_2D", "spatial", (("x", _POOL, "normal"),),
             F32 * (math.prod(_POOL) + math.prod(_POOL) // 4),
             extra={"kernel_size": 3, "stride": 2, "padding": 1, "dilation": 1}),
    Workload("batch_norm_train", "33_BatchNorm", "spatial",
             (("x", _BN, "normal"), ("weight", (_BN[1],), "gamma"), ("bias", (_BN[1],), "beta")),
             3 * F32 * math.prod(_BN) + 2 * F32 * _BN[1],
             compulsory_bytes=2 * F32 * math.prod(_BN) + 2 * F32 * _BN[1]),
    Workload("matmul", "1_Square_matrix_multiplication_", "gemm",
             (("A", (8192, 8192), "gemm"), ("B", (8192, 8192), "gemm")),
             3 * F32 * 8192 * 8192, flops=2 * 8192 ** 3, bound="tensor"),
    Workload("bmm", "3_Batched_matrix_multiplication", "gemm",
             (("A", (256, 512, 1024), "gemm"), ("B", (256, 1024, 512), "gemm")),
             F32 * 256 * (512 * 1024 * 2 + 512 * 512), flops=2 * 256 * 512 * 1024 * 512,
             bound="tensor"),
    Workload("matmul_splitk", "6_Matmul_with_large_K_dimension_", "gemm",
             (("A", (256, 4194304), "gemm"), ("B", (4194304, 256), "gemm")),
             F32 * (2 * 256 * 4194304 + 256 * 256), flops=2 * 256 * 256 * 4194304, bound="tensor"),
    Workload("gemv", "4_Matrix_vector_multiplication_", "gemm",
             (("A", (4096, 1048576), "normal"), ("x", (1048576,), "normal")),
             F32 * (4096 * 1048576 + 1048576 + 4096), flops=2 * 4096 * 1048576),
    # the reference's remaining candidates (structured / shaped matmuls)
    Workload("matmul_transposed_a", "16_Matmul_with_transposed_A", "structured",
             (("A", (8192, 8192), "gemm_t"), ("B", (8192, 8192), "gemm")),
             3 * F32 * 8192 * 8192, flops=2 * 8192 ** 3, bound="tensor"),
    Workload("matmul_symmetric", "13_Matmul_for_symmetric_matrices", "structured",
             (("A", (8192, 8192), "gemm_sym"), ("B", (8192, 8192), "gemm_sym")),
             3 * F32 * 8192 * 8192, flops=2 * 8192 ** 3, bound="tensor"),
    Workload("diag_matmul", "12_Matmul_with_diagonal_matrices_", "structured",
             (("A", (4096,), "normal"), ("B", (4096, 4096), "normal")),
             F32 * (4096 + 2 * 4096 * 4096)),
    Workload("matmul_small_k", "7_Matmul_with_small_K_dimension_", "structured",
             (("A", (32768, 64), "gemm"), ("B", (64, 32768), "gemm")),
             F32 * (2 * 32768 * 64 + 32768 * 32768), flops=2 * 32768 * 32768 * 64),
    # problems the reference lists but never attempted
    Workload("avg_pool2d", "45_Average_Pooling_2D", "adjacent", (("x", _POOL, "normal"),),
             F32 * (math.prod(_POOL) + math.prod(_POOL) // 4),
             extra={"kernel_size": 3, "stride": 2, "padding": 1}),
    Workload("cumsum", "89_cumsum", "adjacent", (("x", (_SM_ROWS, _SM_COLS), "normal"),),
             2 * F32 * _SM_ROWS * _SM_COLS),
    Workload("cross_entropy", "95_CrossEntropyLoss", "adjacent",
             (("predictions", (_CE_ROWS, _CE_CLASSES), "normal"), ("targets", (_CE_ROWS,), "labels")),
             F32 * _CE_ROWS * _CE_CLASSES + 8 * _CE_ROWS + F32),
]}

FAMILIES = {
    "gelu": ["gelu_tanh", "gelu_erf", "swish", "relu"],
    "rownorm": ["layer_norm", "rms_norm", "softmax", "log_softmax"],
    "reductions": ["sum_dim", "mean_dim", "argmax_dim", "mse_loss", "frobenius_normalize"],
    "spatial": ["max_pool2d", "batch_norm_train"],
    "gemm": ["matmul", "bmm", "matmul_splitk", "gemv"],
    "structured": ["matmul_transposed_a", "matmul_symmetric", "diag_matmul", "matmul_small_k"],
    "adjacent": ["avg_pool2d", "cumsum", "cross_entropy"],
}


def fill_(t: torch.Tensor, dist: str, gen: torch.Generator, fan_in: int = 1) -> torch.Tensor:
    """Fill `t` in place from the named distribution (see module doc)."""
    if dist == "normal":
        return t.normal_(0.0, 1.0, generator=gen)
    if dist == "normal_std2":
        return t.normal_(0.0, 2.0, generator=gen)
    if dist == "uniform":
        return t.uniform_(-1.0, 1.0, generator=gen)
    if dist == "gamma":
        return t.normal_(1.0, 0.02, generator=gen)
    if dist == "beta":
        return t.normal_(0.0, 0.02, generator=gen)
    if dist == "gemm":
        return t.normal_(0.0, 1.0 / math.sqrt(fan_in), generator=gen)
    if dist == "gemm_t":  # A stored [K, M]
        return t.normal_(0.0, 1.0 / math.sqrt(t.shape[0]), generator=gen)
    if dist == "gemm_sym":  # symmetric, entries ~ N(0, 1/K)
        t.normal_(0.0, 1.0 / math.sqrt(2.0 * t.shape[-1]), generator=gen)
        return t.add_(t.T.clone())
    if dist == "labels":  # int64 class indices in [0, fan_in)
        return t.random_(0, fan_in, generator=gen)
    raise ValueError(dist)


def make_inputs(w: Workload, device, seed: int = 0, shapes: dict | None = None) -> list[torch.Tensor]:
    """Seeded synthetic inputs for workload `w` generated directly on `device`
    (device RNG; the parity tests use CPU-seeded inputs instead)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    out = []
    for name, shape, dist in w.inputs:
        shape = tuple((shapes or {}).get(name, shape))
        dtype = torch.int64 if dist == "labels" else torch.float32
        t = torch.empty(shape, device=device, dtype=dtype)
        if dist == "labels":  # number of classes: the last dim of the first input
            fan_in = out[0].shape[-1]
        else:
            fan_in = shape[-2] if (dist == "gemm" and name == "B") else (shape[-1] if dist == "gemm" else 1)
        out.append(fill_(t, dist, gen, fan_in))
    return out
