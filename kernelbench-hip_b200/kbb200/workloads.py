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
# the 19 operators of the benchmark configs, in config order
FAMILIES["northstar"] = (FAMILIES["gelu"] + FAMILIES["rownorm"] + FAMILIES["reductions"]
                         + FAMILIES["spatial"] + FAMILIES["gemm"])
FAMILIES["all"] = FAMILIES["northstar"] + FAMILIES["structured"] + FAMILIES["adjacent"]

# ---------------------------------------------------------------- sharding
# How each op's global input is partitioned over the ranks of a multi-GPU
# job: input name -> the dimension cut into contiguous shards
# (kbb200.dist.shard_range; the first n % world ranks take one extra unit).
# Inputs not named are replicated on every rank (the GEMM's B, the matvec's
# x, affine parameters).  The output is cut along the same units.
SHARD_DIMS: dict[str, dict[str, int]] = {
    **{n: {"x": 0} for n in ("gelu_tanh", "gelu_erf", "swish", "relu", "layer_norm", "rms_norm",
                             "softmax", "log_softmax", "sum_dim", "mean_dim", "argmax_dim",
                             "frobenius_normalize", "max_pool2d", "batch_norm_train", "avg_pool2d",
                             "cumsum")},
    "mse_loss": {"predictions": 0, "targets": 0},
    "cross_entropy": {"predictions": 0, "targets": 0},
    "matmul": {"A": 0},                      # rows of A and C; B replicated
    "matmul_symmetric": {"A": 0},
    "matmul_small_k": {"A": 0},
    "matmul_transposed_a": {"A": 1},         # A stored [K, M]: columns are C's rows
    "bmm": {"A": 0, "B": 0},                 # batch
    "matmul_splitk": {"A": 1, "B": 0},       # K slices; partial C summed across ranks
    "gemv": {"A": 0},                        # rows of A and y; x replicated
    "diag_matmul": {"A": 0, "B": 0},
}
# The cross-GPU step of the ops whose result spans every shard (one
# collective between a local partial kernel and a local finish, kbb200.dist);
# every other op needs none.
EXCHANGE: dict[str, str] = {
    "mse_loss": "all-reduce of fp64 (sum of squares, count): 16 B",
    "frobenius_normalize": "all-reduce of the fp64 sum of squares: 8 B",
    "batch_norm_train": "all-reduce of fp64 per-channel (sum, sum of squares) + count: 16 C + 8 B",
    "matmul_splitk": "all-reduce of the fp32 partial C: 4 M N B",
    "cross_entropy": "all-reduce of fp64 (sum of losses, rows): 16 B",
}

# Ops that read the very same input tensors as an earlier op of the step (same
# shapes and distribution): the bench keeps one copy on the device and on the
# host.  Each is >= 1 GB and read front to back, so at most the last 126 MB
# of the earlier op's pass can still sit in L2 when the later op starts at
# the front; it is evicted long before the later op gets there.
SHARED_INPUTS = {"rms_norm": "layer_norm", "log_softmax": "softmax", "mean_dim": "sum_dim",
                 "argmax_dim": "sum_dim"}


def shard_shapes(w: Workload, rank: int, world: int) -> dict:
    """Input shapes of rank's shard of workload `w` (all inputs, sharded or
    replicated)."""
    from .dist import shard_range

    dims = SHARD_DIMS.get(w.name, {})
    out = {}
    for name, shape, _ in w.inputs:
        shape = list(shape)
        if name in dims and world > 1:
            d = dims[name]
            lo, hi = shard_range(shape[d], rank, world)
            shape[d] = hi - lo
        out[name] = tuple(shape)
    return out


def shard_fraction(w: Workload, rank: int, world: int) -> float:
    """The share of the op's units (and algorithmic work) a rank holds."""
    if world <= 1:
        return 1.0
    name, d = next(iter(SHARD_DIMS[w.name].items()))
    full = dict((n, s) for n, s, _ in w.inputs)[name][d]
    return shard_shapes(w, rank, world)[name][d] / full


# ---------------------------------------------------------------- rooflines
def roofline_seconds(w: Workload, hbm_gbs: float, tensor_tflops: float) -> float:
    """Lower bound on one launch's time on one B200: the algorithmic bytes at
    the measured copy bandwidth, and for tensor-core contractions also the
    useful FLOPs at the 3xTF32 ceiling (the larger of the two)."""
    t = w.algo_bytes / (hbm_gbs * 1e9)
    if w.bound == "tensor":
        t = max(t, w.flops / (tensor_tflops * 1e12))
    return t


def roofline_bound(w: Workload, hbm_gbs: float, tensor_tflops: float) -> str:
    if w.bound == "tensor" and w.flops / (tensor_tflops * 1e12) >= w.algo_bytes / (hbm_gbs * 1e9):
        return "tensor"
    return "hbm"


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


def make_inputs(w: Workload, device, seed: int = 0, shapes: dict | None = None,
                global_scale: bool = False) -> list[torch.Tensor]:
    """Seeded synthetic inputs for workload `w` generated directly on `device`
    (device RNG; the parity tests use CPU-seeded inputs instead).  `shapes`
    overrides input shapes (a reduced case, or a rank's shard).  The GEMM
    operands' scale 1/sqrt(K) follows the K of the given shapes, or with
    `global_scale` the workload's own K (a shard of a split-K job)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    out = []
    for name, full, dist in w.inputs:
        shape = tuple((shapes or {}).get(name, full))
        dtype = torch.int64 if dist == "labels" else torch.float32
        if dist == "labels":  # number of classes: the last dim of the first input
            fan_in = out[0].shape[-1]
        elif dist == "gemm":  # K: A's last dim, B's second to last
            ref = full if global_scale else shape
            fan_in = ref[-2] if name == "B" else ref[-1]
        else:
            fan_in = 1
        if dist == "gemm_sym" and shape[0] != shape[-1]:
            # rows of a symmetric matrix: draw the whole square, keep the first rows
            sq = fill_(torch.empty(full, device=device, dtype=dtype), dist, gen, fan_in)
            out.append(sq[: shape[0]].contiguous())
            continue
        t = torch.empty(shape, device=device, dtype=dtype)
        out.append(fill_(t, dist, gen, fan_in))
    return out
