"""Generate the golden fixtures: seeded inputs and the reference arm's
torch-eager fp32 CPU outputs for every problem at small shapes.

The reference ships no stored outputs; its protected eval pins parity only at
run time against the torch-eager model (harness/eval_protected.py:366-399).
These fixtures freeze that reference arm's answers (torch-eager CPU, the
models in oracle/problems.py) so the oracle and the CUDA kernels are checked
against the same recorded vectors on any machine.

    python tests/golden/make_golden.py [problem ...]   # rewrites tests/golden/*.npz
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import problems  # noqa: E402

# fixture shapes: small, ragged where the op allows it, and covering each
# kernel path family (warp rows, block rows, vector tails)
GOLDEN_SHAPES = {
    "88_MinGPTNewGelu": {"x": (7, 1001)},
    "26_GELU_": {"x": (7, 1001)},
    "25_Swish": {"x": (7, 1001)},
    "19_ReLU": {"x": (7, 1001)},
    "40_LayerNorm": {"x": (6, 2048), "weight": (2048,), "bias": (2048,)},
    "36_RMSNorm_": {"x": (6, 2048), "weight": (2048,)},
    "23_Softmax": {"x": (4, 3000)},
    "24_LogSoftmax": {"x": (4, 3000)},
    "47_Sum_reduction_over_a_dimension": {"x": (2, 129, 130)},
    "48_Mean_reduction_over_a_dimension": {"x": (2, 129, 130)},
    "51_Argmax_over_a_dimension": {"x": (2, 129, 130)},
    "94_MSELoss": {"predictions": (20011,), "targets": (20011,)},
    "37_FrobeniusNorm_": {"x": (2, 33, 65)},
    "42_Max_Pooling_2D": {"x": (2, 2, 34, 64)},
    "33_BatchNorm": {"x": (3, 128, 6, 10), "weight": (128,), "bias": (128,)},
    "1_Square_matrix_multiplication_": {"A": (64, 96), "B": (96, 80)},
    "3_Batched_matrix_multiplication": {"A": (2, 32, 48), "B": (2, 48, 40)},
    "6_Matmul_with_large_K_dimension_": {"A": (16, 2048), "B": (2048, 24)},
    "4_Matrix_vector_multiplication_": {"A": (17, 1031), "x": (1031,)},
    "16_Matmul_with_transposed_A": {"A": (72, 64), "B": (72, 48)},
    "13_Matmul_for_symmetric_matrices": {"A": (64, 64), "B": (64, 64)},
    "12_Matmul_with_diagonal_matrices_": {"A": (33,), "B": (33, 257)},
    "7_Matmul_with_small_K_dimension_": {"A": (96, 64), "B": (64, 80)},
    "45_Average_Pooling_2D": {"x": (2, 3, 34, 64)},
    "89_cumsum": {"x": (3, 5000)},
    "95_CrossEntropyLoss": {"predictions": (37, 1000), "targets": (37,)},
}
SEED = 0


def generate(name: str) -> dict:
    Model, get_inputs, get_init_inputs, _ = problems.load_problem(name, GOLDEN_SHAPES[name])
    torch.manual_seed(SEED)
    inputs = get_inputs()
    model = Model(*get_init_inputs())
    with torch.no_grad():
        out = model(*inputs)
    rec = {f"in{i}": t.numpy() for i, t in enumerate(inputs)}
    rec["out"] = out.numpy()
    if name == "33_BatchNorm":
        rec["running_mean"] = model.running_mean.numpy()
        rec["running_var"] = model.running_var.numpy()
    return rec


def fixture_path(name: str) -> Path:
    return HERE / f"{name}.npz"


def main() -> int:
    torch.set_num_threads(1)
    total = 0
    names = sys.argv[1:] or problems.SUBSET
    for name in names:
        rec = generate(name)
        np.savez_compressed(fixture_path(name), **rec, torch_version=np.array(torch.__version__))
        total += fixture_path(name).stat().st_size
    print(f"wrote {len(names)} fixtures, {total / 1e6:.2f} MB")
    return 0


if __name__ == "__main__":
    sys.exit(main())
