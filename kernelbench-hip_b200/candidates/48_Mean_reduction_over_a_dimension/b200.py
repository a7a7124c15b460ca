# 48_Mean_reduction_over_a_dimension on B200 — mean over dim 1
# Drop-in for candidates/48_Mean_reduction_over_a_dimension/v1.py: same ENTRY / Model contract, compiled entry
# served by libkbb200.so (sm_100a) through kbb200.ext.
ENTRY = "colreduce_mean_entry"

import torch

import kbb200.ext as EXT


class Model(torch.nn.Module):
    """torch.mean(x, dim=1)"""

    def __init__(self, dim: int = 1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        B, _, J = x.shape
        out = torch.empty(B, J, device=x.device, dtype=torch.float32)
        EXT.colreduce_mean_entry(x, out, 1)
        return out


ModelNew = Model
