# 47_Sum_reduction_over_a_dimension on B200 — sum over dim 1, keepdim
# Drop-in for candidates/47_Sum_reduction_over_a_dimension/v1.py: same ENTRY / Model contract, compiled entry
# served by libkbb200.so (sm_100a) through kbb200.ext.
ENTRY = "colreduce_entry"

import torch

import kbb200.ext as EXT


class Model(torch.nn.Module):
    """torch.sum(x, dim=1, keepdim=True)"""

    def __init__(self, dim: int = 1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        B, _, J = x.shape
        out = torch.empty(B, 1, J, device=x.device, dtype=torch.float32)
        EXT.colreduce_entry(x, out.view(B, J), 0)
        return out


ModelNew = Model
