# 89_cumsum on B200 — inclusive prefix sum along one dimension
# The reference lists this problem but has no candidate for it
# (scripts/milestone_table.py:21); same ENTRY / Model contract as its other
# candidates, compiled entry served by libkbb200.so (sm_100a) through kbb200.ext.
ENTRY = "cumsum_entry"

import torch

import kbb200.ext as EXT


class Model(torch.nn.Module):
    def __init__(self, dim: int = 1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        y = torch.empty_like(x)
        EXT.cumsum_entry(x, y, self.dim)
        return y


ModelNew = Model
