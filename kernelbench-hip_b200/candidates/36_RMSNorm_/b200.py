# 36_RMSNorm_ on B200 — RMSNorm over the last dim with weight, row read once
# Drop-in for candidates/36_RMSNorm_/v3.py: same ENTRY / Model contract, compiled entry
# served by libkbb200.so (sm_100a) through kbb200.ext.
ENTRY = "rmsnorm_entry"

import torch

import kbb200.ext as EXT


class Model(torch.nn.Module):
    def __init__(self, eps: float = 1e-5):
        super().__init__()
        self.eps = eps

    def forward(self, x, weight):
        y = torch.empty_like(x)
        F = x.size(-1)
        rows = x.numel() // F
        EXT.rmsnorm_entry(x, y, weight, self.eps, rows, F, 1)
        return y


ModelNew = Model
