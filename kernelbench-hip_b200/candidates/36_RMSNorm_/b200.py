# 36_RMSNorm_ on B200 — RMSNorm over the last dim with weight, row read once
# Drop-in for candidates/36_RMSNorm_/v3.py: same ENTRY / Model contract, compiled entry
# served by libkbb200.so (sm_100a) through kbb200.ext.
ENTRY = "rmsnorm_entry"

import torch

import kbb200.ext as EXT


class Model(torch.nn.Module):
    """RMSNorm.  Given `num_features` (the reference's constructor), x is
    [B, num_features, ...] normalised over dim 1; otherwise over the last dim,
    with an optional per-feature weight."""

    def __init__(self, num_features: int | None = None, eps: float = 1e-5):
        super().__init__()
        self.num_features = num_features
        self.eps = eps

    def forward(self, x, weight=None):
        y = torch.empty_like(x)
        if self.num_features is not None and x.dim() > 2:
            F = x.size(1)
            inner = x[0, 0].numel()
            EXT.rmsnorm_entry(x, y, weight, self.eps, x.size(0) * inner, F, inner)
        else:
            F = x.size(-1)
            EXT.rmsnorm_entry(x, y, weight, self.eps, x.numel() // F, F, 1)
        return y


ModelNew = Model
