# 40_LayerNorm on B200 — LayerNorm over the last dim with affine, row read once
# Drop-in for candidates/40_LayerNorm/v1.py: same ENTRY / Model contract, compiled entry
# served by libkbb200.so (sm_100a) through kbb200.ext.
ENTRY = "layernorm_entry"

import torch

import kbb200.ext as EXT


class Model(torch.nn.Module):
    """LayerNorm over the trailing dims.  `normalized_shape` (the reference's
    constructor argument) fixes the normalised size; without it the size is
    weight.numel() or the last dim.  weight/bias omitted = identity affine,
    as the reference candidate's nn.LayerNorm defaults."""

    def __init__(self, normalized_shape=None, eps: float = 1e-5):
        super().__init__()
        if isinstance(normalized_shape, int):
            normalized_shape = (normalized_shape,)
        self.normalized_shape = tuple(normalized_shape) if normalized_shape is not None else None
        self.eps = eps

    def forward(self, x, weight=None, bias=None):
        y = torch.empty_like(x)
        if self.normalized_shape is not None:
            size = 1
            for d in self.normalized_shape:
                size *= d
            if weight is not None:
                weight = weight.reshape(-1)
            if bias is not None:
                bias = bias.reshape(-1)
            if weight is None and bias is None:
                EXT.layernorm_entry(x, y, None, None, self.eps, size)
                return y
        EXT.layernorm_entry(x, y, weight, bias, self.eps)
        return y


ModelNew = Model
