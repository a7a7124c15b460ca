# 26_GELU_ on B200 — exact (erf) GELU, one streaming pass
# Drop-in for candidates/26_GELU_/v1.py: same ENTRY / Model contract, compiled entry
# served by libkbb200.so (sm_100a) through kbb200.ext.
ENTRY = "gelu_entry"

import torch

import kbb200.ext as EXT


class Model(torch.nn.Module):
    def forward(self, x):
        y = torch.empty_like(x)
        EXT.gelu_entry(x, y)
        return y


ModelNew = Model
