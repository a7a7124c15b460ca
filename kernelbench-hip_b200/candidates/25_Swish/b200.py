# 25_Swish on B200 — x * sigmoid(x), one streaming pass
# Drop-in for candidates/25_Swish/v1.py: same ENTRY / Model contract, compiled entry
# served by libkbb200.so (sm_100a) through kbb200.ext.
ENTRY = "swish_entry"

import torch

import kbb200.ext as EXT


class Model(torch.nn.Module):
    def forward(self, x):
        y = torch.empty_like(x)
        EXT.swish_entry(x, y)
        return y


ModelNew = Model
