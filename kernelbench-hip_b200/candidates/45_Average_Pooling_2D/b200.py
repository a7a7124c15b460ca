# 45_Average_Pooling_2D on B200 — AvgPool2d (floor mode, count_include_pad)
# The reference lists this problem but has no candidate for it
# (scripts/milestone_table.py:18); same ENTRY / Model contract as its other
# candidates, compiled entry served by libkbb200.so (sm_100a) through kbb200.ext.
ENTRY = "avgpool_entry"

import torch

import kbb200.ext as EXT


class Model(torch.nn.Module):
    def __init__(self, kernel_size: int = 3, stride: int = 2, padding: int = 1):
        super().__init__()
        self.kernel_size = kernel_size
        self.stride = stride
        self.padding = padding

    def forward(self, x):
        N, C, H, W = x.shape
        K, S, P = self.kernel_size, self.stride, self.padding
        OH = (H + 2 * P - K) // S + 1
        OW = (W + 2 * P - K) // S + 1
        y = torch.empty(N, C, OH, OW, device=x.device, dtype=torch.float32)
        EXT.avgpool_entry(x, y, K, P, S)
        return y


ModelNew = Model
