# 42_Max_Pooling_2D on B200 — MaxPool2d with stride/pad/dilation honoured
# Drop-in for candidates/42_Max_Pooling_2D/v1.py: same ENTRY / Model contract, compiled entry
# served by libkbb200.so (sm_100a) through kbb200.ext.
ENTRY = "maxpool_entry"

import torch

import kbb200.ext as EXT


class Model(torch.nn.Module):
    def __init__(self, kernel_size: int = 3, stride: int = 2, padding: int = 1,
                 dilation: int = 1):
        super().__init__()
        self.kernel_size = kernel_size
        self.stride = stride
        self.padding = padding
        self.dilation = dilation

    def forward(self, x):
        N, C, H, W = x.shape
        K, S, P, D = self.kernel_size, self.stride, self.padding, self.dilation
        OH = (H + 2 * P - D * (K - 1) - 1) // S + 1
        OW = (W + 2 * P - D * (K - 1) - 1) // S + 1
        y = torch.empty(N, C, OH, OW, device=x.device, dtype=torch.float32)
        EXT.maxpool_entry(x, y, K, P, S, D)
        return y


ModelNew = Model
