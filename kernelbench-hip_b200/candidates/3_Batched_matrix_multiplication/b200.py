# 3_Batched_matrix_multiplication on B200 — batched 3xTF32 tcgen05 GEMM
# Drop-in for candidates/3_Batched_matrix_multiplication/v1.py: same ENTRY / Model contract, compiled entry
# served by libkbb200.so (sm_100a) through kbb200.ext.
ENTRY = "sgemm_entry"

import torch

import kbb200.ext as EXT


class Model(torch.nn.Module):
    """torch.matmul(A, B) on tcgen05 tensor cores (3xTF32)."""
    TRANS_A = False
    BATCHED = True

    def forward(self, A, B):
        if self.BATCHED:
            C = torch.empty(A.size(0), A.size(1), B.size(2), device=A.device, dtype=torch.float32)
        else:
            M = A.size(1) if self.TRANS_A else A.size(0)
            C = torch.empty(M, B.size(1), device=A.device, dtype=torch.float32)
        EXT.sgemm_entry(A, B, C, 1 if self.TRANS_A else 0, A.size(0) if self.BATCHED else 1)
        return C


ModelNew = Model
