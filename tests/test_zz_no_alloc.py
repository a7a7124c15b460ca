"""GPU: the allocation-free BatchNorm entry point.

kb_batchnorm_train_f32_noalloc serves callers that may not allocate device
memory themselves (a host framework owns all device allocations, or the call
sits in a latency-bound loop where cudaMalloc's implicit synchronisation is
not allowed): its scratch is a fixed 128 KiB device array inside the library
instead of caller workspace.  These tests call it through the C ABI and check
it against the workspace entry point, kb_batchnorm_train_f32, and the fp64
oracle, on two calls in a row (the second with a different shape, so leftovers of the first call in
the shared array cannot leak into the result), plus the size limit.

This file is collected last (test_zz_*) so that a failing run that stops at
the first failure has already run every other test.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-5  # the BatchNorm tolerance of the parity tests


def _call_noalloc(x, w, b, y, rm, rv, eps=1e-5, momentum=0.1):
    from kbb200 import ops
    from kbb200._lib import LIB

    N, Cc = x.shape[0], x.shape[1]
    HW = x[0, 0].numel()
    return LIB.kb_batchnorm_train_f32_noalloc(
        x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), N, Cc, HW, eps, momentum,
        rm.data_ptr(), rv.data_ptr(), ops._stream(x))


@pytest.mark.parametrize("shapes", [[(8, 64, 32, 32), (3, 200, 17, 19)]])
def test_noalloc_matches_workspace_entry(shapes, cuda_device):
    from kbb200 import ops
    from oracle import ops as O

    for shape in shapes:  # two calls in a row, different shapes
        g = torch.Generator(device=cuda_device).manual_seed(sum(shape))
        x = torch.randn(shape, device=cuda_device, generator=g) * 1.7 + 0.4
        Cc = shape[1]
        w = 1 + 0.02 * torch.randn(Cc, device=cuda_device, generator=g)
        b = 0.02 * torch.randn(Cc, device=cuda_device, generator=g)
        rm_ref, rv_ref = torch.zeros(Cc, device=cuda_device), torch.ones(Cc, device=cuda_device)
        ref = ops.batch_norm_train(x, w, b, 1e-5, 0.1, rm_ref, rv_ref)
        y = torch.full_like(x, float("nan"))
        rm, rv = torch.zeros(Cc, device=cuda_device), torch.ones(Cc, device=cuda_device)
        assert _call_noalloc(x, w, b, y, rm, rv) == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(y, ref, atol=TOL, rtol=TOL)
        torch.testing.assert_close(rm, rm_ref, atol=TOL, rtol=TOL)
        torch.testing.assert_close(rv, rv_ref, atol=TOL, rtol=TOL)
        # and directly against the fp64 oracle, not only the workspace entry
        xh, wh, bh = x.cpu().numpy(), w.cpu().numpy(), b.cpu().numpy()
        np.testing.assert_allclose(y.cpu().numpy(), O.batch_norm_train(xh, wh, bh), atol=TOL, rtol=TOL)
        erm, erv = O.batch_norm_running_update(xh, np.zeros(Cc), np.ones(Cc))
        np.testing.assert_allclose(rm.cpu().numpy(), erm, atol=TOL, rtol=TOL)
        np.testing.assert_allclose(rv.cpu().numpy(), erv, atol=TOL, rtol=TOL)


def test_noalloc_rejects_more_channels_than_its_scratch(cuda_device):
    from kbb200._lib import LIB

    x = torch.zeros(2, 9000, 1, 4, device=cuda_device)   # 9000 channels > 8192 slots
    w = torch.ones(9000, device=cuda_device)
    b = torch.zeros(9000, device=cuda_device)
    y = torch.empty_like(x)
    rm, rv = torch.zeros(9000, device=cuda_device), torch.ones(9000, device=cuda_device)
    assert _call_noalloc(x, w, b, y, rm, rv) == 2          # KB_ERR_UNSUPPORTED
    assert b"built-in scratch" in LIB.kb_last_error()
