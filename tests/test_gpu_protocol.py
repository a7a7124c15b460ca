"""GPU: every candidate driven the way harness/eval_protected.py drives one.

For each problem: build the candidate from source with the eval's restricted
globals, build the reference model, then for seeds 0-4 draw fresh seeded
inputs, hash them (R1), run reference and candidate, check shape and
closeness, re-hash; finally re-run seed 0 and compare the (shape, numel, min,
max) digest (R2) — harness/eval_protected.py:338-411.  Closeness uses both
the reference's allclose(1e-2) and the library's per-op tolerance.

Also: the candidates accept the reference candidates' constructor forms
(LayerNorm(normalized_shape) with identity affine, RMSNorm(num_features)
over dim 1, BatchNorm(num_features) without affine inputs).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import problems
from tests.opmap import EXACT, ORACLE, assert_close
from tests.protocol import (build_candidate, candidate_path, digest, digest_close,
                            hash_tensor)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", problems.SUBSET)
def test_protocol_small_shapes(name, cuda_device):
    Model_ref, get_inputs, get_init_inputs, _ = problems.load_problem(name, "small")
    cand_cls, _ = build_candidate(candidate_path(name).read_text())
    init = get_init_inputs()
    ref_model = Model_ref(*init).to(cuda_device)
    cand_model = cand_cls(*init).to(cuda_device)
    _, tol = ORACLE[name]
    digests = {}
    for seed in range(5):
        torch.manual_seed(seed)
        inputs = [t.to(cuda_device) for t in get_inputs()]
        pre = [hash_tensor(t) for t in inputs]
        with torch.no_grad():
            want = ref_model(*inputs)
            got = cand_model(*inputs)
        torch.cuda.synchronize()
        assert [hash_tensor(t) for t in inputs] == pre, "R1: candidate mutated its inputs"
        assert got.shape == want.shape
        if tol == EXACT:
            assert torch.equal(got, want)
        else:
            assert torch.allclose(got.float(), want.float(), atol=1e-2, rtol=1e-2)
            assert_close(got.cpu().numpy(), want.cpu().numpy(), tol, f"{name} seed {seed}")
        digests[seed] = digest(got.float())
    torch.manual_seed(0)
    inputs = [t.to(cuda_device) for t in get_inputs()]
    with torch.no_grad():
        again = cand_model(*inputs)
    assert digest_close(digests[0], digest(again.float())), "R2: recompute digest differs"


def test_layernorm_reference_constructor(cuda_device):
    """Model(normalized_shape) normalising the trailing 3 dims, identity affine."""
    cand_cls, _ = build_candidate(candidate_path("40_LayerNorm").read_text())
    x = torch.randn(4, 8, 16, 32, device=cuda_device)
    ref = torch.nn.LayerNorm((8, 16, 32)).to(cuda_device)
    with torch.no_grad():
        got = cand_cls((8, 16, 32))(x)
        want = ref(x)
    assert_close(got.cpu().numpy(), want.cpu().numpy(), 1e-5)


def test_rmsnorm_reference_constructor(cuda_device):
    """Model(num_features, eps) normalising dim 1 of [B, F, H, W]."""
    cand_cls, _ = build_candidate(candidate_path("36_RMSNorm_").read_text())
    x = torch.randn(3, 64, 9, 17, device=cuda_device)
    want = x / torch.sqrt(torch.mean(x ** 2, dim=1, keepdim=True) + 1e-5)
    with torch.no_grad():
        got = cand_cls(64, 1e-5)(x)
    assert_close(got.cpu().numpy(), want.cpu().numpy(), 1e-5)


def test_batchnorm_reference_constructor(cuda_device):
    """Model(num_features) with forward(x): nn.BatchNorm2d defaults, train mode."""
    cand_cls, _ = build_candidate(candidate_path("33_BatchNorm").read_text())
    x = torch.randn(6, 16, 20, 24, device=cuda_device) * 3 + 1
    ref = torch.nn.BatchNorm2d(16).to(cuda_device).train()
    cand = cand_cls(16).to(cuda_device)
    with torch.no_grad():
        want = ref(x)
        got = cand(x)
    assert_close(got.cpu().numpy(), want.cpu().numpy(), 1e-5)
    np.testing.assert_allclose(cand.running_mean.cpu().numpy(), ref.running_mean.cpu().numpy(),
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(cand.running_var.cpu().numpy(), ref.running_var.cpu().numpy(),
                               rtol=1e-5, atol=1e-6)
