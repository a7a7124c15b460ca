"""GPU, one device: the sharded partial / finish entries that kbb200.dist
puts around its one collective, with the shards emulated in one process.

Each "rank" runs the partial kernel on its own slice, the partials are
summed on the device (what the all-reduce does), and the finish kernel runs
on every slice with the count taken from the summed partial (total_n /
total_count 0).  The slices are of unequal sizes and include an empty one,
the cases where a count derived as world_size x local size would be wrong.
Compared with the oracle on the whole input.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _slices(n, sizes):
    assert sum(sizes) == n
    out, lo = [], 0
    for s in sizes:
        out.append((lo, lo + s))
        lo += s
    return out


def test_mse_partials_carry_their_counts(cuda_device):
    from kbb200 import ops as K
    from oracle import ops as O

    g = torch.Generator().manual_seed(11)
    a, b = torch.randn(100_003, generator=g), torch.randn(100_003, generator=g)
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    parts = [K.mse_partial(ad[lo:hi], bd[lo:hi]) for lo, hi in _slices(a.numel(), [70_000, 0, 30_003])]
    for p, (lo, hi) in zip(parts, _slices(a.numel(), [70_000, 0, 30_003])):
        assert p.shape == (2,) and float(p[1]) == hi - lo      # [sum, element count]
    total = torch.stack(parts).sum(0)                         # the collective
    got = float(K.mse_finalize(total))                        # count from total[1]
    assert got == pytest.approx(float(O.mse_loss(a.numpy(), b.numpy())), rel=1e-6)
    assert float(K.mse_finalize(total, a.numel())) == got     # an explicit count agrees


def test_batchnorm_stats_carry_counts_and_empty_shard_updates_running(cuda_device):
    from kbb200 import ops as K
    from oracle import ops as O

    g = torch.Generator().manual_seed(12)
    x = torch.randn(7, 16, 9, 12, generator=g) * 2 + 1
    w, bb = 1 + 0.1 * torch.randn(16, generator=g), 0.1 * torch.randn(16, generator=g)
    sizes = [4, 0, 3]
    xd = x.to(cuda_device)
    stats = [K.batch_norm_stats(xd[lo:hi]) for lo, hi in _slices(7, sizes)]
    for st, n in zip(stats, sizes):
        assert st.shape == (2 * 16 + 1,) and float(st[-1]) == n * 9 * 12
    empty = stats[1].cpu().numpy()
    assert not empty.any(), "an empty shard contributes zero sums and zero elements"
    total = torch.stack(stats).sum(0)                          # the collective
    want = O.batch_norm_train(x.numpy(), w.numpy(), bb.numpy())
    erm, erv = O.batch_norm_running_update(x.numpy(), np.zeros(16), np.ones(16))
    for (lo, hi) in _slices(7, sizes):
        rm = torch.zeros(16, device=cuda_device)
        rv = torch.ones(16, device=cuda_device)
        y = K.batch_norm_apply(xd[lo:hi], total, 0, w.to(cuda_device), bb.to(cuda_device), 1e-5, 0.1, rm, rv)
        np.testing.assert_allclose(y.cpu().numpy(), want[lo:hi], rtol=1e-5, atol=1e-5)
        # every shard, the empty one included, moves its running statistics alike
        np.testing.assert_allclose(rm.cpu().numpy(), erm, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(rv.cpu().numpy(), erv, rtol=1e-5, atol=1e-6)
