"""GPU, one device: the fused sharded reductions (kb_mse_sharded_f32,
kb_sumsq_sharded_f64, kb_batchnorm_stats_sharded_f64) — the partial pass and
the peer exchange in one launch — with the second rank played by the host,
as in tests/test_gpu_p2p.py: its folded values and ready flag are written
into this rank's buffer before the launch, so no kernel waits for another.

Checked: the exchanged result equals this rank's own partial (the unfused
entry) plus the peer's values, over several epochs with one reused
workspace (the arrival counter must come back to zero); a peer that sends
zeros leaves the single-GPU result bit for bit; uneven and empty shards
carry their element count; an expired wait yields NaN and the fault word.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from tests.test_gpu_p2p import Emulated, _fault, _stream

pytestmark = pytest.mark.gpu
WAIT_NS = 2_000_000_000


def _ws(em, nbytes):
    return torch.zeros(int(nbytes), dtype=torch.uint8, device=em.device)


def test_fused_mse_matches_local_plus_peer(cuda_device):
    from kbb200 import ops

    em = Emulated(cuda_device)
    try:
        ws = _ws(em, em.LIB.kb_sharded_workspace_size())
        g = torch.Generator(device=cuda_device).manual_seed(0)
        for epoch, (n, peer_sum, peer_n) in enumerate([(1 << 20, 0.0, 0.0), (1000003, 512.25, 77.0),
                                                       (0, 9.5, 3.0), (5, 1.0, 1.0)], start=1):
            a = torch.randn(max(n, 1), device=cuda_device, generator=g)[:n]
            b = torch.randn(max(n, 1), device=cuda_device, generator=g)[:n]
            em.set_peer(epoch, torch.tensor([peer_sum, peer_n], dtype=torch.float64, device=cuda_device))
            out = torch.full((), float("nan"), device=cuda_device)
            em.check("mse", em.LIB.kb_mse_sharded_f32(a.data_ptr(), b.data_ptr(), out.data_ptr(), n, ws.data_ptr(),
                                                      ws.numel(), em.bufs.data_ptr(), 0, 2, em.buf_bytes, epoch,
                                                      WAIT_NS, _stream()))
            assert _fault() == 0
            local = ops.mse_partial(a, b)  # [sum, count], the unfused partial entry
            want = (float(local[0]) + peer_sum) / (n + peer_n)
            assert float(out) == pytest.approx(want, rel=1e-6), (epoch, float(out), want)
            if peer_n == 0:  # nothing from the peer: the single-GPU result, bit for bit
                assert torch.equal(out, ops.mse_loss(a, b))
        assert int(ws[:4].view(torch.int32)) == 0, "arrival counter not reset"
    finally:
        em.close()


def test_fused_sumsq_and_scale(cuda_device):
    from kbb200 import ops

    em = Emulated(cuda_device)
    try:
        ws = _ws(em, em.LIB.kb_sharded_workspace_size())
        x = torch.randn(3, 64, 129, device=cuda_device)
        for epoch, peer in enumerate([0.0, 1234.5], start=1):
            em.set_peer(epoch, torch.tensor([peer], dtype=torch.float64, device=cuda_device))
            total = torch.empty((), dtype=torch.float64, device=cuda_device)
            em.check("sumsq", em.LIB.kb_sumsq_sharded_f64(x.data_ptr(), total.data_ptr(), x.numel(), ws.data_ptr(),
                                                          ws.numel(), em.bufs.data_ptr(), 0, 2, em.buf_bytes, epoch,
                                                          WAIT_NS, _stream()))
            assert _fault() == 0
            local = ops.sumsq_partial(x)
            assert float(total) == float(local) + peer
            y = ops.scale_by_inv_norm(x, total)
            want = x.double() / np.sqrt(float(total))
            torch.testing.assert_close(y.double(), want, atol=1e-6, rtol=1e-5)
    finally:
        em.close()


@pytest.mark.parametrize("shape", [(8, 128, 64, 64), (3, 40, 17, 19), (0, 16, 8, 8)])
def test_fused_batchnorm_stats(shape, cuda_device):
    from kbb200 import ops

    em = Emulated(cuda_device, payload_bytes=1 << 16)
    try:
        N, Cc, H, W = shape
        ws = _ws(em, em.LIB.kb_batchnorm_sharded_workspace_size(N, Cc, H * W))
        x = torch.randn(shape, device=cuda_device) * 1.3 + 0.2
        for epoch in (1, 2):
            peer = torch.rand(2 * Cc + 1, dtype=torch.float64, device=cuda_device) * 100
            em.set_peer(epoch, peer)
            stats = torch.full((2 * Cc + 1,), float("nan"), dtype=torch.float64, device=cuda_device)
            em.check("bn", em.LIB.kb_batchnorm_stats_sharded_f64(x.data_ptr(), stats.data_ptr(), N, Cc, H * W,
                                                                 ws.data_ptr(), ws.numel(), em.bufs.data_ptr(), 0, 2,
                                                                 em.buf_bytes, epoch, WAIT_NS, _stream()))
            assert _fault() == 0
            local = ops.batch_norm_stats(x)  # [sums | sums of squares | elements], unfused entry
            assert torch.equal(stats, local + peer)
        assert int(ws[:4].view(torch.int32)) == 0, "arrival counter not reset"
    finally:
        em.close()


def test_fused_peer_that_never_signals_gives_nan(cuda_device):
    """No flag from the peer: the last CTA's bounded wait expires (50 ms), the
    fault word names the peer signal of rank 1, the result is NaN, and the
    workspace counter is back at zero."""
    em = Emulated(cuda_device)
    try:
        ws = _ws(em, em.LIB.kb_sharded_workspace_size())
        a = torch.randn(4096, device=cuda_device)
        out = torch.zeros((), device=cuda_device)
        em.check("mse", em.LIB.kb_mse_sharded_f32(a.data_ptr(), a.data_ptr(), out.data_ptr(), 4096, ws.data_ptr(),
                                                  ws.numel(), em.bufs.data_ptr(), 0, 2, em.buf_bytes, 1, 50_000_000,
                                                  _stream()))
        assert _fault() == (2 << 8) | 1
        assert bool(torch.isnan(out))
        assert int(ws[:4].view(torch.int32)) == 0
    finally:
        em.close()


def test_fused_rejects_oversized_exchange(cuda_device):
    em = Emulated(cuda_device, payload_bytes=1024)
    try:
        Cc = 100  # 201 doubles > a 1 KiB slot
        x = torch.zeros(2, Cc, 4, 4, device=cuda_device)
        stats = torch.empty(2 * Cc + 1, dtype=torch.float64, device=cuda_device)
        ws = _ws(em, em.LIB.kb_batchnorm_sharded_workspace_size(2, Cc, 16))
        st = em.LIB.kb_batchnorm_stats_sharded_f64(x.data_ptr(), stats.data_ptr(), 2, Cc, 16, ws.data_ptr(),
                                                   ws.numel(), em.bufs.data_ptr(), 0, 2, em.buf_bytes, 1, WAIT_NS,
                                                   _stream())
        assert st != 0 and b"exceeds" in em.LIB.kb_last_error()
    finally:
        em.close()


@pytest.mark.parametrize("world", [4, 8])
def test_fused_exchange_with_many_ranks(world, cuda_device):
    """Rank 0 of 4 and 8 ranks (the others played by the host): the slot
    layout for that world size, the wait for every peer's flag, and the sum
    in rank order over all parts, for the MSE and BatchNorm exchanges."""
    from kbb200 import ops

    em = Emulated(cuda_device, payload_bytes=1 << 16, world=world)
    try:
        ws = _ws(em, max(em.LIB.kb_sharded_workspace_size(), em.LIB.kb_batchnorm_sharded_workspace_size(8, 128, 1024)))
        g = torch.Generator(device=cuda_device).manual_seed(world)
        a = torch.randn(1 << 20, device=cuda_device, generator=g)
        b = torch.randn(1 << 20, device=cuda_device, generator=g)
        peers = [torch.tensor([float(10 * p), float(p)], dtype=torch.float64, device=cuda_device)
                 for p in range(1, world)]
        for p, t in enumerate(peers, start=1):
            em.set_peer(1, t, peer=p)
        out = torch.empty((), device=cuda_device)
        em.check("mse", em.LIB.kb_mse_sharded_f32(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(),
                                                  ws.data_ptr(), ws.numel(), em.bufs.data_ptr(), 0, world,
                                                  em.buf_bytes, 1, WAIT_NS, _stream()))
        assert _fault() == 0
        local = ops.mse_partial(a, b)
        tot = float(local[0])
        cnt = float(local[1])
        for t in peers:  # rank order
            tot += float(t[0])
            cnt += float(t[1])
        assert float(out) == pytest.approx(tot / cnt, rel=1e-6)

        x = torch.randn(8, 128, 32, 32, device=cuda_device, generator=g)
        pst = [torch.rand(257, dtype=torch.float64, device=cuda_device, generator=g) for _ in range(1, world)]
        for p, t in enumerate(pst, start=1):
            em.set_peer(2, t, peer=p)
        stats = torch.empty(257, dtype=torch.float64, device=cuda_device)
        em.check("bn", em.LIB.kb_batchnorm_stats_sharded_f64(x.data_ptr(), stats.data_ptr(), 8, 128, 1024,
                                                             ws.data_ptr(), ws.numel(), em.bufs.data_ptr(), 0,
                                                             world, em.buf_bytes, 2, WAIT_NS, _stream()))
        assert _fault() == 0
        want = ops.batch_norm_stats(x)
        for t in pst:
            want = want + t
        torch.testing.assert_close(stats, want, rtol=1e-12, atol=1e-9)
    finally:
        em.close()
