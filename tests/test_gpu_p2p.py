"""GPU, one device: the peer-memory all-reduce kernel (kb_p2p_*) with a
second rank emulated on the host.

The "peer" buffer is a second symmetric buffer on the same GPU; the data the
peer would push into our buffer and its ready flag in our header are written
by the host before the launch, so no kernel waits for another kernel.  Checked: the rank-ordered sum
(float32, float64, in place), the fused split-K form, slot alternation over
epochs, and a wait that runs out (a peer flag that nothing sets) — the
kernel reports it in the fault word and fills dst with NaN.  The real
multi-GPU path is in tests/test_gpu_dist.py.
"""
from __future__ import annotations

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_RANKS = 64  # flags[2][64] uint32 at byte 0 of each buffer (csrc/p2p.cu)


class Emulated:
    """Rank 0 of a world of `world` ranks whose other ranks are played by the
    host: one buffer per rank on this GPU (rank 0 pushes into all of them),
    and the peers' parts and flags written into rank 0's buffer before the
    launch."""

    def __init__(self, device, payload_bytes=1 << 16, world=2):
        from kbb200._lib import LIB, check

        self.LIB, self.check = LIB, check
        self.world = world
        self.buf_bytes = LIB.kb_p2p_buffer_bytes(payload_bytes, self.world)
        self.hdr = LIB.kb_p2p_header_bytes()
        self.cap = ((self.buf_bytes - self.hdr) // 2 // self.world) & ~255  # bytes per rank part
        self.ptrs = []
        for _ in range(world):
            p = C.c_void_p()
            check("alloc", LIB.kb_p2p_buffer_alloc(self.buf_bytes, C.byref(p)))
            self.ptrs.append(p.value)
        self.bufs = torch.tensor(self.ptrs, dtype=torch.int64, device=device)
        self.device = device

    def write(self, addr: int, t: torch.Tensor) -> None:
        """Device-to-device copy of t into raw buffer memory at addr."""
        from cuda.bindings import runtime as rt

        t = t.contiguous()
        torch.cuda.synchronize()
        (err,) = rt.cudaMemcpy(addr, t.data_ptr(), t.numel() * t.element_size(),
                               rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
        assert err == rt.cudaError_t.cudaSuccess, err
        torch.cuda.synchronize()

    def set_peer(self, epoch: int, data: torch.Tensor, peer: int = 1) -> None:
        """What rank `peer` would push into our buffer (part `peer` of slot
        epoch & 1), and its ready flag."""
        slot = epoch & 1
        self.write(self.ptrs[0] + self.hdr + (slot * self.world + peer) * self.cap, data)
        flag = torch.tensor([epoch], dtype=torch.int32, device=self.device)
        self.write(self.ptrs[0] + (slot * MAX_RANKS + peer) * 4, flag)

    def close(self) -> None:
        torch.cuda.synchronize()
        for p in self.ptrs:
            self.LIB.kb_p2p_buffer_free(C.c_void_p(p))


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _fault() -> int:
    from kbb200._lib import LIB

    v = C.c_int(0)
    torch.cuda.synchronize()
    LIB.kb_p2p_read_fault(1, C.byref(v))
    return v.value


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_allreduce_rank_ordered_sum_over_epochs(dtype, cuda_device):
    em = Emulated(cuda_device)
    try:
        fn = em.LIB.kb_p2p_allreduce_f64 if dtype == torch.float64 else em.LIB.kb_p2p_allreduce_f32
        for epoch, n in [(1, 1), (2, 1000), (3, 4097), (4, 2)]:
            mine = torch.randn(n, dtype=dtype, device=cuda_device)
            peer = torch.randn(n, dtype=dtype, device=cuda_device)
            em.set_peer(epoch, peer)
            out = torch.full_like(mine, float("nan"))
            em.check("allreduce", fn(em.bufs.data_ptr(), 0, 2, em.buf_bytes, mine.data_ptr(), out.data_ptr(),
                                     n, epoch, 2_000_000_000, _stream()))
            assert _fault() == 0
            assert torch.equal(out, mine + peer), f"epoch {epoch}"
        # in place (src == dst)
        t = torch.randn(300, dtype=dtype, device=cuda_device)
        peer = torch.randn(300, dtype=dtype, device=cuda_device)
        want = t + peer
        em.set_peer(5, peer)
        em.check("allreduce", fn(em.bufs.data_ptr(), 0, 2, em.buf_bytes, t.data_ptr(), t.data_ptr(), 300, 5,
                                 2_000_000_000, _stream()))
        assert _fault() == 0 and torch.equal(t, want)
    finally:
        em.close()


def test_splitk_fused_reduction(cuda_device):
    em = Emulated(cuda_device)
    try:
        n, splits = 3000, 3
        parts = torch.randn(splits, n, device=cuda_device)
        peer = torch.randn(n, device=cuda_device)
        em.set_peer(1, peer)
        out = torch.empty(n, device=cuda_device)
        em.check("splitk", em.LIB.kb_p2p_splitk_allreduce_f32(em.bufs.data_ptr(), 0, 2, em.buf_bytes,
                                                              parts.data_ptr(), splits, out.data_ptr(), n, 1,
                                                              2_000_000_000, _stream()))
        assert _fault() == 0
        local = (parts[0] + parts[1]) + parts[2]  # split order
        assert torch.equal(out, local + peer)
    finally:
        em.close()


def test_peer_that_never_signals_times_out_and_reports(cuda_device):
    """A flag that nothing sets: the bounded wait expires (50 ms), the fault
    word names phase 2 (peer signal) and rank 1, and dst holds NaN, so an
    in-place exchange that failed cannot pass for this rank's partial."""
    em = Emulated(cuda_device)
    try:
        mine = torch.randn(64, dtype=torch.float64, device=cuda_device)
        out = torch.full_like(mine, 7.0)
        em.check("allreduce", em.LIB.kb_p2p_allreduce_f64(em.bufs.data_ptr(), 0, 2, em.buf_bytes,
                                                          mine.data_ptr(), out.data_ptr(), 64, 1, 50_000_000,
                                                          _stream()))
        assert _fault() == (2 << 8) | 1
        assert bool(torch.isnan(out).all())
        # the device is still usable afterwards
        assert float((mine * 2).sum()) == pytest.approx(float(mine.sum()) * 2)
    finally:
        em.close()


def test_bad_arguments_are_rejected(cuda_device):
    from kbb200._lib import KbError, check

    em = Emulated(cuda_device)
    try:
        x = torch.zeros(4, dtype=torch.float64, device=cuda_device)
        st = em.LIB.kb_p2p_allreduce_f64(em.bufs.data_ptr(), 2, 2, em.buf_bytes, x.data_ptr(), x.data_ptr(),
                                         4, 1, 1_000_000, _stream())
        with pytest.raises(KbError):
            check("kb_p2p_allreduce_f64", st)
        big = em.cap // 8 + 1
        st = em.LIB.kb_p2p_allreduce_f64(em.bufs.data_ptr(), 0, 2, em.buf_bytes, x.data_ptr(), x.data_ptr(),
                                         big, 1, 1_000_000, _stream())
        assert st != 0
    finally:
        em.close()


@pytest.mark.parametrize("world", [4, 8])
def test_allreduce_many_ranks_rank_ordered(world, cuda_device):
    """Rank 0 of 4 and 8 ranks: the standalone peer all-reduce sums every
    rank's part in rank order (the other ranks played by the host)."""
    em = Emulated(cuda_device, world=world)
    try:
        n = 3000
        mine = torch.randn(n, dtype=torch.float64, device=cuda_device)
        parts = [torch.randn(n, dtype=torch.float64, device=cuda_device) for _ in range(1, world)]
        for p, t in enumerate(parts, start=1):
            em.set_peer(3, t, peer=p)
        out = torch.empty_like(mine)
        em.check("allreduce", em.LIB.kb_p2p_allreduce_f64(em.bufs.data_ptr(), 0, world, em.buf_bytes,
                                                          mine.data_ptr(), out.data_ptr(), n, 3, 2_000_000_000,
                                                          _stream()))
        assert _fault() == 0
        want = torch.zeros_like(mine) + mine
        for t in parts:
            want = want + t
        assert torch.equal(out, want)
    finally:
        em.close()


@pytest.mark.parametrize("world", [4, 8])
def test_splitk_fold_many_ranks(world, cuda_device):
    """The fused split-K form as rank 0 of 4 and 8 ranks: its own K-split
    tiles summed in split order, then every rank's part in rank order."""
    em = Emulated(cuda_device, payload_bytes=1 << 18, world=world)
    try:
        n, splits = 65536, 5  # a 256 x 256 C, the split-K benchmark's exchange
        parts = torch.randn(splits, n, device=cuda_device)
        peers = [torch.randn(n, device=cuda_device) for _ in range(1, world)]
        for p, t in enumerate(peers, start=1):
            em.set_peer(1, t, peer=p)
        out = torch.empty(n, device=cuda_device)
        em.check("splitk", em.LIB.kb_p2p_splitk_allreduce_f32(em.bufs.data_ptr(), 0, world, em.buf_bytes,
                                                              parts.data_ptr(), splits, out.data_ptr(), n, 1,
                                                              2_000_000_000, _stream()))
        assert _fault() == 0
        local = parts[0].clone()
        for z in range(1, splits):
            local = local + parts[z]
        want = torch.zeros_like(local) + local
        for t in peers:
            want = want + t
        assert torch.equal(out, want)
    finally:
        em.close()
