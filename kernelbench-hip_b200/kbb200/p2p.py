"""Peer-memory communicator for the sharded ops (one process per GPU).

The sharded MSE, Frobenius, BatchNorm, cross-entropy and split-K GEMM each
exchange one small partial per rank.  `PeerComm` replaces the NCCL
all_reduce there with the library's own cooperative kernel over peer memory
(include/kbb200.h, kb_p2p_*): every rank allocates one symmetric buffer,
the buffers are shared through CUDA IPC handles (exchanged once with
torch.distributed), and each call pushes this rank's contribution into every
rank's buffer, raises a system-scope flag on each, waits for the peers' flags
and sums the parts that arrived in rank order — identical bits on every rank.
Plain peer loads and stores over NVLink: no multicast objects.

Every rank must make the same calls in the same order.  A wait that runs
past `timeout_s` makes the kernel record a fault and skip its output;
`check()` raises it, after which the communicator must be closed.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as tdist

from ._lib import LIB, KbError, check


class PeerComm:
    def __init__(self, group=None, payload_bytes: int = 1 << 20, timeout_s: float = 2.0, device=None):
        self.group = group
        self.rank = tdist.get_rank(group)
        self.world = tdist.get_world_size(group)
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.payload_bytes = int(payload_bytes)  # largest all-reduce of one call
        self.buf_bytes = LIB.kb_p2p_buffer_bytes(self.payload_bytes, self.world)
        self.timeout_ns = int(timeout_s * 1e9)
        self.epoch = 0
        self._own = C.c_void_p()
        self._opened: list[int] = []
        with torch.cuda.device(self.device):
            check("kb_p2p_buffer_alloc", LIB.kb_p2p_buffer_alloc(self.buf_bytes, C.byref(self._own)))
            handle = (C.c_char * 64)()
            check("kb_p2p_ipc_handle", LIB.kb_p2p_ipc_handle(self._own, handle))
            handles = [None] * self.world
            tdist.all_gather_object(handles, bytes(handle), group=group)
            ptrs = []
            for p in range(self.world):
                if p == self.rank:
                    ptrs.append(self._own.value)
                    continue
                q = C.c_void_p()
                h = (C.c_char * 64).from_buffer_copy(handles[p])
                check("kb_p2p_ipc_open", LIB.kb_p2p_ipc_open(h, C.byref(q)))
                self._opened.append(q.value)
                ptrs.append(q.value)
            # device table of base pointers (uint64 values stored as int64 bits)
            self.bufs = torch.tensor([p if p < 2**63 else p - 2**64 for p in ptrs], dtype=torch.int64,
                                     device=self.device)
        tdist.barrier(group=group)

    def _next(self) -> int:
        self.epoch = self.epoch % 0xFFFFFFFF + 1  # 1, 2, ... (never 0: flags start zeroed)
        return self.epoch

    def _stream(self, t: torch.Tensor) -> int:
        return torch.cuda.current_stream(t.device).cuda_stream

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        """In-place sum over ranks of a contiguous float64 / float32 device tensor."""
        if t.dtype == torch.float64:
            fn = "kb_p2p_allreduce_f64"
        elif t.dtype == torch.float32:
            fn = "kb_p2p_allreduce_f32"
        else:
            raise RuntimeError(f"PeerComm.all_reduce_: unsupported dtype {t.dtype}")
        if not t.is_contiguous() or t.device != self.device:
            raise RuntimeError("PeerComm.all_reduce_: tensor must be contiguous on the communicator's device")
        check(fn, getattr(LIB, fn)(self.bufs.data_ptr(), self.rank, self.world, self.buf_bytes, t.data_ptr(),
                                   t.data_ptr(), t.numel(), self._next(), self.timeout_ns, self._stream(t)))
        return t

    def splitk_all_reduce(self, partials: torch.Tensor, splits: int, out: torch.Tensor) -> torch.Tensor:
        """out[n] = sum over ranks of (sum over this rank's splits of partials[z, n])."""
        fn = "kb_p2p_splitk_allreduce_f32"
        n = out.numel()
        check(fn, LIB.kb_p2p_splitk_allreduce_f32(self.bufs.data_ptr(), self.rank, self.world, self.buf_bytes,
                                                  partials.data_ptr(), int(splits), out.data_ptr(), n,
                                                  self._next(), self.timeout_ns, self._stream(out)))
        return out

    def check(self) -> None:
        """Synchronise and raise if a wait of this communicator's kernels expired."""
        torch.cuda.synchronize(self.device)
        v = C.c_int(0)
        check("kb_p2p_read_fault", LIB.kb_p2p_read_fault(1, C.byref(v)))
        if v.value:
            phase, peer = v.value >> 8, v.value & 0xFF
            what = {1: "grid barrier", 2: f"signal of rank {peer}"}.get(phase, f"phase {phase}")
            raise KbError("PeerComm", 4, f"wait for the {what} expired")

    def close(self) -> None:
        if self._own.value is None:
            return
        torch.cuda.synchronize(self.device)
        tdist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for q in self._opened:
                check("kb_p2p_ipc_close", LIB.kb_p2p_ipc_close(C.c_void_p(q)))
            self._opened = []
            tdist.barrier(group=self.group)  # no peer still maps our buffer
            check("kb_p2p_buffer_free", LIB.kb_p2p_buffer_free(self._own))
        self._own = C.c_void_p()
