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

For MSE, Frobenius and BatchNorm the exchange is fused into the kernel that
computes the shard's partial (`mse_loss`, `sumsq`, `batch_norm_stats`): the
CTA that finishes the partial pass last pushes the folded values to every
peer and sums what arrived, so partial, all-reduce and finish are one
launch.  Those calls reuse one zeroed workspace owned by the communicator,
so a communicator serves one stream at a time (its calls are ordered on the
stream anyway: every rank makes the same calls in the same order).

Every rank must make the same calls in the same order.  A wait that runs
past `timeout_s` makes the kernel record a fault and write NaN as its
output; `check()` raises it, after which the communicator must be closed.
"""
from __future__ import annotations

import ctypes as C
import math

import torch
import torch.distributed as tdist

from ._lib import LIB, KbError, check


class PeerComm:
    def __init__(self, group=None, payload_bytes: int = 1 << 20, timeout_s: float = 2.0, device=None,
                 fused: bool = True):
        self.group = group
        self.fused = fused  # sharded MSE / Frobenius / BatchNorm as one launch each (kbb200.dist)
        self.rank = tdist.get_rank(group)
        self.world = tdist.get_world_size(group)
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.payload_bytes = int(payload_bytes)  # largest all-reduce of one call
        self.buf_bytes = LIB.kb_p2p_buffer_bytes(self.payload_bytes, self.world)
        self.timeout_ns = int(timeout_s * 1e9)
        self.epoch = 0
        self._ws = None
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
        # 1, 2, ..., 0xFFFFFFFE, 1, ...: never 0 (flags start zeroed), and an even
        # period, so the slot (epoch & 1) still alternates across the wrap
        self.epoch = self.epoch % 0xFFFFFFFE + 1
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

    # ---- fused sharded reductions: partial pass + exchange in one launch
    def _workspace(self, nbytes: int) -> torch.Tensor:
        """A zeroed workspace reused by every fused call (they run in stream
        order; each leaves its arrival counter at zero)."""
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.zeros(max(int(nbytes), 1 << 16), dtype=torch.uint8, device=self.device)
        return self._ws

    def _peer_args(self) -> tuple:
        return (self.bufs.data_ptr(), self.rank, self.world, self.buf_bytes, self._next(), self.timeout_ns)

    def mse_loss(self, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """out = mean over every rank's elements of (a - b)^2 (this rank: its
        shard a, b), one launch (kb_mse_sharded_f32)."""
        ws = self._workspace(LIB.kb_sharded_workspace_size())
        check("kb_mse_sharded_f32", LIB.kb_mse_sharded_f32(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(),
                                                            ws.data_ptr(), ws.numel(), *self._peer_args(),
                                                            self._stream(a)))
        return out

    def sumsq(self, x: torch.Tensor, total: torch.Tensor) -> torch.Tensor:
        """total (fp64, one element) = sum over every rank's shard of x^2, one
        launch (kb_sumsq_sharded_f64)."""
        ws = self._workspace(LIB.kb_sharded_workspace_size())
        check("kb_sumsq_sharded_f64", LIB.kb_sumsq_sharded_f64(x.data_ptr(), total.data_ptr(), x.numel(),
                                                                ws.data_ptr(), ws.numel(), *self._peer_args(),
                                                                self._stream(x)))
        return total

    def batch_norm_stats(self, x: torch.Tensor, stats: torch.Tensor) -> torch.Tensor:
        """stats (fp64, 2C + 1) = global per-channel sums, sums of squares and
        elements per channel over every rank's batch shard, one launch
        (kb_batchnorm_stats_sharded_f64)."""
        N, Cc = x.shape[0], x.shape[1]
        HW = math.prod(x.shape[2:])
        ws = self._workspace(LIB.kb_batchnorm_sharded_workspace_size(N, Cc, HW))
        check("kb_batchnorm_stats_sharded_f64",
              LIB.kb_batchnorm_stats_sharded_f64(x.data_ptr(), stats.data_ptr(), N, Cc, HW, ws.data_ptr(),
                                                 ws.numel(), *self._peer_args(), self._stream(x)))
        return stats

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
