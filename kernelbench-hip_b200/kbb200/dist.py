"""Multi-GPU sharding of the operator library (one process per GPU).

Ops whose units are independent (elementwise, row ops, dim-1 reductions,
max-pool, GEMM rows, GEMV rows) shard by rows or batch items and need no
collective: each rank runs the single-GPU kernel on its shard.  Four ops have a
real exchange step, and each takes exactly one collective between a local
partial kernel and a local finishing kernel (the split C-ABI entry pairs):

    op                 local partial            collective            finish
    mse_loss           sum (a-b)^2, count       all_reduce 16 B       divide by total count
    frobenius          sum x^2      (fp64)      all_reduce 8 B        x / sqrt(total)
    batch_norm_train   per-channel sum, sum^2,  all_reduce 16*C+8 B   normalise + affine
                       count
    cross_entropy      sum of losses, count     all_reduce 16 B       divide
    matmul_splitk      partial C over K slice   all_reduce M*N*4 B    (result replicated)

The collective is either torch.distributed's all_reduce (NCCL over NVLink on
B200s; gloo on CPU) or, given `comm=PeerComm(...)` (kbb200.p2p), the
library's own all-reduce kernel over peer memory; for split-K that kernel
also performs the rank's own K-split reduction, so local finish and
cross-GPU sum are one launch.  The peer kernel pushes each rank's payload to
every peer; it serves every exchange that fits the communicator's slot
(measured faster than or equal to NCCL from 8 B to 256 KiB on 2 and 8
ranks), and NCCL takes larger ones (see peer_path).  The per-shard kernels are injectable
(`kernels=`) so the composition can be tested with CPU implementations on a
gloo process group; by default they are the CUDA kernels of kbb200.ops.
"""
from __future__ import annotations


import torch
import torch.distributed as tdist


def _default_kernels():
    from . import ops

    return ops


def _world(group=None) -> tuple[int, int]:
    if not tdist.is_available() or not tdist.is_initialized():
        return 0, 1
    return tdist.get_rank(group), tdist.get_world_size(group)


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of rank's contiguous share of n units (first n % world ranks
    take one extra unit)."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard(t: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    lo, hi = shard_range(t.shape[dim], rank, world)
    return t.narrow(dim, lo, hi - lo)


# Measured on B200s (µs per call, peer kernel vs NCCL all_reduce, NVLS off,
# bench.py --exchange-sweep), after the peer kernel raised its flags with one
# fence per lane and parallel relaxed stores: 2 ranks 12.7 / 10.7 / 12.7 /
# 16.8 vs 17.3 / 17.3 / 19.1 / 40.9 for 8 B / 16 B / 2 KiB / 256 KiB; 8 ranks
# 14.1 / 14.2 / 17.2 / 27.6 vs 20.3 / 20.4 / 26.3 / 28.1, and the split-K
# fold + all-reduce in one kernel 32.9 against 59.3 for a local reduction +
# NCCL.  (With one release store per peer, one after another, the kernel
# had lost to NCCL from 2 KiB up on 4 ranks: 21.5 vs 17.7 and 30.7 vs 19.5.)
# So the peer kernel serves every payload that fits its slot.
# The fused sharded kernels (one CTA pushes this rank's fold to every peer at
# the end of the partial pass) serve exchanges up to this size on any world
# size: BatchNorm's 16 C + 8 bytes for C <= 1024.  The push is a few KiB per
# peer from one CTA, so it does not grow into the standalone kernel's
# per-rank traffic problem; larger exchanges keep the three-step form.
FUSED_MAX_BYTES = 16 * 1024 + 8


def peer_path(comm, nbytes: int) -> bool:
    """Whether an exchange of nbytes per rank goes through the PeerComm: never
    beyond the communicator's slot (comm.payload_bytes), which NCCL handles
    instead.  Every rank passes the same nbytes and world size, so all ranks
    take the same path and the collective order stays identical."""
    return comm is not None and nbytes <= comm.payload_bytes


def _fused(comm, nbytes: int) -> bool:
    """Whether the sharded reduction runs as one fused launch (partial pass
    and exchange in the same kernel, kbb200.p2p.PeerComm): on the peer path,
    whose one-CTA exchange carries at most FUSED_MAX_BYTES per rank."""
    return (comm is not None and getattr(comm, "fused", False) and nbytes <= FUSED_MAX_BYTES
            and nbytes <= comm.payload_bytes)


def _all_reduce_sum(t: torch.Tensor, group=None, comm=None) -> torch.Tensor:
    if peer_path(comm, t.numel() * t.element_size()):
        return comm.all_reduce_(t)
    if _world(group)[1] > 1:
        tdist.all_reduce(t, op=tdist.ReduceOp.SUM, group=group)
    return t


def global_count(local: int, device, group=None) -> int:
    """Sum of a per-rank element count (one small all_reduce)."""
    if _world(group)[1] == 1:
        return int(local)
    c = torch.tensor([float(local)], dtype=torch.float64, device=device)
    _all_reduce_sum(c, group)
    return int(c.item())


def mse_loss(a: torch.Tensor, b: torch.Tensor, total_n: int | None = None, out=None, group=None,
             kernels=None, comm=None):
    """mean((a - b)^2) over the union of all ranks' shards (replicated 0-d
    result).  The element count travels with the partial sum, so shards may
    differ in size (or be empty); total_n overrides it."""
    k = kernels or _default_kernels()
    if total_n is None and _fused(comm, 16):
        y = out if out is not None else torch.empty((), device=a.device, dtype=torch.float32)
        return comm.mse_loss(a, b, y)
    part = k.mse_partial(a, b)
    _all_reduce_sum(part, group, comm)
    return k.mse_finalize(part, total_n if total_n is not None else 0, out=out)


def frobenius_normalize(x: torch.Tensor, out=None, group=None, kernels=None, comm=None):
    """x_shard / ||x||_F where the norm spans all ranks' shards."""
    k = kernels or _default_kernels()
    if _fused(comm, 8):
        part = comm.sumsq(x, torch.empty((), device=x.device, dtype=torch.float64))
    else:
        part = k.sumsq_partial(x)
        _all_reduce_sum(part, group, comm)
    return k.scale_by_inv_norm(x, part, out=out)


def batch_norm_train(x: torch.Tensor, weight=None, bias=None, eps: float = 1e-5,
                     momentum: float = 0.1, running_mean=None, running_var=None, out=None,
                     total_count: int | None = None, group=None, kernels=None, comm=None):
    """Training-mode BatchNorm with statistics over the global batch (every
    rank holds a slice of the batch dim): SyncBatchNorm semantics, equal to
    BatchNorm on the concatenated batch.  The per-channel element count is
    summed with the statistics, so slices may differ in size; a rank with an
    empty slice still updates its running statistics.  total_count
    overrides the count."""
    k = kernels or _default_kernels()
    nbytes = 8 * (2 * x.shape[1] + 1)
    if _fused(comm, nbytes) and x.shape[1] > 0:
        stats = comm.batch_norm_stats(x, torch.empty(2 * x.shape[1] + 1, device=x.device, dtype=torch.float64))
    else:
        stats = k.batch_norm_stats(x)
        _all_reduce_sum(stats, group, comm)
    count = total_count if total_count is not None else 0
    return k.batch_norm_apply(x, stats, count, weight, bias, eps, momentum, running_mean,
                              running_var, out=out)


def matmul_splitk(a: torch.Tensor, b: torch.Tensor, out=None, group=None, kernels=None, comm=None):
    """C = A @ B with K sharded: rank r holds A[:, K_r] and B[K_r, :].  Each
    rank computes its partial C (split-K across its own SMs as well), then one
    all_reduce sums the partials; every rank ends with the full C.  With a
    PeerComm whose slot holds C, the rank's K-split tiles go straight into
    the peer all-reduce kernel, which sums them (split order) and then
    across ranks (rank order)."""
    k = kernels or _default_kernels()
    if peer_path(comm, a.shape[0] * b.shape[1] * 4):
        parts, splits = k.matmul_splitk_partials(a, b)
        c = out if out is not None else torch.empty(a.shape[0], b.shape[1], device=a.device,
                                                    dtype=torch.float32)
        return comm.splitk_all_reduce(parts, splits, c)
    c = k.matmul_splitk(a, b, out=out)
    _all_reduce_sum(c, group)
    return c


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100, out=None,
                  group=None, kernels=None, comm=None):
    """Mean cross-entropy over the union of all ranks' row shards (replicated
    0-d result): per-shard (sum of losses, rows not ignored), one all_reduce
    of those 16 bytes, then the division."""
    k = kernels or _default_kernels()
    part = k.cross_entropy_partial(logits, targets, ignore_index)
    _all_reduce_sum(part, group, comm)
    return k.cross_entropy_finalize(part, out=out)
