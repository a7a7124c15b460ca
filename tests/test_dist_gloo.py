"""CPU, world sizes 2, 3 and 7 (gloo): the sharded ops of kbb200.dist compose their
per-shard partials and one collective into the same answer as the oracle on
the whole (unsharded) input.  The per-shard kernels are the CPU stand-ins of
tests/cpu_kernels.py; the GPU versions are the C-ABI kernels."""
from __future__ import annotations

import datetime
import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, q):
    try:
        for p in (str(REPO), str(REPO / "kernelbench-hip_b200")):
            if p not in sys.path:
                sys.path.insert(0, p)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch.distributed as tdist

        tdist.init_process_group("gloo", rank=rank, world_size=world,
                                 timeout=datetime.timedelta(seconds=20))
        from kbb200 import dist
        from oracle import ops as O
        from tests import cpu_kernels as CK

        g = torch.Generator().manual_seed(123)
        if case == "mse":
            a, b = torch.randn(10001, generator=g), torch.randn(10001, generator=g)
            # no total_n: the shards' element counts travel with the partial sums
            got = dist.mse_loss(dist.shard(a, rank, world), dist.shard(b, rank, world), kernels=CK)
            want = O.mse_loss(a.numpy(), b.numpy())
            res = (float(got), float(want))
        elif case == "frobenius":
            x = torch.randn(7, 33, 10, generator=g)
            xs = dist.shard(x, rank, world)
            got = dist.frobenius_normalize(xs, kernels=CK)
            lo, hi = dist.shard_range(7, rank, world)
            want = O.frobenius_normalize(x.numpy())[lo:hi]
            res = (got.numpy(), want)
        elif case == "batchnorm":
            x = torch.randn(6, 5, 4, 3, generator=g) * 2 + 1
            w, b = 1 + 0.1 * torch.randn(5, generator=g), 0.1 * torch.randn(5, generator=g)
            rm, rv = torch.zeros(5), torch.ones(5)
            xs = dist.shard(x, rank, world)
            got = dist.batch_norm_train(xs, w, b, 1e-5, 0.1, rm, rv, kernels=CK)
            lo, hi = dist.shard_range(6, rank, world)
            want = O.batch_norm_train(x.numpy(), w.numpy(), b.numpy())[lo:hi]
            erm, erv = O.batch_norm_running_update(x.numpy(), np.zeros(5), np.ones(5))
            res = (got.numpy(), want, rm.numpy(), erm, rv.numpy(), erv)
        elif case == "splitk":
            A, B = torch.randn(8, 1000, generator=g), torch.randn(1000, 6, generator=g)
            got = dist.matmul_splitk(dist.shard(A, rank, world, dim=1), dist.shard(B, rank, world, dim=0),
                                     kernels=CK)
            res = (got.numpy(), O.matmul(A.numpy(), B.numpy()))
        elif case == "crossentropy":
            x = torch.randn(11, 30, generator=g) * 2
            t = torch.randint(0, 30, (11,), generator=g)
            t[[2, 9]] = -100                                   # ignored rows on both shards
            got = dist.cross_entropy(dist.shard(x, rank, world), dist.shard(t, rank, world), kernels=CK)
            res = (float(got), float(O.cross_entropy(x.numpy(), t.numpy())))
        elif case == "count":
            res = (dist.global_count(10 + rank, "cpu"), 10 * world + sum(range(world)))
        elif case == "rank_fails":
            if rank == 1:
                raise RuntimeError("injected failure on rank 1")
            t = torch.ones(1)
            tdist.all_reduce(t)  # peer never joins -> gloo timeout error
            res = ("no error",)
        tdist.destroy_process_group()
        q.put((rank, "ok", res))
    except Exception as e:  # report to the parent instead of hanging
        q.put((rank, "err", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-400:]}"))


def _run(case, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, status, res = q.get(timeout=timeout)
            out[rank] = (status, res)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return out


# world 3: every case has shards of unequal sizes (10001 elements, 7 / 6 / 11
# rows, K = 1000); world 7 gives BatchNorm's 6 images an empty shard, whose
# rank must still update its running statistics like the others
@pytest.mark.parametrize("case,world", [(c, w) for w in (2, 3) for c in
                                        ("mse", "frobenius", "batchnorm", "splitk", "crossentropy", "count")] +
                         [("batchnorm", 7)])
def test_sharded_composition_matches_oracle(case, world):
    out = _run(case, world=world)
    assert sorted(out) == list(range(world))
    for rank, (status, res) in out.items():
        assert status == "ok", res
        if case in ("mse", "crossentropy"):
            np.testing.assert_allclose(res[0], res[1], rtol=1e-6)
        elif case == "batchnorm":
            np.testing.assert_allclose(res[0], res[1], rtol=1e-5, atol=1e-5)
            np.testing.assert_allclose(res[2], res[3], rtol=1e-5, atol=1e-6)
            np.testing.assert_allclose(res[4], res[5], rtol=1e-5, atol=1e-6)
        elif case == "count":
            assert res[0] == res[1]
        else:
            np.testing.assert_allclose(res[0], res[1], rtol=1e-5, atol=1e-6)


def test_failed_rank_surfaces_as_error_not_hang():
    """A rank that dies before a collective must end its peer's collective
    with an error within the process-group timeout."""
    out = _run("rank_fails", timeout=120)
    assert out[1][0] == "err" and "injected failure" in out[1][1]
    assert out[0][0] == "err", out[0]


def test_shard_range_partitions_exactly():
    from kbb200.dist import shard_range

    for n in (0, 1, 7, 64, 4097):
        for w in (1, 2, 3, 8):
            spans = [shard_range(n, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(w - 1))
            sizes = [h - l for l, h in spans]
            assert max(sizes) - min(sizes) <= 1


def test_peer_path_routing():
    """The peer all-reduce serves every payload that fits the communicator's
    slot, on any world size; without a PeerComm it is never used."""
    from types import SimpleNamespace

    from kbb200.dist import peer_path

    two, four, eight = (SimpleNamespace(world=w, payload_bytes=1 << 20) for w in (2, 4, 8))
    assert peer_path(two, 8) and peer_path(two, 256 * 1024)
    assert peer_path(four, 16) and peer_path(eight, 2056) and peer_path(eight, 256 * 1024)
    assert peer_path(eight, 1 << 20) and not peer_path(eight, (1 << 20) + 1)
    assert not peer_path(None, 8)
    # an exchange larger than the communicator's slot goes to NCCL, on any world size
    small = SimpleNamespace(world=2, payload_bytes=4096)
    assert peer_path(small, 4096) and not peer_path(small, 4097)


def test_fused_routing():
    """The fused one-launch sharded reductions serve exchanges up to
    FUSED_MAX_BYTES on every world size, only with a PeerComm that has them
    enabled and whose slot is large enough."""
    from types import SimpleNamespace

    from kbb200.dist import FUSED_MAX_BYTES, _fused

    c8 = SimpleNamespace(world=8, payload_bytes=1 << 20, fused=True)
    assert _fused(c8, 16) and _fused(c8, 8 * 257) and _fused(c8, FUSED_MAX_BYTES)
    assert not _fused(c8, FUSED_MAX_BYTES + 1)
    assert not _fused(SimpleNamespace(world=2, payload_bytes=1 << 20, fused=False), 16)
    assert not _fused(SimpleNamespace(world=2, payload_bytes=1024, fused=True), 2056)
    assert not _fused(None, 16)


def test_peer_epoch_wrap_keeps_slots_alternating():
    """PeerComm's epoch never takes 0 (the flags start zeroed) and keeps an
    even period, so the slot (epoch & 1) of two consecutive calls differs,
    across the 32-bit wrap too."""
    from kbb200.p2p import PeerComm

    comm = object.__new__(PeerComm)  # the counter alone: no process group, no buffers
    comm.epoch = 0xFFFFFFFE - 3
    seen = [comm._next() for _ in range(8)]
    assert 0 not in seen and max(seen) <= 0xFFFFFFFE
    assert all((a ^ b) & 1 for a, b in zip(seen, seen[1:])), seen
    assert 1 in seen  # it wrapped
