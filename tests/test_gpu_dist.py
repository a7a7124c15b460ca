"""GPU, 2 / 4 / 8 ranks over NCCL: the sharded ops of kbb200.dist with the CUDA
per-shard kernels reproduce the single-device answer on the global input.

Each rank builds the same seeded global tensors on the CPU, keeps its shard
on its own GPU, runs the sharded op (local partial kernel, one all_reduce,
local finishing kernel) and compares with the oracle on the whole input —
once with NCCL's all_reduce and once with the library's own all-reduce
kernel over peer memory (kbb200.p2p.PeerComm, CUDA IPC).
Each world size is skipped unless the process sees that many GPUs.  NVLS is switched off (plain
NCCL rings over NVLink).
"""
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

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        for p in (str(REPO), str(REPO / "kernelbench-hip_b200")):
            if p not in sys.path:
                sys.path.insert(0, p)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        import torch.distributed as tdist

        tdist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                 timeout=datetime.timedelta(seconds=60))
        from kbb200 import dist
        from oracle import ops as O

        res = {}
        g = torch.Generator().manual_seed(7)
        a, b = torch.randn(1 << 20, generator=g), torch.randn(1 << 20, generator=g)
        got = dist.mse_loss(dist.shard(a, rank, world).to(dev), dist.shard(b, rank, world).to(dev),
                            total_n=a.numel())
        res["mse"] = (float(got), float(O.mse_loss(a.numpy(), b.numpy())), 1e-3)

        x = torch.randn(8, 64, 130, generator=g)
        got = dist.frobenius_normalize(dist.shard(x, rank, world).to(dev)).cpu().numpy()
        lo, hi = dist.shard_range(8, rank, world)
        res["frobenius"] = (got, O.frobenius_normalize(x.numpy())[lo:hi], 1e-5)
        x0, lo0, hi0 = x, lo, hi

        x = torch.randn(6, 32, 20, 24, generator=g) * 2 + 1
        w, bb = 1 + 0.02 * torch.randn(32, generator=g), 0.02 * torch.randn(32, generator=g)
        xs_bn = dist.shard(x, rank, world).to(dev)
        rm, rv = torch.zeros(32, device=dev), torch.ones(32, device=dev)
        got = dist.batch_norm_train(xs_bn, w.to(dev), bb.to(dev), 1e-5, 0.1, rm, rv).cpu().numpy()
        lo, hi = dist.shard_range(6, rank, world)
        want_bn = O.batch_norm_train(x.numpy(), w.numpy(), bb.numpy())[lo:hi]
        res["batchnorm"] = (got, want_bn, 1e-5)
        erm, erv = O.batch_norm_running_update(x.numpy(), np.zeros(32), np.ones(32))
        res["batchnorm_running_mean"] = (rm.cpu().numpy(), erm, 1e-5)   # empty shards too
        res["batchnorm_running_var"] = (rv.cpu().numpy(), erv, 1e-5)
        x_bn, w_bn, b_bn = x, w, bb

        A, B = torch.randn(256, 65536, generator=g), torch.randn(65536, 256, generator=g)
        As = dist.shard(A, rank, world, dim=1).contiguous().to(dev)
        Bs = dist.shard(B, rank, world, dim=0).contiguous().to(dev)
        got = dist.matmul_splitk(As, Bs).cpu().numpy()
        want_c = O.matmul(A.numpy(), B.numpy())
        res["splitk"] = (got, want_c, 1e-3)

        lg = torch.randn(1000, 500, generator=g) * 2
        tg = torch.randint(0, 500, (1000,), generator=g)
        tg[[3, 700]] = -100
        lgs, tgs = dist.shard(lg, rank, world).to(dev), dist.shard(tg, rank, world).to(dev)
        got = dist.cross_entropy(lgs, tgs)
        want_ce = float(O.cross_entropy(lg.numpy(), tg.numpy()))
        res["cross_entropy"] = (float(got), want_ce, 1e-5)

        # the same ops over the library's peer-memory all-reduce (CUDA IPC)
        from kbb200.p2p import PeerComm

        comm = PeerComm(payload_bytes=1 << 20, timeout_s=5.0)
        try:
            sa, sb = dist.shard(a, rank, world).to(dev), dist.shard(b, rank, world).to(dev)
            for rep in range(3):  # several epochs: both slots, reuse
                got = dist.mse_loss(sa, sb, total_n=a.numel(), comm=comm)
                res[f"p2p_mse{rep}"] = (float(got), float(O.mse_loss(a.numpy(), b.numpy())), 1e-3)
            got = dist.frobenius_normalize(dist.shard(x0, rank, world).to(dev), comm=comm).cpu().numpy()
            res["p2p_frobenius"] = (got, O.frobenius_normalize(x0.numpy())[lo0:hi0], 1e-5)
            got = dist.cross_entropy(lgs, tgs, comm=comm)
            res["p2p_cross_entropy"] = (float(got), want_ce, 1e-5)
            got = dist.batch_norm_train(xs_bn, w_bn.to(dev), b_bn.to(dev), comm=comm).cpu().numpy()
            res["p2p_batchnorm"] = (got, want_bn, 1e-5)
            c1 = dist.matmul_splitk(As, Bs, comm=comm)
            c2 = dist.matmul_splitk(As, Bs, comm=comm)
            res["p2p_splitk"] = (c1.cpu().numpy(), want_c, 1e-3)
            res["p2p_splitk_deterministic"] = (float(torch.equal(c1, c2)), 1.0, 0.0)
            # every rank holds the same bits (rank-ordered sum)
            gathered = [torch.empty_like(c1) for _ in range(world)]
            tdist.all_gather(gathered, c1)
            res["p2p_splitk_replicated"] = (float(all(torch.equal(gathered[0], t) for t in gathered)), 1.0, 0.0)
            comm.check()
        finally:
            comm.close()
        torch.cuda.synchronize()
        tdist.destroy_process_group()
        q.put((rank, "ok", res))
    except Exception as e:
        q.put((rank, "err", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-600:]}"))


# 4 and 8 ranks give uneven shards (BatchNorm's 6 images: 2/2/1/1, and two
# empty shards at 8) and exercise the peer all-reduce with more than one peer
@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_ops_on_several_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _run_workers(_worker, world)


# uneven batch splits of BatchNorm's 64 images (every rank non-empty)
BN_SPLITS = {2: [37, 27], 4: [23, 9, 17, 15], 8: [13, 5, 8, 8, 9, 7, 6, 8]}


def _bench_worker(rank, world, port, q):
    """The sharded ops at the benchmark shapes: every rank draws the same
    global input on its own GPU (seeded device generator), keeps its shard,
    runs the sharded op and compares with an fp64 evaluation of the global op
    on the device and with the single-GPU kernel on the whole input."""
    try:
        for p in (str(REPO), str(REPO / "kernelbench-hip_b200")):
            if p not in sys.path:
                sys.path.insert(0, p)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        import torch.distributed as tdist
        import torch.nn.functional as F

        tdist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                 timeout=datetime.timedelta(seconds=120))
        from kbb200 import dist, ops
        from kbb200.p2p import PeerComm

        comm = PeerComm(payload_bytes=1 << 20, timeout_s=10.0)
        res = {}

        def gen(seed):
            return torch.Generator(device=dev).manual_seed(seed)

        try:
            # MSE over two 2^28 vectors, contiguous slices
            n = 1 << 28
            a = torch.randn(n, device=dev, generator=gen(1))
            b = torch.randn(n, device=dev, generator=gen(2))
            want = float(((a.double() - b.double()) ** 2).mean())
            sa, sb = dist.shard(a, rank, world), dist.shard(b, rank, world)
            for label, c in (("nccl", None), ("p2p", comm)):
                got = float(dist.mse_loss(sa, sb, comm=c))
                res[f"mse_2^28_{label}"] = (got, want, 1e-3)
            res["mse_2^28_single_gpu"] = (float(ops.mse_loss(a, b)), want, 1e-3)
            del a, b, sa, sb

            # Frobenius normalisation of [256, 1024, 1024], batch shards
            x = torch.randn(256, 1024, 1024, device=dev, generator=gen(3))
            lo, hi = dist.shard_range(256, rank, world)
            norm = float(torch.linalg.vector_norm(x.double()))
            for label, c in (("nccl", None), ("p2p", comm)):
                y = dist.frobenius_normalize(x[lo:hi], comm=c)
                ref = (x[lo:hi].double() / norm).float()
                rel = float(((y - ref).abs() / (ref.abs() + 1e-12)).max())
                res[f"frobenius_max_rel_err_{label}"] = (rel, 0.0, 1e-5)
            del x, y, ref

            # BatchNorm [64, 128, 256, 256], uneven batch shards, running statistics
            x = torch.randn(64, 128, 256, 256, device=dev, generator=gen(4)) * 1.5 + 0.25
            w = 1 + 0.02 * torch.randn(128, device=dev, generator=gen(5))
            bb = 0.02 * torch.randn(128, device=dev, generator=gen(6))
            sizes = BN_SPLITS[world]
            lo = sum(sizes[:rank])
            hi = lo + sizes[rank]
            rm64, rv64 = torch.zeros(128, device=dev, dtype=torch.float64), torch.ones(128, device=dev,
                                                                                       dtype=torch.float64)
            ref = F.batch_norm(x.double(), rm64, rv64, w.double(), bb.double(),
                               training=True, momentum=0.1, eps=1e-5)[lo:hi].float()
            for label, c in (("nccl", None), ("p2p", comm)):
                rm, rv = torch.zeros(128, device=dev), torch.ones(128, device=dev)
                y = dist.batch_norm_train(x[lo:hi], w, bb, 1e-5, 0.1, rm, rv, comm=c)
                res[f"batchnorm_max_err_{label}"] = (float((y - ref).abs().max()), 0.0, 1e-5)
                res[f"batchnorm_running_mean_{label}"] = (rm.cpu().numpy(), rm64.float().cpu().numpy(), 1e-5)
                res[f"batchnorm_running_var_{label}"] = (rv.cpu().numpy(), rv64.float().cpu().numpy(), 1e-5)
            del x, y, ref

            # split-K 256 x 4,194,304 @ 4,194,304 x 256, K slices
            K = 4194304
            A = torch.randn(256, K, device=dev, generator=gen(7)) / K ** 0.5
            B = torch.randn(K, 256, device=dev, generator=gen(8)) / K ** 0.5
            want = torch.zeros(256, 256, device=dev, dtype=torch.float64)
            for k0 in range(0, K, 1 << 19):  # fp64 in chunks of K (bounded memory)
                want += A[:, k0:k0 + (1 << 19)].double() @ B[k0:k0 + (1 << 19)].double()
            lo, hi = dist.shard_range(K, rank, world)
            As, Bs = A[:, lo:hi].contiguous(), B[lo:hi]
            del A, B
            outs = {}
            for label, c in (("nccl", None), ("p2p", comm)):
                cmat = dist.matmul_splitk(As, Bs, comm=c)
                outs[label] = cmat
                err = float(((cmat.double() - want).abs() - 1e-3 * want.abs()).max())
                res[f"splitk_K4M_excess_err_{label}"] = (max(err, 0.0), 0.0, 1e-3)
            again = dist.matmul_splitk(As, Bs, comm=comm)
            res["splitk_K4M_p2p_deterministic"] = (float(torch.equal(again, outs["p2p"])), 1.0, 0.0)
            gathered = [torch.empty_like(again) for _ in range(world)]
            tdist.all_gather(gathered, again)
            res["splitk_K4M_replicated"] = (float(all(torch.equal(gathered[0], t) for t in gathered)), 1.0, 0.0)
            del As, Bs

            # row shards without an exchange: SGEMM rows of 8192^3, matvec rows
            A = torch.randn(8192, 8192, device=dev, generator=gen(9)) / 8192 ** 0.5
            B = torch.randn(8192, 8192, device=dev, generator=gen(10)) / 8192 ** 0.5
            lo, hi = dist.shard_range(8192, rank, world)
            whole = ops.matmul(A, B)
            res["sgemm_rows_equal_whole"] = (float(torch.equal(ops.matmul(A[lo:hi], B), whole[lo:hi])), 1.0, 0.0)
            del A, B, whole
            A = torch.randn(4096, 1 << 20, device=dev, generator=gen(11))
            v = torch.randn(1 << 20, device=dev, generator=gen(12))
            lo, hi = dist.shard_range(4096, rank, world)
            y = ops.gemv(A[lo:hi], v)
            # rows are independent with a fixed summation order: the shard's
            # rows equal the whole-input kernel's bit for bit (that kernel is
            # checked against torch at this shape by the parity tests); and
            # against fp64, within fp32 accumulation error of 2^20-term rows
            res["gemv_rows_equal_whole"] = (float(torch.equal(y, ops.gemv(A, v)[lo:hi])), 1.0, 0.0)
            ref = A[lo:hi].double() @ v.double()
            res["gemv_rows_fp64_excess"] = (float(((y.double() - ref).abs() - (1e-2 + 1e-3 * ref.abs())).clamp_min(0).max()),
                                            0.0, 0.0)
            del A, v
            comm.check()
        finally:
            comm.close()
        torch.cuda.synchronize()
        tdist.destroy_process_group()
        q.put((rank, "ok", res))
    except Exception as e:
        q.put((rank, "err", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-800:]}"))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_ops_at_benchmark_shapes(world):
    """MSE on 2^28 elements, Frobenius [256, 1024, 1024], BatchNorm
    [64, 128, 256, 256] split unevenly by batch, split-K with K = 4,194,304
    split by K, and the row-sharded SGEMM / matvec, each over NCCL and over
    the peer all-reduce, against the global op."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _run_workers(_bench_worker, world, timeout=600)


def _run_workers(target, world, timeout=300):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, status, res = q.get(timeout=timeout)
            out[rank] = (status, res)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, (status, res) in out.items():
        assert status == "ok", res
        for name, (got, want, tol) in res.items():
            np.testing.assert_allclose(got, want, rtol=tol, atol=tol, err_msg=f"rank {rank} {name}")


def test_strict_eval_on_two_gpus(tmp_path):
    """The strict eval sibling under torchrun: every rank checks parity and
    times the candidate on its own GPU; rank 0's verdict carries ngpu 2, the
    per-rank medians and their max."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import json
    import subprocess

    out = tmp_path / "v.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(REPO / "tests" / "eval_b200.py"),
           "--problem", "40_LayerNorm", "--small", "--trials", "5", "--no-cpu", "--out", str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    v = json.loads(out.read_text())
    assert v["ngpu"] == 2 and v["parity"]["parity"] and v["parity"]["all_ranks"]
    per = v["cand_time"]["per_rank_median_ms"]
    assert len(per) == 2 and v["cand_time"]["median_ms"] == max(per)
