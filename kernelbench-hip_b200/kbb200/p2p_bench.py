"""Per-call cost of the cross-GPU step of the sharded ops: the library's
peer-memory all-reduce (kbb200.p2p.PeerComm) against NCCL's all_reduce, at
the payloads the sharded ops exchange, plus the fused split-K reduction
against a local split reduction followed by NCCL.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 \
        --master-addr 127.0.0.1 --master-port 29531 \
        -m kbb200.p2p_bench [--iters 200]

Device time per call with CUDA events on the launching stream over `iters`
back-to-back calls after warm-up, max over ranks; rank 0 prints one JSON
line.  NVLS is switched off for NCCL (plain rings over NVLink).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as tdist


def _time(fn, iters: int, device) -> float:
    for _ in range(10):
        fn()
    torch.cuda.synchronize(device)
    tdist.barrier()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(iters):
        fn()
    s1.record()
    torch.cuda.synchronize(device)
    t = torch.tensor([s0.elapsed_time(s1) * 1e3 / iters], dtype=torch.float64, device=device)
    tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
    return round(t.item(), 2)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=200)
    a = ap.parse_args()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    tdist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    from . import ops
    from .p2p import PeerComm

    comm = PeerComm(payload_bytes=1 << 20, timeout_s=10.0, device=dev)
    res = {"world": tdist.get_world_size(), "unit": "us per call", "iters": a.iters}
    try:
        for name, n, dtype in [("frobenius 8 B", 1, torch.float64),
                               ("mse / cross-entropy 16 B", 2, torch.float64),
                               ("batchnorm C=128 2 KiB", 257, torch.float64),
                               ("split-K C 256x256 256 KiB", 65536, torch.float32)]:
            t = torch.randn(n, dtype=dtype, device=dev)
            res[name] = {"p2p": _time(lambda: comm.all_reduce_(t), a.iters, dev),
                         "nccl": _time(lambda: tdist.all_reduce(t), a.iters, dev)}
        # split-K: this rank's K-split partial tiles -> full C on every rank
        g = torch.Generator(device=dev).manual_seed(0)
        A = torch.randn(256, 1 << 21, device=dev, generator=g)
        B = torch.randn(1 << 21, 256, device=dev, generator=g)
        parts, splits = ops.matmul_splitk_partials(A, B)
        c = torch.empty(256, 256, device=dev)
        fused = lambda: comm.splitk_all_reduce(parts, splits, c)

        def unfused():
            torch.sum(parts, dim=0, out=c)  # stands in for the local split reduction
            tdist.all_reduce(c)

        res[f"split-K fold of {splits} splits + all-reduce"] = {
            "p2p fused": _time(fused, a.iters, dev), "torch sum + nccl": _time(unfused, a.iters, dev)}
        comm.check()
    finally:
        comm.close()
    if tdist.get_rank() == 0:
        print(json.dumps(res))
    tdist.barrier()
    tdist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
