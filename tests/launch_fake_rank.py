"""A fake bench rank for the launcher's CPU tests (gloo, no GPU).

    torchrun --nproc-per-node N tests/launch_fake_rank.py PID_DIR MODE MS

Every rank records its pid in PID_DIR; MODE "hang" makes rank 1 sleep
forever after the rendezvous (rank 0 then waits at a barrier), "fail" makes
rank 0 exit 3, anything else prints one bench-style result line from rank 0
with ms_per_step = MS / world.
"""
import json
import os
import sys
import time
from pathlib import Path

import torch.distributed as dist

pid_dir, mode, ms = Path(sys.argv[1]), sys.argv[2], float(sys.argv[3])
if "RANK" in os.environ:
    dist.init_process_group("gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
else:
    rank, world = 0, 1
(pid_dir / f"rank{rank}.pid").write_text(str(os.getpid()))
if mode == "hang" and rank == 1:
    time.sleep(3600)
if mode == "fail" and rank == 0:
    sys.exit(3)
if world > 1:
    dist.barrier()
if rank == 0:
    print(json.dumps({"value": world * 1.0, "unit": "x", "ms_per_step": ms / world, "steps": 1}), flush=True)
if world > 1:
    dist.destroy_process_group()
