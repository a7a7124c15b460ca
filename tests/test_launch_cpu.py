"""CPU: the multi-GPU sweep launcher (kbb200.launch) isolates every cell in
its own process group with a wall-clock limit, records an honest -1 verdict
for a hung, failed or silent cell, resumes from recorded cells, and derives
the parallel efficiency from the 1-GPU cell.  The cells here are fake ranks
on gloo (tests/launch_fake_rank.py), launched by torch.distributed.run."""
from __future__ import annotations

import json
import os
import sys
import time
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
FAKE = REPO / "tests" / "launch_fake_rank.py"


def _alive(pid: int) -> bool:
    try:
        state = Path(f"/proc/{pid}/status").read_text()
    except FileNotFoundError:
        return False
    return "\nState:\tZ" not in state  # a zombie has already exited


def _fake_command(pid_root: Path, mode_of, ms_of):
    from kbb200.launch import torchrun_prefix

    def command(kind, op, ngpu, out_file):
        d = pid_root / f"{op}.{ngpu}"
        d.mkdir(parents=True, exist_ok=True)
        return torchrun_prefix(ngpu) + [str(FAKE), str(d), mode_of(op), str(ms_of(op))]

    return command


def test_hung_rank_is_killed_with_its_group(tmp_path):
    """Rank 1 never reaches the barrier: at the wall limit the launcher
    SIGKILLs torchrun and both ranks and records milestone -1."""
    from kbb200.launch import sweep

    out = tmp_path / "r.json"
    cmd = _fake_command(tmp_path / "pids", lambda op: "hang", lambda op: 10.0)
    t0 = time.monotonic()
    res = sweep("bench", ["hang_op"], [2], out, timeout_s=25.0, steps=1, warmup=1, command=cmd)
    assert time.monotonic() - t0 < 90
    r = res["hang_op@2gpu"]
    assert r["milestone"] == -1 and "killed at 25s" in r["why"]
    pids = [int(p.read_text()) for p in (tmp_path / "pids" / "hang_op.2").glob("rank*.pid")]
    assert len(pids) == 2, "both fake ranks started"
    deadline = time.monotonic() + 10
    while any(_alive(p) for p in pids) and time.monotonic() < deadline:
        time.sleep(0.2)
    assert not any(_alive(p) for p in pids), "a rank survived the group kill"
    assert json.loads(out.read_text())["hang_op@2gpu"]["milestone"] == -1


def test_failed_and_ok_cells_resume_and_efficiency(tmp_path):
    """A cell that exits non-zero gets -1; good cells record value and
    ms_per_step; a rerun skips recorded cells; parallel_eff = T1/(N TN)."""
    from kbb200.launch import markdown, sweep

    out = tmp_path / "r.json"
    calls = tmp_path / "calls"
    calls.mkdir()
    base = _fake_command(tmp_path / "pids", lambda op: "fail" if op == "bad" else "ok",
                         lambda op: 8.0)

    def counted(kind, op, ngpu, out_file):
        (calls / f"{op}.{ngpu}.{time.monotonic_ns()}").write_text("")
        return base(kind, op, ngpu, out_file)

    res = sweep("bench", ["good", "bad"], [1, 2], out, timeout_s=120.0, steps=1, warmup=1, command=counted)
    assert res["bad@1gpu"]["milestone"] == -1 and "exited 3" in res["bad@1gpu"]["why"]
    assert res["good@1gpu"]["ms_per_step"] == 8.0 and res["good@2gpu"]["ms_per_step"] == 4.0
    assert res["good@2gpu"]["parallel_eff"] == pytest.approx(1.0)
    n_calls = len(list(calls.iterdir()))
    assert n_calls == 4
    again = sweep("bench", ["good", "bad"], [1, 2], out, timeout_s=120.0, steps=1, warmup=1, command=counted)
    assert len(list(calls.iterdir())) == n_calls, "recorded cells ran again"
    assert again == res
    md = markdown(again)
    assert "good@2gpu" in md and "| -1" in md


def test_cell_commands_use_torchrun_beyond_one_gpu(tmp_path):
    from kbb200.launch import cell_command

    one = cell_command("bench", "layer_norm", 1, 20, 5, tmp_path / "o.json")
    eight = cell_command("bench", "layer_norm", 8, 20, 5, tmp_path / "o.json")
    assert one[0] == sys.executable and "torch.distributed.run" not in one
    assert "torch.distributed.run" in eight and eight[eight.index("--nproc-per-node") + 1] == "8"
    assert "--master-addr" in eight and eight[eight.index("--master-addr") + 1] == "127.0.0.1"
    ev = cell_command("eval", "40_LayerNorm", 2, 20, 5, tmp_path / "o.json")
    assert str(tmp_path / "o.json") in ev and ev[-4] == "--problem"
    ref = cell_command("reference", "layer_norm", 1, 3, 1, tmp_path / "o.json")
    assert "--impl" in ref and ref[ref.index("--impl") + 1] == "reference"


def test_family_cell_efficiency_per_op():
    """A family cell (all ops in one bench step) gets the step's and every
    op's parallel efficiency against the 1-GPU cell."""
    from kbb200.launch import add_efficiency

    res = {
        "northstar@1gpu": {"kind": "bench", "op": "northstar", "ngpu": 1, "milestone": 1, "ms_per_step": 20.0,
                           "per_op": {"matmul": {"ms": 5.0}, "mse_loss": {"ms": 0.32}}},
        "northstar@8gpu": {"kind": "bench", "op": "northstar", "ngpu": 8, "milestone": 1, "ms_per_step": 2.7,
                           "per_op": {"matmul": {"ms": 0.7}, "mse_loss": {"ms": 0.05}}},
    }
    add_efficiency(res)
    r = res["northstar@8gpu"]
    assert r["parallel_eff"] == pytest.approx(20.0 / (8 * 2.7), abs=1e-4)
    assert r["per_op_parallel_eff"]["matmul"] == pytest.approx(5.0 / 5.6, abs=1e-4)
    assert r["per_op_parallel_eff"]["mse_loss"] == pytest.approx(0.8, abs=1e-4)


def test_eval_cells_read_the_verdict_file(tmp_path):
    """Eval cells take their record from the verdict file the eval writes; a
    cell whose eval exits non-zero keeps the verdict's reason and gets -1."""
    from kbb200.launch import sweep

    def command(kind, op, ngpu, out_file):
        ms = -1 if op == "bad" else 1
        body = (f"import json, sys; json.dump({{'problem': {op!r}, 'milestone': {ms}, 'why': 'parity failed' "
                f"if {ms} < 0 else None, 'cand_time': {{'median_ms': 0.5}}}}, open({str(out_file)!r}, 'w')); "
                f"sys.exit(0 if {ms} > 0 else 1)")
        return [sys.executable, "-c", body]

    res = sweep("eval", ["good", "bad"], [1], tmp_path / "e.json", timeout_s=60.0, steps=1, warmup=1,
                command=command)
    assert res["good@1gpu"]["milestone"] == 1 and res["good@1gpu"]["cand_time"]["median_ms"] == 0.5
    assert res["bad@1gpu"]["milestone"] == -1 and res["bad@1gpu"]["why"] == "parity failed"
