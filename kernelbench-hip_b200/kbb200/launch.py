"""Multi-GPU sweep launcher: problems x {1, 2, 4, 8} GPUs, one isolated job per
cell — the B200 replacement of the reference's subprocess-per-candidate
driver (scripts/run_batch.py:24-47) and its crash-safe baseline sweep
(scripts/run_baselines.py:24-29, :62-63).

    python -m kbb200.launch --kind bench --ops northstar --gpus 1,2,4,8 --out sweep.json
    python -m kbb200.launch --kind bench --ops northstar --split-family --gpus 1,8 --out per_op.json
    python -m kbb200.launch --kind eval --ops 40_LayerNorm,23_Softmax --gpus 1 --out evals.json
    python -m kbb200.launch --kind reference --ops northstar --out cpu.json

Cell kinds (each cell is one command, run under `torch.distributed.run` with
one process per GPU when it has more than one GPU):
  bench      bench.py --workload <op or family> --gpus N: the global
             problem sharded over N ranks; the cell records the max-over-ranks
             step time, per-op times and roofline fractions, and the parallel
             efficiency T1 / (N * TN) against the 1-GPU cell (for a family
             cell also per op);
  eval       the strict eval (tests/eval_b200.py) of one problem: parity on
             every rank, the reference's timing protocol, milestones;
  reference  bench.py --impl reference --workload <op>: the torch-eager fp32
             CPU reference on the host cores (core count recorded).

Isolation, as the reference's driver does it: every cell runs in a new
session (its own process group) with a wall-clock limit; on expiry the
cell's whole process tree (torchrun, and every rank, which torchrun starts
in sessions of their own) is SIGKILLed and the cell gets an
honest -1 verdict (`"milestone": -1, "why": "killed at ..."`), as does a cell
that exits non-zero or prints no result.  Results are written after every
cell (to a temporary file, then renamed), keyed "<op>@<N>gpu"; a rerun skips
the cells already recorded (resume after a crash), unless --redo.
"""
from __future__ import annotations

import argparse
import json
import os
import signal
import socket
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]
BENCH = REPO / "bench.py"
EVAL = REPO / "tests" / "eval_b200.py"
DEFAULT_TIMEOUT_S = 900  # the reference's per-candidate wall (scripts/run_batch.py:22)


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def torchrun_prefix(ngpu: int) -> list[str]:
    """The launch prefix of an N-GPU job: one process per GPU, rendezvous on
    the loopback address; plain python for one GPU."""
    if ngpu <= 1:
        return [sys.executable]
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(ngpu),
            "--master-addr", "127.0.0.1", "--master-port", str(free_port())]


def cell_command(kind: str, op: str, ngpu: int, steps: int, warmup: int, out_file: Path) -> list[str]:
    if kind == "bench":
        return torchrun_prefix(ngpu) + [str(BENCH), "--gpus", str(ngpu), "--workload", op, "--steps", str(steps),
                                        "--warmup", str(warmup), "--no-e2e", "--no-cpu-baseline"]
    if kind == "reference":
        return [sys.executable, str(BENCH), "--impl", "reference", "--workload", op, "--steps", str(steps),
                "--warmup", "1"]
    if kind == "eval":
        return torchrun_prefix(ngpu) + [str(EVAL), "--problem", op, "--out", str(out_file)]
    raise ValueError(kind)


def kill_tree(pid: int) -> None:
    """SIGKILL a cell: its process group, and every descendant with its own
    process group — torchrun starts each rank in a new session, so killing
    the launcher's group alone would leave hung ranks (and the GPU memory
    they hold) behind.  The descendants are collected before anything is
    killed, so none is reparented out of reach."""
    import psutil

    try:
        kids = psutil.Process(pid).children(recursive=True)
    except psutil.NoSuchProcess:
        kids = []
    groups = {pid}
    for k in kids:
        try:
            groups.add(os.getpgid(k.pid))
        except ProcessLookupError:
            pass
    for g in groups:
        try:
            os.killpg(g, signal.SIGKILL)
        except (ProcessLookupError, PermissionError):
            pass
    for k in kids:
        try:
            k.kill()
        except psutil.NoSuchProcess:
            pass


def run_cell(cmd: list[str], timeout_s: float, log_path: Path | None = None,
             env: dict | None = None) -> dict:
    """Run one cell in its own session with a wall-clock limit.  Returns
    {"rc", "wall_s", "stdout", "killed"}; on expiry the cell's process tree
    (a torchrun launcher and all its ranks) is SIGKILLed (kill_tree)."""
    t0 = time.monotonic()
    log = open(log_path, "w") if log_path else subprocess.DEVNULL
    try:
        proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=log, text=True, start_new_session=True,
                                env=env, cwd=str(REPO))
        try:
            out, _ = proc.communicate(timeout=timeout_s)
            killed = False
        except subprocess.TimeoutExpired:
            kill_tree(proc.pid)
            try:
                out, _ = proc.communicate(timeout=30)
            except subprocess.TimeoutExpired:  # a descendant escaped and still holds the pipe
                out = ""
                proc.kill()
                proc.wait()
            killed = True
    finally:
        if log_path:
            log.close()
    return {"rc": proc.returncode, "wall_s": round(time.monotonic() - t0, 2), "stdout": out or "",
            "killed": killed}


def _last_json(text: str) -> dict | None:
    for line in reversed(text.strip().splitlines()):
        line = line.strip()
        if line.startswith("{"):
            try:
                return json.loads(line)
            except json.JSONDecodeError:
                continue
    return None


def verdict(kind: str, op: str, ngpu: int, run: dict, timeout_s: float, out_file: Path) -> dict:
    """The cell's record; -1 for a kill, a non-zero exit or a missing result."""
    base = {"op": op, "ngpu": ngpu, "kind": kind, "wall_s": run["wall_s"]}
    if run["killed"]:
        return {**base, "milestone": -1,
                "why": f"killed at {timeout_s:.0f}s wall (process tree SIGKILLed; hung rank suspected)"}
    if kind == "eval":
        v = json.loads(out_file.read_text()) if out_file.exists() else {}
        if run["rc"] != 0 or "milestone" not in v:
            return {**base, **v, "milestone": -1, "why": v.get("why", f"eval exited {run['rc']}")}
        return {**base, **{k: v[k] for k in v if k not in ("parity",)}}
    line = _last_json(run["stdout"])
    if run["rc"] != 0 or line is None or line.get("value") is None:
        return {**base, "milestone": -1, "why": f"exited {run['rc']} without a result line"}
    rec = {**base, "milestone": 1, "value": line["value"], "unit": line.get("unit"),
           "ms_per_step": line.get("ms_per_step"), "steps": line.get("steps")}
    if kind == "bench":
        rec["per_op"] = line.get("per_op")
        rec["clocks"] = line.get("clocks")
    else:
        rec["cores"] = (line.get("cpu_baseline") or {}).get("cores")
        rec["sample"] = (line.get("cpu_baseline") or {}).get("sample")
    return rec


def add_efficiency(results: dict) -> None:
    """parallel_eff = T1 / (N * TN) for every bench cell whose op (or family)
    has a 1-GPU cell, and per op inside a family cell (from its per_op
    times)."""
    for key, rec in results.items():
        if rec.get("kind") != "bench" or rec.get("milestone", -1) < 0:
            continue
        one = results.get(f"{rec['op']}@1gpu")
        if one and one.get("milestone", -1) >= 0 and rec.get("ms_per_step"):
            rec["parallel_eff"] = round(one["ms_per_step"] / (rec["ngpu"] * rec["ms_per_step"]), 4)
            per1, perN = one.get("per_op") or {}, rec.get("per_op") or {}
            if len(perN) > 1:
                rec["per_op_parallel_eff"] = {n: round(per1[n]["ms"] / (rec["ngpu"] * d["ms"]), 4)
                                              for n, d in perN.items() if n in per1 and d.get("ms")}


def save(path: Path, results: dict) -> None:
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_text(json.dumps(results, indent=1, default=str) + "\n")
    os.replace(tmp, path)


def markdown(results: dict) -> str:
    rows = ["| cell | verdict | ms/step | value | parallel eff | wall s |", "|---|---|---|---|---|---|"]
    for key, r in results.items():
        ok = "ok" if r.get("milestone", -1) >= 0 else f"-1 ({r.get('why', '')[:60]})"
        rows.append(f"| {key} | {ok} | {r.get('ms_per_step', '')} | {r.get('value', '')} | "
                    f"{r.get('parallel_eff', '')} | {r.get('wall_s', '')} |")
    # per-op efficiency of family cells, one column per GPU count
    fam = [(k, r) for k, r in results.items() if r.get("per_op_parallel_eff")]
    if fam:
        ops = list(fam[0][1]["per_op_parallel_eff"])
        rows += ["", "| op | " + " | ".join(k for k, _ in fam) + " |", "|---|" + "---|" * len(fam)]
        for o in ops:
            rows.append(f"| {o} | " + " | ".join(str(r["per_op_parallel_eff"].get(o, "")) for _, r in fam) + " |")
    return "\n".join(rows) + "\n"


def sweep(kind: str, ops: list[str], gpus: list[int], out: Path, timeout_s: float, steps: int, warmup: int,
          redo: bool = False, log_dir: Path | None = None, command=None) -> dict:
    """Run every (op, ngpu) cell not yet in `out`; returns all results.
    `command(kind, op, ngpu, out_file) -> argv` overrides the cell command."""
    results = json.loads(out.read_text()) if out.exists() and not redo else {}
    work = out.parent / (out.stem + "_cells")
    work.mkdir(parents=True, exist_ok=True)
    for ngpu in gpus:
        for op in ops:
            key = f"{op}@{ngpu}gpu"
            if key in results:
                continue  # resume: recorded by an earlier run
            out_file = work / f"{op}.{ngpu}gpu.json"
            if out_file.exists():
                out_file.unlink()
            cmd = (command(kind, op, ngpu, out_file) if command is not None
                   else cell_command(kind, op, ngpu, steps, warmup, out_file))
            log = (log_dir / f"{op}.{ngpu}gpu.log") if log_dir else None
            env = dict(os.environ)
            env.setdefault("NCCL_NVLS_ENABLE", "0")
            run = run_cell(cmd, timeout_s, log, env)
            results[key] = verdict(kind, op, ngpu, run, timeout_s, out_file)
            add_efficiency(results)
            save(out, results)
            r = results[key]
            print(f"{key}: " + (f"-1 {r['why']}" if r.get("milestone", -1) < 0 else
                                f"value {r.get('value')} ms/step {r.get('ms_per_step')} "
                                f"eff {r.get('parallel_eff', '-')}"), flush=True)
    return results


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--kind", choices=("bench", "eval", "reference"), default="bench")
    ap.add_argument("--ops", default="northstar",
                    help="comma-separated ops (bench/reference) or problems (eval), or a workload family")
    ap.add_argument("--gpus", default="1,2,4,8")
    ap.add_argument("--out", default="sweep.json")
    ap.add_argument("--md", default=None, help="also write a markdown table here")
    ap.add_argument("--timeout", type=float, default=DEFAULT_TIMEOUT_S, help="wall seconds per cell")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--redo", action="store_true", help="ignore recorded cells")
    ap.add_argument("--log-dir", default=None)
    ap.add_argument("--split-family", action="store_true",
                    help="one cell per op of a family (default: the family's ops share one bench step per cell)")
    a = ap.parse_args(argv)
    from .workloads import FAMILIES, WORKLOADS

    if a.ops in FAMILIES and (a.kind == "eval" or a.split_family):
        ops = FAMILIES[a.ops]
        if a.kind == "eval":
            ops = [WORKLOADS[o].problem for o in ops]
    else:
        ops = a.ops.split(",")  # a family name stays one cell: all its ops in one bench step
    gpus = [1] if a.kind == "reference" else [int(g) for g in a.gpus.split(",")]
    log_dir = Path(a.log_dir) if a.log_dir else None
    if log_dir:
        log_dir.mkdir(parents=True, exist_ok=True)
    out = Path(a.out)
    results = sweep(a.kind, ops, gpus, out, a.timeout, a.steps, a.warmup, a.redo, log_dir)
    if a.md:
        Path(a.md).write_text(markdown(results))
    return 0 if all(r.get("milestone", -1) >= 0 for r in results.values()) else 1


if __name__ == "__main__":
    sys.exit(main())
