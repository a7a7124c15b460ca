"""Strict evaluation of the B200 candidates — the reference's protected-eval
protocol with the library's own bars added (test infrastructure).

Per problem it reproduces harness/eval_protected.py — static anti-hack check
(:150-159), candidate build with restricted globals (:286-300), parity on
seeds 0-4 with R1 input hashes and the R2 recompute digest (:338-411),
event timing with warm-up 5, 100 trials, first discarded, L2 thrashed before
every trial and a median / stall flag (:94-123), milestones 1/2/3 (:242-253)
— and adds:
  - the per-op tolerance (1e-5 elementwise/norm, 1e-3 reductions/GEMMs,
    bit-exact argmax / max-pool) next to the reference's allclose(1e-2);
  - GB/s or TFLOP/s of the candidate and its fraction of the measured B200
    roofline (MEASURED_PEAKS.json);
  - the torch-eager fp32 CPU time on a bounded sample (grown until one call
    takes a quarter second), with the core count;
  - the L2 thrash sized from the device's L2 (2x), not a fixed 256 MB.
Verdicts keep the reference's JSON fields and add the new ones.  Inputs at
the benchmark shapes are generated on the device with a seeded generator
(CPU generation of 8 GB inputs per seed is too slow); `--small` uses the
oracle's small shapes with CPU-seeded inputs exactly as the reference does.

    python tests/eval_b200.py --problem 40_LayerNorm --out v.json [--small]
    python tests/eval_b200.py --all --out-dir verdicts/ [--small]   # one subprocess each
    torchrun --nproc-per-node N tests/eval_b200.py --problem P --out v.json   # N GPUs

Under torchrun every rank runs the whole protocol on its own GPU at the same
time (weak scaling: each GPU evaluates the full problem, L2 thrashed on every
device): parity must hold on every rank, each timed arm starts after a
barrier, and the verdict (written by rank 0) reports the max over ranks of
the median times, the per-rank medians, `ngpu`, and GB/s or TFLOP/s of the
whole job.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
for p in (str(REPO), str(REPO / "kernelbench-hip_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402

from oracle import problems  # noqa: E402
from tests.opmap import EXACT, ORACLE  # noqa: E402
from tests.protocol import (build_candidate, candidate_entry, candidate_path, digest,  # noqa: E402
                            digest_close, hash_tensor, static_check)

EVAL_SHA = hashlib.sha256(Path(__file__).read_bytes()).hexdigest()
SEEDS = [0, 1, 2, 3, 4]
REF_TOL = 1e-2
WARMUP, TRIALS, DISCARD_FIRST, STALL_RATIO = 5, 100, 1, 3.0
TIMEOUT_S = 900
# problems whose op tolerance is checked against the reference model run in
# float64 on the device: torch's fp32 CUDA cumsum is itself off by ~2e-3 at
# the benchmark shape, above the 1e-4 the library promises (the reference's
# own allclose(1e-2) is still checked against the fp32 eager model)
OP_REFERENCE_F64 = {"89_cumsum"}


def _peaks() -> dict:
    f = REPO / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# 3xTF32 ceiling: the bench's TF32 figure (cuBLAS TF32 8192^3 burst from its
# probe, bench.measure_tf32_tflops) divided by 3 — one denominator for both
from bench import TF32_CEILING_TFLOPS as TF32_BURST_TFLOPS  # noqa: E402


def clear_l2(device, nbytes: int) -> None:
    dummy = torch.empty(nbytes // 8, dtype=torch.int64, device=device)
    dummy.fill_(42)
    del dummy


def time_fn(fn, args, device, l2_bytes: int, trials: int = TRIALS) -> dict:
    for _ in range(WARMUP):
        fn(*args)
        torch.cuda.synchronize(device)
    times = []
    for trial in range(trials + DISCARD_FIRST):
        torch.cuda.synchronize(device)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clear_l2(device, l2_bytes)
        s.record()
        fn(*args)
        e.record()
        torch.cuda.synchronize(device)
        if trial >= DISCARD_FIRST:
            times.append(s.elapsed_time(e))
    med = statistics.median(times)
    return {"median_ms": round(med, 6), "mean_ms": round(statistics.fmean(times), 6),
            "std_ms": round(statistics.pstdev(times), 6), "min_ms": round(min(times), 6),
            "n": len(times), "stall_flag": med > STALL_RATIO * min(times)}


def _workload(name: str):
    from kbb200.workloads import WORKLOADS

    return next(w for w in WORKLOADS.values() if w.problem == name)


def _inputs(name, seed, device, small: bool):
    if small:
        _, get_inputs, _, _ = problems.load_problem(name, "small")
        torch.manual_seed(seed)
        return [t.to(device) for t in get_inputs()]
    from kbb200.workloads import make_inputs

    return make_inputs(_workload(name), device, seed=seed)


def _close(got, want, tol) -> bool:
    if tol == EXACT:
        return bool(torch.equal(got, want.to(got.dtype)))
    return bool(torch.isclose(got.float(), want.float(), atol=tol, rtol=tol).all())


def _cpu_sample(name: str, rows: int):
    """(shapes, fraction of the full workload) for a sample of `rows` along the
    leading (independent) dimension; None when the op cannot be cut."""
    spec = problems.input_spec(name)
    if name in ("6_Matmul_with_large_K_dimension_",):
        return None  # the K dimension cannot be cut without changing the op
    if name in ("3_Batched_matrix_multiplication",):
        return {"A": (rows, 512, 1024), "B": (rows, 1024, 512)}, rows / 256
    if name in ("12_Matmul_with_diagonal_matrices_",):
        return {"A": (rows,), "B": (rows, 4096)}, rows / 4096
    if name in ("95_CrossEntropyLoss",):
        full = dict((nm, shape) for nm, shape, _, _ in spec)["predictions"]
        rows = min(rows, full[0])
        return {"predictions": (rows, full[1]), "targets": (rows,)}, rows / full[0]
    shapes, frac = {}, 1.0
    for nm, shape, _, _ in spec:
        if len(shape) >= 2 and nm in ("x", "A") and shape[0] > rows:
            frac = rows / shape[0]
            shapes[nm] = (rows,) + tuple(shape[1:])
        elif nm in ("predictions", "targets") and shape[0] > rows * 4096:
            frac = rows * 4096 / shape[0]
            shapes[nm] = (rows * 4096,)
    return shapes, frac


def _cpu_time(name: str, target_s: float = 0.2, max_bytes: int = 512 << 20) -> dict | None:
    """torch-eager fp32 CPU forward on a bounded sample of the leading
    dimension, grown 4x at a time until one call takes >= target_s (so fixed
    per-call overhead does not inflate the full-size estimate), the sample is
    the whole tensor, or the next sample's inputs would pass max_bytes."""
    torch.set_num_threads(os.cpu_count() or 1)
    full_bytes = sum(4 * math.prod(shape) for _, shape, _, _ in problems.input_spec(name))
    rows, best = 4, None
    while True:
        cut = _cpu_sample(name, rows)
        if cut is None:
            return None
        shapes, frac = cut
        Model, get_inputs, get_init_inputs, _ = problems.load_problem(name, shapes)
        torch.manual_seed(0)
        ins = get_inputs()
        m = Model(*get_init_inputs())
        with torch.no_grad():
            m(*ins)
            t0 = time.perf_counter()
            m(*ins)
            dt = time.perf_counter() - t0
            done = dt >= target_s or frac >= 1.0 or full_bytes * min(1.0, 4 * frac) > max_bytes
            reps = 1
            if done and dt < target_s:  # final sample: repeat it up to target_s of work
                reps = min(50, max(1, math.ceil(target_s / max(dt, 1e-6))))
                t0 = time.perf_counter()
                for _ in range(reps):
                    m(*ins)
                dt = (time.perf_counter() - t0) / reps
        best = {"sample_ms": round(dt * 1e3, 3), "sample_fraction": frac, "sample_rows": rows,
                "sample_reps": reps, "full_ms_estimate": round(dt * 1e3 / frac, 3),
                "cores": os.cpu_count()}
        del ins, m
        if done:
            return best
        rows *= 4


def _ranks() -> tuple[int, int, int]:
    """(rank, world, local rank) of a torchrun launch; (0, 1, 0) otherwise."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def _all_ranks_ok(ok: bool, device) -> bool:
    import torch.distributed as tdist

    if not tdist.is_initialized():
        return ok
    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    tdist.all_reduce(t, op=tdist.ReduceOp.MIN)
    return bool(t.item())


def _timed_all_ranks(fn, args, device, l2, trials) -> dict:
    """time_fn on every rank at once; max over ranks of the medians."""
    import torch.distributed as tdist

    if not tdist.is_initialized():
        return time_fn(fn, args, device, l2, trials)
    tdist.barrier(device_ids=[device.index])
    r = time_fn(fn, args, device, l2, trials)
    meds = [torch.zeros(1, dtype=torch.float64, device=device) for _ in range(tdist.get_world_size())]
    tdist.all_gather(meds, torch.tensor([r["median_ms"]], dtype=torch.float64, device=device))
    per_rank = [round(m.item(), 6) for m in meds]
    r["per_rank_median_ms"] = per_rank
    r["median_ms"] = max(per_rank)
    return r


def evaluate(name: str, out_path: str | None = None, small: bool = False, trials: int = TRIALS,
             with_compile: bool = False, with_cpu: bool = True) -> dict:
    rank, world, local = _ranks()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if rank != 0:
        out_path = None  # rank 0 writes the verdict
    path = candidate_path(name)
    src = path.read_text()
    Model_ref, _, get_init_inputs, _ = problems.load_problem(name, "small" if small else None)
    init = get_init_inputs()
    _, tol = ORACLE[name]
    l2 = int(torch.cuda.get_device_properties(device).L2_cache_size) * 2
    v = {"problem": name, "candidate": str(path.relative_to(REPO)), "eval_sha": EVAL_SHA,
         "tol": REF_TOL, "op_tol": tol,
         "op_reference": "float64" if name in OP_REFERENCE_F64 else "float32 eager", "warmup": WARMUP, "trials": trials, "torch": torch.__version__,
         "device": torch.cuda.get_device_name(device), "shapes": "small" if small else "benchmark",
         "ngpu": world}
    entry = candidate_entry(src)
    v["static_check"] = static_check(src, entry)
    if not v["static_check"]["ok"]:
        v.update(milestone=-1, why="static anti-hack violation")
        return _write(out_path, v)
    t0 = time.time()
    try:
        cand_cls, _ = build_candidate(src)
    except Exception as e:  # noqa: BLE001
        v.update(milestone=-1, why=f"build failed: {type(e).__name__}: {e}")
        return _write(out_path, v)
    v["compile_s"] = round(time.time() - t0, 2)
    ref_model = Model_ref(*init).to(device)
    cand_model = cand_cls(*init).to(device)

    trials_out, passed, digests = [], 0, {}
    for seed in SEEDS:
        inputs = _inputs(name, seed, device, small)
        pre = [hash_tensor(t) for t in inputs]
        with torch.no_grad():
            want = ref_model(*inputs)
            torch.cuda.synchronize(device)
            got = cand_model(*inputs)
            torch.cuda.synchronize(device)
            want_op = (ref_model(*[t.double() if t.is_floating_point() else t for t in inputs]).float()
                       if name in OP_REFERENCE_F64 else want)
        row = {"seed": seed}
        if [hash_tensor(t) for t in inputs] != pre:
            row.update({"pass": False, "why": "R1 input mutated"})
        elif got.shape != want.shape:
            row.update({"pass": False, "why": f"shape {tuple(got.shape)} vs {tuple(want.shape)}"})
        else:
            ref_ok = bool(torch.allclose(got.float(), want.float(), atol=REF_TOL, rtol=REF_TOL))
            op_ok = _close(got, want_op, tol)
            row.update({"pass": ref_ok and op_ok, "ref_allclose": ref_ok, "op_tolerance": op_ok,
                        "max_diff": float((got.double() - want.double()).abs().max().item()),
                        "max_diff_op": float((got.double() - want_op.double()).abs().max().item())})
            if row["pass"]:
                digests[seed] = digest(got.float())
                passed += 1
        trials_out.append(row)
        del inputs, want, want_op, got
        torch.cuda.empty_cache()
    inputs0 = _inputs(name, 0, device, small)
    with torch.no_grad():
        again = cand_model(*inputs0)
    r2 = 0 in digests and digest_close(digests[0], digest(again.float()))
    del again
    ok_all = _all_ranks_ok(passed == len(SEEDS) and r2, device)
    v["parity"] = {"parity": ok_all, "trials_passed": passed, "recompute_check": r2,
                   "trials": trials_out}
    if world > 1:
        v["parity"]["all_ranks"] = ok_all
    if not v["parity"]["parity"]:
        v.update(milestone=-1, why="parity failed")
        return _write(out_path, v)

    with torch.no_grad():
        v["cand_time"] = _timed_all_ranks(cand_model, inputs0, device, l2, trials)
        v["eager_time"] = _timed_all_ranks(ref_model, inputs0, device, l2, trials)
        if with_compile:
            try:
                torch._dynamo.reset()
                cm = torch.compile(ref_model, backend="inductor", mode="default")
                v["compiled_time"] = _timed_all_ranks(cm, inputs0, device, l2, trials)
            except Exception as e:  # noqa: BLE001
                v["compiled_time"] = None
                v["compiled_error"] = repr(e)[:300]
    c, e = v["cand_time"]["median_ms"], v["eager_time"]["median_ms"]
    v["speedup_eager"] = round(e / c, 4) if c > 0 else None
    if v.get("compiled_time"):
        v["speedup_compiled"] = round(v["compiled_time"]["median_ms"] / c, 4)
    milestone = 1 + (v["speedup_eager"] and v["speedup_eager"] > 1.0)
    if v.get("speedup_compiled") and v["speedup_compiled"] > 1.0:
        milestone = 3
    v["milestone"] = int(milestone)

    if not small:
        w = _workload(name)
        v["algo_bytes"] = w.algo_bytes
        v["gbs"] = round(w.algo_bytes * world / (c * 1e-3) / 1e9, 1)  # whole job
        if w.flops:
            v["tflops"] = round(w.flops * world / (c * 1e-3) / 1e12, 2)
        peaks = _peaks()
        if w.bound == "tensor":
            v["roofline_frac"] = round(v["tflops"] / world / (TF32_BURST_TFLOPS / 3.0), 4)
            v["roofline"] = "3xTF32 = measured TF32 burst / 3 (per GPU)"
        else:
            v["roofline_frac"] = round(v["gbs"] / world / peaks["hbm_gbs"], 4)
            v["roofline"] = f"HBM copy {peaks['hbm_gbs']} GB/s per GPU ({peaks['source']})"
        if with_cpu and rank == 0:
            try:
                v["cpu"] = _cpu_time(name)
            except Exception as ex:  # noqa: BLE001
                v["cpu"] = {"error": repr(ex)[:200]}
    return _write(out_path, v)


def _write(out_path, v):
    if out_path:
        Path(out_path).parent.mkdir(parents=True, exist_ok=True)
        Path(out_path).write_text(json.dumps(v, indent=1, default=str) + "\n")
    return v


def run_all(out_dir: str, small: bool, names=None, extra=()) -> int:
    """One subprocess per problem (a fault or hang costs one verdict, not
    the sweep), SIGKILL of the process group after TIMEOUT_S, resumable:
    problems with a verdict file already present are skipped."""
    import signal

    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    for name in names or problems.SUBSET:
        vf = out / f"{name}.json"
        if vf.exists():
            continue
        cmd = [sys.executable, str(Path(__file__).resolve()), "--problem", name, "--out", str(vf), *extra]
        if small:
            cmd.append("--small")
        proc = subprocess.Popen(cmd, start_new_session=True)
        try:
            rc = proc.wait(timeout=TIMEOUT_S)
            if rc != 0 and not vf.exists():
                vf.write_text(json.dumps({"problem": name, "milestone": -1, "why": f"eval exited {rc}"}) + "\n")
        except subprocess.TimeoutExpired:
            os.killpg(proc.pid, signal.SIGKILL)
            proc.wait()
            vf.write_text(json.dumps({"problem": name, "milestone": -1,
                                      "why": f"eval killed after {TIMEOUT_S} s"}) + "\n")
        v = json.loads(vf.read_text())
        print(f"{name}: milestone {v.get('milestone')} speedup_eager {v.get('speedup_eager')} "
              f"roofline {v.get('roofline_frac')}", flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--problem")
    ap.add_argument("--out")
    ap.add_argument("--all", action="store_true")
    ap.add_argument("--out-dir", default="verdicts")
    ap.add_argument("--small", action="store_true")
    ap.add_argument("--trials", type=int, default=TRIALS)
    ap.add_argument("--compile", action="store_true", help="also time torch.compile(inductor)")
    ap.add_argument("--no-cpu", action="store_true")
    a = ap.parse_args()
    rank, world, local = _ranks()
    if a.all:
        if world > 1:
            ap.error("--all runs one subprocess per problem on one GPU; use --problem under torchrun")
        extra = ["--trials", str(a.trials)] + (["--compile"] if a.compile else []) + (
            ["--no-cpu"] if a.no_cpu else [])
        return run_all(a.out_dir, a.small, extra=extra)
    if world > 1:
        import datetime

        import torch.distributed as tdist

        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                 timeout=datetime.timedelta(seconds=300))
    try:
        v = evaluate(a.problem, a.out, a.small, a.trials, a.compile, not a.no_cpu)
    finally:
        if world > 1:
            import torch.distributed as tdist

            tdist.barrier()
            tdist.destroy_process_group()
    if rank == 0:
        print(json.dumps({k: v.get(k) for k in ("problem", "ngpu", "milestone", "speedup_eager", "gbs",
                                                "tflops", "roofline_frac", "why")}, default=str))
    return 0


if __name__ == "__main__":
    sys.exit(main())
