"""Benchmark: per-op HBM GB/s (or TFLOP/s) of the B200 operator library as a
fraction of the measured roofline, beside the reference arm on the host CPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload rownorm]
    torchrun --nproc-per-node N bench.py --gpus N ...          (N > 1)
    python bench.py --impl reference ...                       (CPU reference arm)

A step is one pass of the workload family's ops over their benchmark-shape
inputs (default family "rownorm": LayerNorm and RMSNorm on x[65536, 8192],
softmax and log-softmax on logits[8192, 32768]).  Inputs are seeded synthetic
tensors generated on the device and resident before timing.  Between two
launches of one op the step moves at least twice the L2 (126 MB) through
other buffers (the op's own inputs, or the family's other ops); an op for which
that does not hold gets a 256 MB L2 flush before each launch, outside its
per-op events but inside the step time.  Multi-GPU is weak scaling: every rank
runs the full workload on its own GPU (rows are independent; no collective on
this family), and the step time is the max over ranks.

One JSON line is printed by rank 0.  `value` is GB/s of algorithmic bytes
over device time; `e2e` repeats the step through the public candidate API
with pinned host inputs and outputs (H2D + kernels + D2H timed; ops whose
rows are independent stream through in row blocks, copies in both
directions overlapping the kernels on three streams); `roofline`
covers the dominant kernel; `cpu_baseline` is the torch-eager CPU reference
on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "kernelbench-hip_b200"))
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

PEAKS_FILE = REPO / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
L2_BYTES = 126 * 1024 * 1024
# ops whose sharded form has a cross-GPU step (kbb200.dist)
COLLECTIVE_OPS = {"mse_loss", "frobenius_normalize", "batch_norm_train", "matmul_splitk", "cross_entropy"}
FLUSH_BYTES = 256 * 1024 * 1024

# kernels launched per op call (for gpu_launches)
LAUNCHES = {"gelu_tanh": 1, "gelu_erf": 1, "swish": 1, "relu": 1, "layer_norm": 1, "rms_norm": 1,
            "softmax": 1, "log_softmax": 1, "sum_dim": 1, "mean_dim": 1, "argmax_dim": 1,
            "mse_loss": 2, "frobenius_normalize": 3, "max_pool2d": 1, "batch_norm_train": 2,
            "matmul": 1, "bmm": 1, "matmul_splitk": 2, "gemv": 1, "matmul_transposed_a": 1,
            "matmul_symmetric": 1, "diag_matmul": 1, "matmul_small_k": 1,
            "avg_pool2d": 1, "cumsum": 1, "cross_entropy": 2}
# sharded forms (world > 1): partial kernels + finishing kernel, plus the
# peer-memory all-reduce kernel when the collective is ours (NCCL's own
# kernels are not counted); split-K: partial GEMM + fused reduction, or
# GEMM + split reduce before NCCL
LAUNCHES_SHARDED = {"mse_loss": 3, "frobenius_normalize": 3, "batch_norm_train": 3, "cross_entropy": 3,
                    "matmul_splitk": 1}


def launches(name: str, world: int, collective: str) -> int:
    if world > 1 and name in LAUNCHES_SHARDED:
        return LAUNCHES_SHARDED[name] + (1 if collective == "p2p" or name == "matmul_splitk" else 0)
    return LAUNCHES[name]

# DRAM bytes per full-size launch (dram__bytes_read.sum + dram__bytes_write.sum)
# from the ncu captures summarised in profiles/: captured on a quarter of the
# rows (or the full tensor for gelu) and scaled by the rows processed, which
# the streaming kernels' traffic is proportional to.
NCU_DRAM_BYTES: dict[str, float | None] = {
    "layer_norm": 4.0 * (536.950528e6 + 483.113216e6),
    "softmax": 4.0 * (268.45568e6 + 212.02432e6),
    "gelu_tanh": 268.47744e6 + 214.69824e6,
    "diag_matmul": 67.13344e6 + 19.756544e6,
    # captured on A[8192, 64] (a quarter of the rows; B-resident form), scaled by 4
    "matmul_small_k": 4.0 * (10.549248e6 + 1013.272e6),
    "sum_dim": 4.0 * (2147.519e6 + 3.969536e6),
    "max_pool2d": 4.0 * (540.104192e6 + 107.429888e6),
    "gemv": 4.0 * (4299.227e6 + 3.568896e6),
    "batch_norm_train": 4.0 * (536.913408e6 + 4.80512e6 + 536.905984e6 + 490.593024e6),
}

# bounded CPU samples (fraction of the leading dim) for the CPU reference arm
CPU_SAMPLE_ROWS = {"layer_norm": 1024, "rms_norm": 1024, "softmax": 256, "log_softmax": 256,
                   "gelu_tanh": 512, "gelu_erf": 512, "swish": 512, "relu": 512,
                   "sum_dim": 4, "mean_dim": 4, "argmax_dim": 4, "frobenius_normalize": 8,
                   "max_pool2d": 1, "batch_norm_train": 2, "avg_pool2d": 1, "cumsum": 256,
                   "cross_entropy": 1024}


def load_peaks() -> dict:
    if PEAKS_FILE.exists():
        p = json.loads(PEAKS_FILE.read_text())
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS, "source": "fallback"}


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock, power and throttle reasons of one GPU via NVML in a
    background thread; `mark()` brackets the timed region."""

    REASONS = {  # NVML clocks-event reason bits
        0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
        0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, gpu_index: int, period_s: float = 0.02):
        self.samples: list[tuple[float, float, int, float]] = []
        self.window = [None, None]
        self._stop = threading.Event()
        self.ok = False
        self.sm_max = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
            self.sm_max = float(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
            self.ok = True
        except Exception:
            return
        self._t = threading.Thread(target=self._run, args=(period_s,), daemon=True)
        self._t.start()

    def _run(self, period):
        nv, h = self._nv, self._h
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                try:
                    r = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                except AttributeError:
                    r = int(nv.nvmlDeviceGetCurrentClocksThrottleReasons(h))
                pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                self.samples.append((time.perf_counter(), sm, r, pw))
            except Exception:
                pass
            time.sleep(period)

    def mark(self, i: int):
        self.window[i] = time.perf_counter()

    def summary(self) -> dict | None:
        if not self.ok:
            return None
        self._stop.set()
        self._t.join(timeout=1)
        t0, t1 = self.window
        inside = [s for s in self.samples if t0 is not None and t1 is not None and t0 <= s[0] <= t1]
        scope = "timed_region"
        if len(inside) < 3:  # region shorter than a few sample periods
            inside, scope = self.samples, "whole_run"
        if not inside:
            return None
        reasons = set()
        for _, _, r, _ in inside:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": self.sm_max,
                "power_w_max": round(max(s[3] for s in inside), 1), "reasons": sorted(reasons),
                "samples": len(inside), "scope": scope}


# ----------------------------------------------------------------- workload plumbing
def make_runner(name: str, inputs: list, world: int, rank: int, comm=None):
    """Returns (run() -> None, outputs) launching op `name` into preallocated
    outputs through the public tensor API (kbb200.ops; kbb200.dist for the
    ops with a cross-GPU step when world > 1, over `comm` if given, else
    NCCL)."""
    from kbb200 import ops as K
    from kbb200.workloads import WORKLOADS

    w = WORKLOADS[name]
    x = inputs[0]
    if name in ("gelu_tanh", "gelu_erf", "swish", "relu", "softmax", "log_softmax",
                "frobenius_normalize"):
        y = torch.empty_like(x)
        fn = getattr(K, name)
        if name == "frobenius_normalize" and world > 1:
            from kbb200 import dist

            return (lambda: dist.frobenius_normalize(x, out=y, comm=comm)), y
        return (lambda: fn(x, out=y)), y
    if name == "layer_norm":
        y = torch.empty_like(x)
        return (lambda: K.layer_norm(x, inputs[1], inputs[2], 1e-5, out=y)), y
    if name == "rms_norm":
        y = torch.empty_like(x)
        return (lambda: K.rms_norm(x, inputs[1], 1e-5, out=y)), y
    if name in ("sum_dim", "mean_dim"):
        y = torch.empty(x.shape[0], x.shape[2], device=x.device)
        fn = getattr(K, name)
        return (lambda: fn(x, 1, out=y)), y
    if name == "argmax_dim":
        y = torch.empty(x.shape[0], x.shape[2], device=x.device, dtype=torch.int64)
        return (lambda: K.argmax_dim(x, 1, out=y)), y
    if name == "mse_loss":
        y = torch.empty((), device=x.device)
        if world > 1:
            from kbb200 import dist

            return (lambda: dist.mse_loss(x, inputs[1], out=y, comm=comm)), y
        return (lambda: K.mse_loss(x, inputs[1], out=y)), y
    if name == "max_pool2d":
        e = w.extra
        N, C, H, W = x.shape
        y = torch.empty(N, C, H // 2, W // 2, device=x.device)
        return (lambda: K.max_pool2d(x, e["kernel_size"], e["stride"], e["padding"],
                                     e["dilation"], out=y)), y
    if name == "batch_norm_train":
        y = torch.empty_like(x)
        if world > 1:
            from kbb200 import dist

            return (lambda: dist.batch_norm_train(x, inputs[1], inputs[2], out=y, comm=comm)), y
        return (lambda: K.batch_norm_train(x, inputs[1], inputs[2], out=y)), y
    if name == "matmul":
        y = torch.empty(x.shape[0], inputs[1].shape[1], device=x.device)
        return (lambda: K.matmul(x, inputs[1], out=y)), y
    if name == "bmm":
        y = torch.empty(x.shape[0], x.shape[1], inputs[1].shape[2], device=x.device)
        return (lambda: K.bmm(x, inputs[1], out=y)), y
    if name == "matmul_splitk":
        y = torch.empty(x.shape[0], inputs[1].shape[1], device=x.device)
        if world > 1:
            from kbb200 import dist

            return (lambda: dist.matmul_splitk(x, inputs[1], out=y, comm=comm)), y
        return (lambda: K.matmul_splitk(x, inputs[1], out=y)), y
    if name == "gemv":
        y = torch.empty(x.shape[0], device=x.device)
        return (lambda: K.gemv(x, inputs[1], out=y)), y
    if name == "matmul_transposed_a":
        y = torch.empty(x.shape[1], inputs[1].shape[1], device=x.device)
        return (lambda: K.matmul(x, inputs[1], trans_a=True, out=y)), y
    if name in ("matmul_symmetric", "matmul_small_k"):
        y = torch.empty(x.shape[0], inputs[1].shape[1], device=x.device)
        return (lambda: K.matmul(x, inputs[1], out=y)), y
    if name == "avg_pool2d":
        e = w.extra
        N, C, H, W = x.shape
        y = torch.empty(N, C, H // 2, W // 2, device=x.device)
        return (lambda: K.avg_pool2d(x, e["kernel_size"], e["stride"], e["padding"], out=y)), y
    if name == "cumsum":
        y = torch.empty_like(x)
        return (lambda: K.cumsum(x, 1, out=y)), y
    if name == "cross_entropy":
        y = torch.empty((), device=x.device)
        if world > 1:
            from kbb200 import dist

            return (lambda: dist.cross_entropy(x, inputs[1], out=y, comm=comm)), y
        return (lambda: K.cross_entropy(x, inputs[1], out=y)), y
    if name == "diag_matmul":
        y = torch.empty_like(inputs[1])
        return (lambda: K.diag_matmul(x, inputs[1], out=y)), y
    raise KeyError(name)


def load_candidate(problem: str):
    """The candidate module for `problem` (ENTRY + Model), the public API."""
    import importlib.util

    path = REPO / "kernelbench-hip_b200" / "candidates" / problem / "b200.py"
    spec = importlib.util.spec_from_file_location(f"cand_{problem}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# inputs split along dim 0 when an op's rows (batch items) are independent;
# the output splits along dim 0 with them, other inputs are copied whole
ROW_SPLIT = {"gelu_tanh": (0,), "gelu_erf": (0,), "swish": (0,), "relu": (0,), "layer_norm": (0,),
             "rms_norm": (0,), "softmax": (0,), "log_softmax": (0,), "sum_dim": (0,), "mean_dim": (0,),
             "argmax_dim": (0,), "max_pool2d": (0,), "avg_pool2d": (0,), "cumsum": (0,), "bmm": (0, 1),
             "gemv": (0,), "diag_matmul": (0, 1), "matmul": (0,), "matmul_symmetric": (0,),
             "matmul_small_k": (0,)}


class E2EStreams:
    """The three streams the end-to-end step runs on (host-to-device copies,
    candidate forwards, device-to-host copies), shared by every op of the
    step so that one op's uploads overlap the previous op's tail."""

    def __init__(self, device):
        self.device = device
        self.s_in, self.s_cmp, self.s_out = (torch.cuda.Stream(device) for _ in range(3))

    def begin(self):  # work already on the current stream comes first
        self.s_in.wait_stream(torch.cuda.current_stream(self.device))

    def end(self):  # the current stream waits for every download
        torch.cuda.current_stream(self.device).wait_stream(self.s_out)


def e2e_runner(name: str, problem: str, host_inputs: list, host_out: torch.Tensor, device, chunks: int,
               streams: E2EStreams):
    """One end-to-end call through the candidate API: pinned host inputs ->
    device, Model.forward (the compiled EXT entry), result -> pinned host.
    Row-independent ops are cut into `chunks` row blocks whose host-to-device
    copy, forward and device-to-host copy run on the three streams, so the two
    copy directions and the kernels overlap; other ops run whole.  A block's
    device input is rewritten (next call) only after its forward finished."""
    model = load_candidate(problem).Model().to(device)
    split = ROW_SPLIT.get(name) if chunks > 1 else None
    rows = host_inputs[0].shape[0] if host_inputs[0].dim() else 1
    k = min(chunks, rows) if split else 1
    bounds = [(rows * i // k, rows * (i + 1) // k) for i in range(k)]
    dev_in = [torch.empty(h.shape, dtype=h.dtype, device=device) for h in host_inputs]
    st = streams
    done = [None] * k  # forward of block i finished (previous call)

    def run():
        for ci, (lo, hi) in enumerate(bounds):
            if done[ci] is not None:
                st.s_in.wait_event(done[ci])
            if ci == 0 and done[k - 1] is not None:  # whole inputs are read by every block
                st.s_in.wait_event(done[k - 1])
            with torch.cuda.stream(st.s_in):
                for j, h in enumerate(host_inputs):
                    if split and j in split:
                        dev_in[j][lo:hi].copy_(h[lo:hi], non_blocking=True)
                    elif ci == 0:
                        dev_in[j].copy_(h, non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(st.s_in)
            st.s_cmp.wait_event(ev_in)
            with torch.cuda.stream(st.s_cmp), torch.no_grad():
                out = model(*[d[lo:hi] if (split and j in split) else d for j, d in enumerate(dev_in)])
                done[ci] = torch.cuda.Event()
                done[ci].record(st.s_cmp)
            st.s_out.wait_event(done[ci])
            out.record_stream(st.s_out)
            with torch.cuda.stream(st.s_out):
                dst = host_out[lo:hi] if split else host_out
                dst.copy_(out.reshape(dst.shape), non_blocking=True)

    return run


def bytes_of(ts) -> int:
    return sum(t.numel() * t.element_size() for t in ts)


# ----------------------------------------------------------------- CPU reference arm
def cpu_reference(ops: list[str], steps: int, warmup: int, threads: int,
                  budget_s: float = 60.0) -> dict:
    """Torch-eager fp32 CPU forward of the reference models on a bounded
    sample of each op's benchmark input (leading dim cut to CPU_SAMPLE_ROWS)."""
    from kbb200.workloads import WORKLOADS
    from oracle import problems

    torch.set_num_threads(threads)
    models, samples, nbytes = [], [], 0
    desc = []
    for name in ops:
        w = WORKLOADS[name]
        rows = CPU_SAMPLE_ROWS.get(name)
        shapes = {}
        for nm, shape, _ in w.inputs:
            if nm in ("x", "predictions", "targets", "A") and rows:
                shapes[nm] = (min(rows, shape[0]),) + tuple(shape[1:])
        Model, get_inputs, get_init_inputs, _ = problems.load_problem(w.problem, shapes)
        torch.manual_seed(0)
        ins = get_inputs()
        m = Model(*get_init_inputs())
        with torch.no_grad():
            out = m(*ins)
        frac = ins[0].numel() / w.numel(0)
        nbytes += w.algo_bytes * frac
        models.append((m, ins))
        desc.append(f"{name}{list(ins[0].shape)}")
    with torch.no_grad():
        for _ in range(warmup):
            for m, ins in models:
                m(*ins)
        t0 = time.perf_counter()
        done = 0
        while done < steps:
            for m, ins in models:
                m(*ins)
            done += 1
            if time.perf_counter() - t0 > budget_s:
                break
        dt = time.perf_counter() - t0
    steps = done
    gbs = nbytes * steps / dt / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": "torch-eager fp32 CPU reference models on " + ", ".join(desc),
            "seconds": round(dt, 3), "steps": steps}


# ----------------------------------------------------------------- profiling driver
def profile_op(op: str, frac: float, reps: int = 3) -> int:
    """Run one op `reps` times on a reduced copy of its benchmark input (the
    leading dim scaled by `frac`; GEMMs at 4096^3 or a K/batch fraction) so a
    single launch can be captured by ncu within a few GB of device memory."""
    from kbb200 import ops as K
    from kbb200.workloads import WORKLOADS, make_inputs

    w = WORKLOADS[op]
    dev = torch.device("cuda:0")
    shapes = {}
    for nm, shape, _ in w.inputs:
        if op in ("matmul", "matmul_transposed_a", "matmul_symmetric"):
            shapes[nm] = (4096, 4096)
        elif op == "matmul_small_k":  # fewer rows of A; K and B unchanged
            if nm == "A":
                shapes[nm] = (max(1, int(shape[0] * frac)), shape[1])
        elif op == "diag_matmul":  # fewer rows of diag(A) and B
            shapes[nm] = (max(1, int(shape[0] * frac)),) + tuple(shape[1:])
        elif op == "matmul_splitk":
            shapes[nm] = (shape[0], int(shape[1] * frac)) if nm == "A" else (int(shape[0] * frac), shape[1])
        elif nm in ("x", "predictions", "targets", "A", "B") and len(shape) > 1 or nm in ("predictions", "targets"):
            if op == "gemv" and nm == "x":
                continue
            shapes[nm] = (max(1, int(shape[0] * frac)),) + tuple(shape[1:])
    ins = make_inputs(w, dev, 0, shapes)
    runner, _ = make_runner(op, ins, 1, 0)
    for _ in range(reps):
        runner()
    torch.cuda.synchronize()
    print("profiled", op, [tuple(t.shape) for t in ins], flush=True)
    return 0


# ----------------------------------------------------------------- main
class _StdoutToStderr:
    """Send everything written to fd 1 (including C-level prints such as
    NCCL's version banner) to stderr, so the result line is the only thing
    on stdout; `emit` writes to the original stdout."""

    def __enter__(self):
        sys.stdout.flush()
        self._saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def emit(self, line: str):
        sys.stdout.flush()
        os.write(self._saved, (line + "\n").encode())

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self._saved, 1)
        os.close(self._saved)
        return False


def main() -> int:
    with _StdoutToStderr() as sink:
        return _main(sink)


def _main(sink) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="rownorm")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--profile-op", default=None, help="run one op 3x on a reduced input (for ncu)")
    ap.add_argument("--e2e-chunks", type=int, default=8,
                    help="row blocks per op in the end-to-end pipeline (1: whole op, serial)")
    ap.add_argument("--collective", choices=("p2p", "nccl"), default="p2p",
                    help="cross-GPU sum of the sharded ops: the library's peer-memory kernel or NCCL")
    ap.add_argument("--frac", type=float, default=0.25, help="input fraction for --profile-op")
    a = ap.parse_args()
    if a.profile_op:
        return profile_op(a.profile_op, a.frac)
    if a.warmup < 3 and a.impl == "ours":
        a.warmup = 3

    from kbb200.workloads import FAMILIES, WORKLOADS

    ops = FAMILIES[a.workload] if a.workload in FAMILIES else a.workload.split(",")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    metric = f"GB/s of algorithmic bytes ({a.workload} family: {', '.join(ops)}); % of B200 roofline"
    config = {"workload": f"{a.workload}: " + "; ".join(
        f"{n} " + "x".join(map(str, WORKLOADS[n].inputs[0][1])) for n in ops),
        "parallelism": f"weak{world}"}

    if a.impl == "reference":
        if rank != 0:
            return 0
        threads = os.cpu_count() or 1
        r = cpu_reference(ops, a.steps, min(a.warmup, 1), threads, budget_s=90.0)
        line = {"metric": metric, "value": r["value"], "unit": "GB/s", "n_gpus": a.gpus,
                "steps": r["steps"], "warmup": min(a.warmup, 1),
                "ms_per_step": round(r["seconds"] / r["steps"] * 1e3, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": config, "impl": "reference",
                "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        sink.emit(json.dumps(line))
        return 0

    if not torch.cuda.is_available():
        sink.emit(json.dumps({"error": "no CUDA device"}))
        return 1
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        import torch.distributed as tdist

        tdist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    from kbb200.workloads import make_inputs

    # ops with a cross-GPU step sum their partials over peer memory with the
    # library's own kernel (kbb200.p2p), or over NCCL with --collective nccl
    comm = None
    if world > 1 and COLLECTIVE_OPS & set(ops):
        config["collective"] = a.collective
        if a.collective == "p2p":
            from kbb200.p2p import PeerComm

            comm = PeerComm(payload_bytes=1 << 20, timeout_s=10.0, device=device)
    peaks = load_peaks()
    runners = []
    for n in ops:
        w = WORKLOADS[n]
        ins = make_inputs(w, device, seed=rank)
        fn, out = make_runner(n, ins, world, rank, comm)
        runners.append((n, w, ins, fn, out))

    def barrier():
        if world > 1:
            torch.distributed.barrier(device_ids=[local_rank])

    # L2 hygiene: the bytes that pass between two launches of one op are its
    # own algorithmic bytes plus those of the family's other ops
    step_total = sum(w.algo_bytes for _, w, *_ in runners)
    need_flush = {n for n, w, *_ in runners if step_total < 2 * L2_BYTES}
    flush_buf = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=device) if need_flush else None
    config["l2"] = (f"L2 flush ({FLUSH_BYTES >> 20} MB write) before " + ", ".join(sorted(need_flush))
                    if need_flush else
                    f"no flush: >= {2 * L2_BYTES >> 20} MB moves between two launches of each op")

    stream = torch.cuda.current_stream(device)
    for _ in range(a.warmup):
        for _, _, _, fn, _ in runners:
            fn()
    torch.cuda.synchronize(device)

    clocks = ClockSampler(local_rank)
    ev = {n: [] for n, *_ in runners}
    barrier()
    torch.cuda.synchronize(device)
    clocks.mark(0)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for _ in range(a.steps):
        for n, _, _, fn, _ in runners:
            if n in need_flush:
                flush_buf.fill_(1.0)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            ev[n].append((e0, e1))
    t_end.record(stream)
    torch.cuda.synchronize(device)
    clocks.mark(1)
    barrier()
    total_ms = t_start.elapsed_time(t_end)
    per_op_ms = {n: sum(e0.elapsed_time(e1) for e0, e1 in ev[n]) / a.steps for n in ev}
    if world > 1:
        t = torch.tensor([total_ms] + [per_op_ms[n] for n in ev], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = t[0].item()
        per_op_ms = {n: t[i + 1].item() for i, n in enumerate(ev)}
    ms_per_step = total_ms / a.steps
    step_bytes = sum(w.algo_bytes for _, w, *_ in runners)
    value = step_bytes * world / (ms_per_step * 1e-3) / 1e9

    per_op = {}
    for n, w, *_ in runners:
        ms = per_op_ms[n]
        d = {"ms": round(ms, 4)}
        if w.flops:
            d["tflops"] = round(w.flops / (ms * 1e-3) / 1e12, 2)
        d["gbs"] = round(w.algo_bytes / (ms * 1e-3) / 1e9, 1)
        d["frac_hbm"] = round(d["gbs"] / peaks["hbm_gbs"], 4)
        per_op[n] = d
    dom_name, dom_w = max(((n, w) for n, w, *_ in runners), key=lambda t: t[1].algo_bytes)
    dom_ms = per_op_ms[dom_name]
    if dom_w.bound == "tensor":
        achieved = dom_w.flops / (dom_ms * 1e-3) / 1e12
        peak = peaks["bf16_tflops"]
        roof = {"bound": "tensor", "unit": "TFLOP/s"}
    else:
        achieved = dom_w.algo_bytes / (dom_ms * 1e-3) / 1e9
        peak = peaks["hbm_gbs"]
        roof = {"bound": "hbm", "unit": "GB/s"}
    roof.update({"kernel": dom_name, "achieved": round(achieved, 1), "peak": peak,
                 "peak_source": peaks["source"], "frac": round(achieved / peak, 4),
                 "traffic": NCU_DRAM_BYTES.get(dom_name), "algo_bytes": dom_w.algo_bytes,
                 "ms_per_launch": round(dom_ms, 4)})

    # ---- end to end through the candidate API with pinned host buffers
    e2e = None
    if not a.no_e2e:
        e2e_fns, h2d, d2h = [], 0, 0
        e2e_streams = E2EStreams(device)
        for n, w, ins, _, out in runners:
            hin = [t.cpu().pin_memory() for t in ins]
            hout = torch.empty(out.shape, dtype=out.dtype).pin_memory()
            e2e_fns.append(e2e_runner(n, w.problem, hin, hout, device, a.e2e_chunks, e2e_streams))
            h2d += bytes_of(hin)
            d2h += bytes_of([hout])
        e2e_streams.begin()
        for f in e2e_fns:
            f()
        e2e_streams.end()
        torch.cuda.synchronize(device)
        e2e_steps = max(1, min(a.steps, 5))
        barrier()
        torch.cuda.synchronize(device)
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        e2e_streams.begin()
        for _ in range(e2e_steps):
            for f in e2e_fns:
                f()
        e2e_streams.end()
        s1.record(stream)
        torch.cuda.synchronize(device)
        e2e_ms = s0.elapsed_time(s1) / e2e_steps
        if world > 1:
            t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e2e_ms = t.item()
        e2e = {"value": round(step_bytes * world / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
               "steps": e2e_steps,
               "pipeline": (f"{a.e2e_chunks} row blocks per row-independent op: H2D, candidate "
                            "Model.forward, D2H on three streams" if a.e2e_chunks > 1 else "serial")}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_reference(ops, a.cpu_steps, 1, os.cpu_count() or 1, budget_s=30.0)
        cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}

    clk = clocks.summary()
    if world > 1:
        import torch.distributed as tdist

        if comm is not None:
            comm.check()
            comm.close()
        tdist.barrier(device_ids=[local_rank])
        tdist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": metric, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, generated on device)", "config": config,
        "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
        "gpu_launches": a.steps * sum(launches(n, world, a.collective) for n in ops), "per_op": per_op,
        "impl": "ours",
    }
    sink.emit(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())
