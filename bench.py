"""Benchmark: the operator library's 19 benchmark operators, each against its
B200 roofline, on 1/2/4/8 GPUs, beside the torch-eager CPU reference.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload northstar]
    torchrun --nproc-per-node N bench.py --gpus N ...          (N > 1: sharded)
    python bench.py --impl reference ...                       (CPU reference arm)
    torchrun --nproc-per-node N bench.py --exchange-sweep      (cross-GPU step cost)

A step launches every op of the workload once on its benchmark-shape input.
Default workload "northstar", in config order: tanh-GELU, erf-GELU, Swish,
ReLU on x[4096, 16384]; LayerNorm and RMSNorm on x[65536, 8192]; softmax and
log-softmax on [8192, 32768]; sum, mean and argmax over dim 1 of
[128, 4096, 4096]; MSE of two 2^28 vectors; Frobenius normalisation of
[256, 1024, 1024]; max-pool k3 s2 p1 on [32, 64, 512, 512]; training-mode
BatchNorm on [64, 128, 256, 256]; the 3xTF32 GEMMs 8192^3, 256 x (512 x 1024
@ 1024 x 512) and 256 x 4,194,304 @ 4,194,304 x 256 (split K); matvec
[4096, 1,048,576].  Inputs are seeded synthetic tensors generated on the
device and resident before timing.

Multi-GPU is strong scaling: the global problem stays fixed and rank r holds
and processes only its shard of each op's input (kbb200.workloads.SHARD_DIMS:
rows, batch items, vector slices, GEMM rows or K slices).  MSE, Frobenius,
BatchNorm and split-K GEMM add their one exchange between a local partial
and a local finish (kbb200.dist): over the library's peer memory — fused into
the partial kernel for MSE, Frobenius and BatchNorm, the peer all-reduce
kernel (with the split fold) for split-K — or with `--collective nccl` over
NCCL.  Step times are the max over ranks.

`value` is roofline-weighted throughput in units of one B200 roofline: the
sum over the step's ops of the op's one-GPU roofline time (algorithmic bytes
at the measured copy bandwidth; for the tensor-core GEMMs the useful FLOPs
at the 3xTF32 ceiling when that takes longer) divided by the measured step
time.  1.0 = every op at its roofline on one B200; N GPUs at perfect
efficiency give N times the one-GPU value.  The 3xTF32 ceiling is a third of
cuBLAS's TF32 burst rate on an 8192^3 GEMM (the highest this probe measured
on the pool; the live probe of the same GPU just before timing is recorded in
`peaks`).  When the op with the largest share of the step is a GEMM, the
`roofline` record divides by the sustained ceiling (the burst one times the
live sustained / burst TF32 ratio: the GEMM runs inside a long, power-capped
step) and keeps the burst fraction beside it.  `per_op` gives each op's time, GB/s or
TFLOP/s of the global problem and fraction of the N-GPU roofline, from a
second pass of K steps with an event pair around every op (the step time
comes from a pass with no events between the ops).

L2: every op's input is larger than the 126 MB L2 or, between two launches of
one op, the step moves gigabytes through other buffers; no flush is needed
(`config.l2`).  `e2e` repeats the step through the public API (the
candidates' Model.forward; kbb200.dist for the sharded ops with an exchange)
from pinned host inputs to pinned host outputs, copies inside the timed
region; as in the benchmark configs, sum / mean / argmax read one x, as do
LayerNorm / RMSNorm and softmax / log-softmax, so that x crosses PCIe once per
step (the device-resident step shares it too).  `cpu_baseline` and
`--impl reference` time the reference arm, torch
eager fp32 on the host cores, on bounded samples of every op (each at least
four times the host's last-level cache) scaled to the same roofline units.
"""
from __future__ import annotations

import argparse
import glob
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
# The tensor-core ceiling of the 3xTF32 GEMMs: cuBLAS's TF32 rate on an 8192^3
# GEMM (measure_tf32_tflops), the highest burst this probe has measured on
# this pool's B200s (758.8 TFLOP/s; later runs 738.1 and 701.7, recorded in
# profiles/tf32_probe_8192cube.md), divided by three.  Both arms use this one
# figure, so their values are in the same units; every run also records its
# own live probe beside it.
TF32_CEILING_TFLOPS = 758.8
L2_BYTES = 126 * 1024 * 1024
FLUSH_BYTES = 256 * 1024 * 1024
# CPU reference samples: at least 4x the host's last-level cache and this
# many bytes per op; contractions about this many useful FLOPs
MIN_SAMPLE_BYTES = 256 << 20
SAMPLE_FLOPS = 2.0e11

# kernels of ours launched per op call (for gpu_launches)
LAUNCHES = {"gelu_tanh": 1, "gelu_erf": 1, "swish": 1, "relu": 1, "layer_norm": 1, "rms_norm": 1,
            "softmax": 1, "log_softmax": 1, "sum_dim": 1, "mean_dim": 1, "argmax_dim": 1,
            "mse_loss": 2, "frobenius_normalize": 3, "max_pool2d": 1, "batch_norm_train": 2,
            "matmul": 1, "bmm": 1, "matmul_splitk": 2, "gemv": 1, "matmul_transposed_a": 1,
            "matmul_symmetric": 1, "diag_matmul": 1, "matmul_small_k": 1,
            "avg_pool2d": 1, "cumsum": 1, "cross_entropy": 2}
# sharded forms with an exchange (world > 1): partial kernel(s) + finish
# kernel(s), not counting the exchange (NCCL's kernels are not ours; the peer
# all-reduce kernel adds one); split-K: GEMM + split reduction before NCCL, or
# the partial GEMM + the fused split fold and peer all-reduce
LAUNCHES_SHARDED = {"mse_loss": 3, "frobenius_normalize": 3, "batch_norm_train": 3, "cross_entropy": 3,
                    "matmul_splitk": 2}
# bytes each rank contributes to the exchange of a sharded op
EXCHANGE_BYTES = {"mse_loss": lambda w: 16, "frobenius_normalize": lambda w: 8,
                  "batch_norm_train": lambda w: 8 * (2 * w.inputs[0][1][1] + 1),
                  "cross_entropy": lambda w: 16,
                  "matmul_splitk": lambda w: 4 * w.inputs[0][1][0] * w.inputs[1][1][1]}


# DRAM bytes per full-size launch (dram__bytes_read.sum + dram__bytes_write.sum)
# from the ncu captures summarised in profiles/: captured on a reduced case
# and scaled by the units processed, which the streaming kernels' traffic is
# proportional to.  Only the streamed part scales: the output lines still in
# L2 when a captured launch ends (at most the 126 MB L2) are not written back
# within the launch, so a scaled figure would count that shortfall several
# times; the scaled figures below add it back once (see profiles/).
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
    # one full 8192^3 launch (grouped tile walk), profiles/gemm3x_8192cube_splitk.md
    "matmul": 2278.3488e6 + 258.073344e6,
}
# write-back still in L2 at the end of a quarter-size capture, per capture:
# output bytes per capture - captured DRAM writes (added back once)
NCU_L2_TAIL: dict[str, float] = {
    "layer_norm": 536.870912e6 - 483.113216e6,
    "softmax": 268.435456e6 - 212.02432e6,
    "max_pool2d": 134.217728e6 - 107.429888e6,
    "batch_norm_train": 536.870912e6 - 490.593024e6,
}


def ncu_traffic(name: str) -> float | None:
    t = NCU_DRAM_BYTES.get(name)
    if t is None:
        return None
    return t + (3.0 * NCU_L2_TAIL[name] if name in NCU_L2_TAIL else 0.0)


def load_peaks() -> dict:
    if PEAKS_FILE.exists():
        p = json.loads(PEAKS_FILE.read_text())
        out = {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
               "source": "measured (MEASURED_PEAKS.json)"}
        if p.get("bf16_tflops_sustained"):
            out["bf16_tflops_sustained"] = float(p["bf16_tflops_sustained"])
        return out
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS, "source": "fallback"}


def measure_tf32_tflops(device, n: int = 8192, reps: int = 10, sustain_s: float = 3.0) -> dict:
    """cuBLAS TF32 dense rate on this GPU (torch.matmul, allow_tf32, n^3):
    the tensor-core rate 3xTF32 divides by three.  `burst`: best of `reps`
    single calls (CUDA events); `sustained`: back-to-back calls for about
    `sustain_s` seconds, timed as one block, so the power cap has settled the
    clock as it does inside a long step.  Runs before any timed region."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        g = torch.Generator(device=device).manual_seed(1)
        a = torch.randn(n, n, device=device, generator=g)
        b = torch.randn(n, n, device=device, generator=g)
        c = torch.empty(n, n, device=device)
        for _ in range(3):
            torch.matmul(a, b, out=c)
        best = math.inf
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            torch.cuda.synchronize(device)
            best = min(best, e0.elapsed_time(e1))
        out = {"burst": 2.0 * n ** 3 / (best * 1e-3) / 1e12}
        if sustain_s > 0:
            calls = max(4, int(sustain_s / (best * 1e-3)))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(calls):
                torch.matmul(a, b, out=c)
            e1.record()
            torch.cuda.synchronize(device)
            out["sustained"] = 2.0 * n ** 3 * calls / (e0.elapsed_time(e1) * 1e-3) / 1e12
            out["sustained_calls"] = calls
        del a, b, c
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _tensor_peak(peaks: dict, live: dict | None) -> None:
    """Record the 3xTF32 ceiling both arms use, and this run's live probe.

    `tensor_tflops` (burst) is the unit of `value` and of the per-op
    fractions.  `tensor_tflops_sustained` is the same ceiling under the power
    cap, the denominator for a GEMM timed inside the long step: the burst
    ceiling times this box's live sustained / burst TF32 ratio (or, without a
    live probe, the pool's measured bf16 sustained / burst ratio)."""
    peaks["tf32_tflops"] = TF32_CEILING_TFLOPS
    peaks["tensor_tflops"] = round(TF32_CEILING_TFLOPS / 3.0, 2)
    peaks["tensor_source"] = ("3xTF32 ceiling = a third of cuBLAS TF32 8192^3, highest burst measured on this "
                              "pool by measure_tf32_tflops")
    ratio, how = None, None
    if live is not None:
        peaks["tf32_tflops_live"] = round(live["burst"], 1)
        if live.get("sustained"):
            peaks["tf32_tflops_live_sustained"] = round(live["sustained"], 1)
            ratio = live["sustained"] / live["burst"]
            how = (f"live cuBLAS TF32 sustained / burst on this GPU ({live['sustained']:.1f} / "
                   f"{live['burst']:.1f}, {live['sustained_calls']} back-to-back 8192^3 calls)")
    if ratio is None and peaks.get("bf16_tflops_sustained"):
        ratio = peaks["bf16_tflops_sustained"] / peaks["bf16_tflops"]
        how = (f"MEASURED_PEAKS.json bf16 sustained / burst ({peaks['bf16_tflops_sustained']} / "
               f"{peaks['bf16_tflops']})")
    if ratio is not None:
        ratio = min(ratio, 1.0)
        peaks["tensor_tflops_sustained"] = round(peaks["tensor_tflops"] * ratio, 2)
        peaks["tensor_sustained_source"] = f"3xTF32 burst ceiling x {ratio:.4f} = {how}"


def host_llc_bytes() -> tuple[int, str]:
    """Total last-level cache of the host (every distinct L3 instance), and
    how it was found."""
    seen, total = set(), 0
    for d in glob.glob("/sys/devices/system/cpu/cpu*/cache/index*"):
        try:
            if Path(d, "level").read_text().strip() != "3":
                continue
            key = Path(d, "shared_cpu_list").read_text().strip()
            if key in seen:
                continue
            seen.add(key)
            size = Path(d, "size").read_text().strip().upper()
            mult = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}.get(size[-1], 1)
            total += int(size.rstrip("KMG")) * mult
        except OSError:
            continue
    if total:
        return total, f"{len(seen)} L3 instance(s) in /sys"
    return 256 << 20, "unknown (assumed 256 MiB)"


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


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
def out_shape(name: str, inputs: list):
    """Shape and dtype of op `name`'s output for `inputs`."""
    x = inputs[0]
    if name in ("sum_dim", "mean_dim"):
        return (x.shape[0], x.shape[2]), torch.float32
    if name == "argmax_dim":
        return (x.shape[0], x.shape[2]), torch.int64
    if name in ("mse_loss", "cross_entropy"):
        return (), torch.float32
    if name in ("max_pool2d", "avg_pool2d"):
        N, C, H, W = x.shape
        return (N, C, H // 2, W // 2), torch.float32
    if name in ("matmul", "matmul_splitk", "matmul_symmetric", "matmul_small_k"):
        return (x.shape[0], inputs[1].shape[1]), torch.float32
    if name == "matmul_transposed_a":
        return (x.shape[1], inputs[1].shape[1]), torch.float32
    if name == "bmm":
        return (x.shape[0], x.shape[1], inputs[1].shape[2]), torch.float32
    if name == "gemv":
        return (x.shape[0],), torch.float32
    if name == "diag_matmul":
        return tuple(inputs[1].shape), torch.float32
    return tuple(x.shape), torch.float32


def make_runner(name: str, inputs: list, world: int, rank: int, comm=None, out=None):
    """Returns (run() -> None, out) launching op `name` into a preallocated
    output through the public tensor API (kbb200.ops; kbb200.dist for the
    ops with a cross-GPU step when world > 1, over `comm` if given, else
    NCCL)."""
    from kbb200 import ops as K
    from kbb200.workloads import WORKLOADS

    w = WORKLOADS[name]
    x = inputs[0]
    if out is None:
        shape, dtype = out_shape(name, inputs)
        out = torch.empty(shape, device=x.device, dtype=dtype)
    y = out
    sharded = world > 1
    if sharded and name in ("mse_loss", "frobenius_normalize", "batch_norm_train", "matmul_splitk",
                            "cross_entropy"):
        from kbb200 import dist

        if name == "mse_loss":
            return (lambda: dist.mse_loss(x, inputs[1], out=y, comm=comm)), y
        if name == "frobenius_normalize":
            return (lambda: dist.frobenius_normalize(x, out=y, comm=comm)), y
        if name == "batch_norm_train":
            return (lambda: dist.batch_norm_train(x, inputs[1], inputs[2], out=y, comm=comm)), y
        if name == "matmul_splitk":
            return (lambda: dist.matmul_splitk(x, inputs[1], out=y, comm=comm)), y
        return (lambda: dist.cross_entropy(x, inputs[1], out=y, comm=comm)), y
    if name in ("gelu_tanh", "gelu_erf", "swish", "relu", "softmax", "log_softmax",
                "frobenius_normalize"):
        fn = getattr(K, name)
        return (lambda: fn(x, out=y)), y
    if name == "layer_norm":
        return (lambda: K.layer_norm(x, inputs[1], inputs[2], 1e-5, out=y)), y
    if name == "rms_norm":
        return (lambda: K.rms_norm(x, inputs[1], 1e-5, out=y)), y
    if name in ("sum_dim", "mean_dim", "argmax_dim"):
        fn = getattr(K, name)
        return (lambda: fn(x, 1, out=y)), y
    if name == "mse_loss":
        return (lambda: K.mse_loss(x, inputs[1], out=y)), y
    if name == "max_pool2d":
        e = w.extra
        return (lambda: K.max_pool2d(x, e["kernel_size"], e["stride"], e["padding"],
                                     e["dilation"], out=y)), y
    if name == "batch_norm_train":
        return (lambda: K.batch_norm_train(x, inputs[1], inputs[2], out=y)), y
    if name in ("matmul", "matmul_symmetric", "matmul_small_k"):
        return (lambda: K.matmul(x, inputs[1], out=y)), y
    if name == "bmm":
        return (lambda: K.bmm(x, inputs[1], out=y)), y
    if name == "matmul_splitk":
        return (lambda: K.matmul_splitk(x, inputs[1], out=y)), y
    if name == "gemv":
        return (lambda: K.gemv(x, inputs[1], out=y)), y
    if name == "matmul_transposed_a":
        return (lambda: K.matmul(x, inputs[1], trans_a=True, out=y)), y
    if name == "avg_pool2d":
        e = w.extra
        return (lambda: K.avg_pool2d(x, e["kernel_size"], e["stride"], e["padding"], out=y)), y
    if name == "cumsum":
        return (lambda: K.cumsum(x, 1, out=y)), y
    if name == "cross_entropy":
        return (lambda: K.cross_entropy(x, inputs[1], out=y)), y
    if name == "diag_matmul":
        return (lambda: K.diag_matmul(x, inputs[1], out=y)), y
    raise KeyError(name)


# the same with the exchange fused into the partial kernel (kbb200.dist._fused)
LAUNCHES_FUSED = {"mse_loss": 1, "frobenius_normalize": 2, "batch_norm_train": 2}


def launches(name: str, world: int, comm, inputs=None) -> int:
    """Kernels of ours one call of op `name` launches (on these inputs)."""
    if name in ("matmul", "matmul_symmetric") and inputs is not None:
        from kbb200._lib import LIB

        M, K = inputs[0].shape
        return 2 if LIB.kb_sgemm_workspace_size(M, inputs[1].shape[1], K, 0) else 1  # K split + its reduction
    if world > 1 and name in LAUNCHES_SHARDED:
        from kbb200.dist import _fused, peer_path
        from kbb200.workloads import WORKLOADS

        nbytes = EXCHANGE_BYTES[name](WORKLOADS[name])
        if name == "matmul_splitk":
            return 2  # GEMM + split reduce (NCCL), or partial GEMM + fused peer fold
        if name in LAUNCHES_FUSED and _fused(comm, nbytes):
            return LAUNCHES_FUSED[name]
        return LAUNCHES_SHARDED[name] + (1 if peer_path(comm, nbytes) else 0)
    return LAUNCHES[name]


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
    forwards, device-to-host copies), shared by every op of the step so that
    one op's uploads overlap the previous op's tail."""

    def __init__(self, device):
        self.device = device
        self.s_in, self.s_cmp, self.s_out = (torch.cuda.Stream(device) for _ in range(3))

    def begin(self):  # work already on the current stream comes first
        self.s_in.wait_stream(torch.cuda.current_stream(self.device))

    def end(self):  # the current stream waits for every download
        torch.cuda.current_stream(self.device).wait_stream(self.s_out)


def e2e_runner(name: str, problem: str, host_inputs: list, host_out: torch.Tensor, device, chunks: int,
               streams: E2EStreams, dev_in: list | None = None, forward=None, extra=()):
    """One end-to-end call through the public API: pinned host inputs ->
    device, the forward, result -> pinned host.  The forward is the
    candidate's Model.forward (the compiled EXT entry) unless `forward`
    (inputs -> output tensor) is given.  `extra` lists further ops of the
    step that read the same inputs, as (forward, number of leading inputs
    it takes, pinned host output): they run on each uploaded block too, so
    the shared input crosses PCIe once per call.  Row-independent ops are
    cut into `chunks` row blocks whose host-to-device copy, forwards and
    device-to-host copies run on the three streams, so the two copy
    directions and the kernels overlap; other ops run whole.  A block's
    device input is rewritten (next call) only after its forwards finished.
    `dev_in` reuses device buffers."""
    if forward is None:
        model = load_candidate(problem).Model().to(device)
        forward = model
    members = [(forward, len(host_inputs), host_out)] + list(extra)
    split = ROW_SPLIT.get(name) if chunks > 1 else None
    rows = host_inputs[0].shape[0] if host_inputs[0].dim() else 1
    k = min(chunks, rows) if split else 1
    bounds = [(rows * i // k, rows * (i + 1) // k) for i in range(k)]
    if dev_in is None:
        dev_in = [torch.empty(h.shape, dtype=h.dtype, device=device) for h in host_inputs]
    st = streams
    done = [None] * k  # forwards of block i finished (previous call)

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
            args = [d[lo:hi] if (split and j in split) else d for j, d in enumerate(dev_in)]
            outs = []
            with torch.cuda.stream(st.s_cmp), torch.no_grad():
                for fwd, nargs, _ in members:
                    outs.append(fwd(*args[:nargs]))
                done[ci] = torch.cuda.Event()
                done[ci].record(st.s_cmp)
            st.s_out.wait_event(done[ci])
            for out, (_, _, hout) in zip(outs, members):
                out.record_stream(st.s_out)
                with torch.cuda.stream(st.s_out):
                    dst = hout[lo:hi] if split else hout
                    dst.copy_(out.reshape(dst.shape), non_blocking=True)

    return run


def bytes_of(ts) -> int:
    return sum(t.numel() * t.element_size() for t in ts)


# ----------------------------------------------------------------- CPU reference arm
def cpu_sample(w, target_bytes: float, target_flops: float) -> tuple[dict, float]:
    """Shapes of a bounded sample of workload `w` for the CPU reference —
    the op's shard units (rows, batch items, slices, K) cut so that the
    sample moves about `target_bytes` (contractions: about `target_flops`) —
    and the fraction of the full workload's units it holds."""
    from kbb200.workloads import SHARD_DIMS

    dims = SHARD_DIMS[w.name]
    first, d = next(iter(dims.items()))
    full = dict((n, s) for n, s, _ in w.inputs)
    units = full[first][d]
    if w.bound == "tensor":
        want = math.ceil(target_flops / (w.flops / units))
    else:
        want = math.ceil(target_bytes / (w.algo_bytes / units))
    take = max(1, min(units, want))
    shapes = {}
    for n, dim in dims.items():
        s = list(full[n])
        s[dim] = take
        shapes[n] = tuple(s)
    return shapes, take / units


def _fast_inputs(problem: str, shapes: dict, seed: int = 0) -> list:
    """Inputs for a CPU sample with the problem's distributions, drawn as one
    seeded 32 MiB block per input and tiled (the CPU reference's time does
    not depend on the values; drawing gigabytes with the CPU generator
    would take minutes)."""
    from oracle import problems

    g = torch.Generator().manual_seed(seed)
    out = []
    for nm, shape, dist, fan_in in problems.input_spec(problem, shapes):
        n = math.prod(shape)
        if dist == "labels":
            out.append(torch.randint(0, fan_in, shape, dtype=torch.int64, generator=g))
            continue
        if dist == "gemm_sym":
            out.append(problems.draw(shape, dist, fan_in))
            continue
        block = min(n, 1 << 23)
        torch.manual_seed(int(torch.randint(0, 2**31 - 1, (1,), generator=g)))
        base = problems.draw((block,), dist if dist != "gemm_t" else "gemm", fan_in if dist == "gemm" else
                             (shape[0] if dist == "gemm_t" else 1))
        t = torch.empty(n)
        for i in range(0, n, block):
            m = min(block, n - i)
            t[i:i + m] = base[:m]
        out.append(t.view(shape))
    return out


def cpu_reference(ops: list[str], steps: int, warmup: int, threads: int, peaks: dict,
                  budget_s: float = 60.0) -> dict:
    """Torch-eager fp32 CPU forward of the reference models (the reference
    arm of the protected eval) on a bounded sample of every op, each sample
    at least 4x the host's last-level cache (contractions: ~0.2 TFLOP),
    timed as one step over all ops.  The result is in the same roofline
    units as the GPU value: the samples' one-B200 roofline time over the CPU
    step time."""
    from kbb200.workloads import WORKLOADS
    from oracle import problems

    torch.set_num_threads(threads)
    llc, llc_how = host_llc_bytes()
    target_bytes = max(4 * llc, MIN_SAMPLE_BYTES)
    target_flops = SAMPLE_FLOPS
    models, desc = [], []
    roof_s, sample_bytes = 0.0, 0.0
    for name in ops:
        w = WORKLOADS[name]
        shapes, frac = cpu_sample(w, target_bytes, target_flops)
        Model, _, get_init_inputs, _ = problems.load_problem(w.problem, shapes)
        ins = _fast_inputs(w.problem, shapes)
        m = Model(*get_init_inputs())
        with torch.no_grad():
            m(*ins)
        t = w.algo_bytes * frac / (peaks["hbm_gbs"] * 1e9)
        if w.bound == "tensor":
            t = max(t, w.flops * frac / (peaks["tensor_tflops"] * 1e12))
        roof_s += t
        sample_bytes += w.algo_bytes * frac
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
    step_s = dt / done
    return {"value": round(roof_s / step_s, 6), "unit": "B200 rooflines", "cores": threads, "kind": "port",
            "sample": ("torch-eager fp32 CPU reference models, one step over samples of every op, each "
                       f">= 4x the host LLC ({llc >> 20} MiB, {llc_how}) or ~0.2 TFLOP: " + ", ".join(desc)),
            "gbs": round(sample_bytes / step_s / 1e9, 3), "seconds": round(dt, 3), "steps": done,
            "ms_per_step": round(step_s * 1e3, 3)}


# ----------------------------------------------------------------- profiling driver
def profile_op(op: str, frac: float, reps: int = 3) -> int:
    """Run one op `reps` times on a reduced copy of its benchmark input (the
    leading dim scaled by `frac`; GEMMs at 4096^3 or a K/batch fraction) so a
    single launch can be captured by ncu within a few GB of device memory.
    `frac` 1 with a square GEMM keeps 8192^3."""
    from kbb200.workloads import WORKLOADS, make_inputs

    w = WORKLOADS[op]
    dev = torch.device("cuda:0")
    shapes = {}
    for nm, shape, _ in w.inputs:
        if op in ("matmul", "matmul_transposed_a", "matmul_symmetric"):
            if frac < 1.0:
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


# ----------------------------------------------------------------- exchange sweep
def exchange_sweep(iters: int, sink=None) -> int:
    """Per-call cost of the cross-GPU step of the sharded ops under torchrun:
    the library's peer-memory all-reduce (kbb200.p2p.PeerComm) against
    NCCL's all_reduce at the payloads the sharded ops exchange, plus the
    fused split-K fold + peer all-reduce against a local split reduction
    followed by NCCL.  Device time per call with CUDA events over `iters`
    back-to-back calls after warm-up, max over ranks; NVLS off."""
    import datetime

    import torch.distributed as tdist

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    tdist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    from kbb200 import ops
    from kbb200.p2p import PeerComm

    def timed(fn) -> float:
        for _ in range(10):
            fn()
        torch.cuda.synchronize(dev)
        tdist.barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(iters):
            fn()
        s1.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([s0.elapsed_time(s1) * 1e3 / iters], dtype=torch.float64, device=dev)
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        return round(t.item(), 2)

    comm = PeerComm(payload_bytes=1 << 20, timeout_s=10.0, device=dev)
    res = {"world": tdist.get_world_size(), "unit": "us per call", "iters": iters}
    try:
        for label, n, dtype in [("frobenius 8 B", 1, torch.float64),
                                ("mse / cross-entropy 16 B", 2, torch.float64),
                                ("batchnorm C=128 2 KiB", 257, torch.float64),
                                ("split-K C 256x256 256 KiB", 65536, torch.float32)]:
            t = torch.randn(n, dtype=dtype, device=dev)
            res[label] = {"p2p": timed(lambda: comm.all_reduce_(t)),
                          "nccl": timed(lambda: tdist.all_reduce(t))}
        g = torch.Generator(device=dev).manual_seed(0)
        A = torch.randn(256, 1 << 21, device=dev, generator=g)
        B = torch.randn(1 << 21, 256, device=dev, generator=g)
        parts, splits = ops.matmul_splitk_partials(A, B)
        c = torch.empty(256, 256, device=dev)

        def unfused():
            torch.sum(parts, dim=0, out=c)  # stands in for the local split reduction
            tdist.all_reduce(c)

        res[f"split-K fold of {splits} splits + all-reduce"] = {
            "p2p fused": timed(lambda: comm.splitk_all_reduce(parts, splits, c)),
            "torch sum + nccl": timed(unfused)}
        comm.check()
    finally:
        comm.close()
    if tdist.get_rank() == 0:
        if sink is not None:
            sink.emit(json.dumps(res))
        else:
            print(json.dumps(res), flush=True)
    tdist.barrier()
    tdist.destroy_process_group()
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


def _workload_desc(ops: list[str]) -> str:
    from kbb200.workloads import WORKLOADS

    return "; ".join(f"{n} " + " @ ".join("x".join(map(str, s)) for nm, s, _ in WORKLOADS[n].inputs
                                          if nm in ("x", "A", "B", "predictions"))
                     for n in ops)


def _main(sink) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="northstar",
                    help="a family of kbb200.workloads.FAMILIES or a comma-separated op list")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--profile-op", default=None, help="run one op 3x on a reduced input (for ncu)")
    ap.add_argument("--exchange-sweep", action="store_true",
                    help="per-call cost of the peer all-reduce vs NCCL (torchrun, N >= 2)")
    ap.add_argument("--iters", type=int, default=200, help="calls per payload for --exchange-sweep")
    ap.add_argument("--e2e-chunks", type=int, default=8,
                    help="row blocks per op in the end-to-end pipeline (1: whole op, serial)")
    ap.add_argument("--collective", choices=("p2p", "nccl"), default="p2p",
                    help="cross-GPU sum of the sharded ops: the library's peer-memory kernel or NCCL")
    ap.add_argument("--frac", type=float, default=0.25, help="input fraction for --profile-op")
    ap.add_argument("--tf32-sustain-s", type=float, default=3.0,
                    help="seconds of back-to-back cuBLAS TF32 calls for the sustained tensor ceiling "
                         "(0: none, the pool's bf16 sustained / burst ratio instead; for launch lists)")
    a = ap.parse_args()
    if a.profile_op:
        return profile_op(a.profile_op, a.frac)
    if a.exchange_sweep:
        return exchange_sweep(a.iters, sink)
    if a.warmup < 3 and a.impl == "ours":
        a.warmup = 3

    from kbb200.workloads import (EXCHANGE, FAMILIES, SHARED_INPUTS, WORKLOADS, roofline_bound,
                                  roofline_seconds, shard_fraction, shard_shapes)

    ops = FAMILIES[a.workload] if a.workload in FAMILIES else a.workload.split(",")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    metric = ("per-op GB/s or TFLOP/s as a fraction of the B200 roofline, summed as roofline-weighted "
              f"throughput over the {a.workload} step ({len(ops)} ops); vs the torch-eager CPU reference")
    unit = "B200 rooflines"
    config = {"workload": f"{a.workload}: " + _workload_desc(ops),
              "parallelism": (f"strong{world}: each op's global input sharded over {world} ranks "
                              "(rows / batch / slices / GEMM rows / K slices)" if world > 1 else "1 GPU"),
              "value_definition": ("sum over ops of (one-B200 roofline time of the global op) / measured "
                                   "step time (max over ranks); 1.0 = one B200 at every op's roofline")}
    peaks = load_peaks()

    if a.impl == "reference":
        if rank != 0:
            return 0
        _tensor_peak(peaks, None)  # the GPU arm's units; the reference arm touches no GPU
        threads = host_cores()
        r = cpu_reference(ops, max(1, min(a.steps, 5)), min(a.warmup, 1), threads, peaks, budget_s=120.0)
        line = {"metric": metric, "value": r["value"], "unit": unit, "n_gpus": a.gpus,
                "steps": r["steps"], "warmup": min(a.warmup, 1), "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded, tiled 32 MiB blocks)", "config": config, "impl": "reference",
                "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "cpu_gbs": r["gbs"], "peaks": peaks,
                "e2e": {"value": r["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
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
    # library's own kernel (kbb200.p2p) where it is faster, else over NCCL
    comm = None
    if world > 1 and set(EXCHANGE) & set(ops):
        config["collective"] = a.collective
        if a.collective == "p2p":
            from kbb200.p2p import PeerComm

            comm = PeerComm(payload_bytes=1 << 20, timeout_s=10.0, device=device)
    _tensor_peak(peaks, measure_tf32_tflops(device, sustain_s=a.tf32_sustain_s))

    runners = []
    shared: dict[str, list] = {}
    for n in ops:
        w = WORKLOADS[n]
        src = SHARED_INPUTS.get(n)
        if src in shared:
            ins = shared[src][: len(w.inputs)]
        else:
            ins = make_inputs(w, device, seed=1000 * rank + len(runners), shapes=shard_shapes(w, rank, world),
                              global_scale=True)
        shared[n] = ins
        fn, out = make_runner(n, ins, world, rank, comm)
        runners.append((n, w, ins, fn, out))

    def barrier():
        if world > 1:
            torch.distributed.barrier(device_ids=[local_rank])

    # L2 hygiene: between two launches of one op the step moves every op's
    # bytes; a step too small for that gets a flush (a 256 MB write) before
    # every op, outside the per-op events, inside the step time
    step_bytes_rank = sum(w.algo_bytes * shard_fraction(w, rank, world) for _, w, *_ in runners)
    flush_buf = None
    if step_bytes_rank < 4 * L2_BYTES:
        flush_buf = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=device)
        config["l2"] = f"L2 flush ({FLUSH_BYTES >> 20} MB write) before every op: step of {step_bytes_rank / 1e6:.0f} MB"
    else:
        config["l2"] = (f"no flush: each rank moves {step_bytes_rank / 1e9:.2f} GB per step, so between two "
                        "launches of an op gigabytes pass through the 126 MB L2")

    stream = torch.cuda.current_stream(device)
    for _ in range(a.warmup):
        for _, _, _, fn, _ in runners:
            fn()
    torch.cuda.synchronize(device)

    # the step time: K steps with nothing but the ops (and flushes) between
    # one pair of events; then the per-op split in a second pass of K steps
    # with an event pair around every op (events between kernels are
    # commands of their own on the stream, so they stay out of the step time)
    clocks = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize(device)
    clocks.mark(0)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for _ in range(a.steps):
        for _, _, _, fn, _ in runners:
            if flush_buf is not None:
                flush_buf.fill_(1.0)
            fn()
    t_end.record(stream)
    torch.cuda.synchronize(device)
    clocks.mark(1)
    barrier()
    total_ms = t_start.elapsed_time(t_end)
    ev = {n: [] for n, *_ in runners}
    torch.cuda.synchronize(device)
    for _ in range(a.steps):
        for n, _, _, fn, _ in runners:
            if flush_buf is not None:
                flush_buf.fill_(1.0)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            ev[n].append((e0, e1))
    torch.cuda.synchronize(device)
    barrier()
    per_op_ms = {n: sum(e0.elapsed_time(e1) for e0, e1 in ev[n]) / a.steps for n in ev}
    if world > 1:
        t = torch.tensor([total_ms] + [per_op_ms[n] for n in ev], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = t[0].item()
        per_op_ms = {n: t[i + 1].item() for i, n in enumerate(ev)}
    ms_per_step = total_ms / a.steps
    hbm, tens = peaks["hbm_gbs"], peaks["tensor_tflops"]
    roof_s = sum(roofline_seconds(w, hbm, tens) for _, w, *_ in runners)
    value = roof_s / (ms_per_step * 1e-3)

    from kbb200.dist import _fused, peer_path

    per_op = {}
    hbm_bytes = hbm_ms = tf_flops = tf_ms = 0.0
    for n, w, *_ in runners:
        ms = per_op_ms[n]
        bound = roofline_bound(w, hbm, tens)
        d = {"ms": round(ms, 4), "bound": bound, "gbs": round(w.algo_bytes / (ms * 1e-3) / 1e9, 1)}
        if w.flops:
            d["tflops"] = round(w.flops / (ms * 1e-3) / 1e12, 2)
        d["frac"] = round(roofline_seconds(w, hbm, tens) / world / (ms * 1e-3), 4)
        if n in EXCHANGE and world > 1:
            nb = EXCHANGE_BYTES[n](w)
            via = ("fused into the partial kernel (peer memory)" if n in LAUNCHES_FUSED and _fused(comm, nb) else
                   "peer all-reduce kernel" if peer_path(comm, nb) else "NCCL all_reduce")
            d["exchange"] = f"{via}: {EXCHANGE[n]}"
        per_op[n] = d
        if bound == "tensor":
            tf_flops += w.flops
            tf_ms += ms
        else:
            hbm_bytes += w.algo_bytes
            hbm_ms += ms
    # the roofline record covers the op that takes the largest share of the step
    dom_name, dom_w = max(((n, w) for n, w, *_ in runners), key=lambda t: per_op_ms[t[0]])
    dom_ms = per_op_ms[dom_name]
    if roofline_bound(dom_w, hbm, tens) == "tensor":
        achieved = dom_w.flops / (dom_ms * 1e-3) / 1e12
        # a GEMM timed inside the long step runs under the power cap: its
        # denominator is the sustained ceiling; the burst one stays beside it
        sus = peaks.get("tensor_tflops_sustained")
        roof = {"bound": "tensor", "unit": "TFLOP/s", "peak": round((sus or tens) * world, 2),
                "peak_source": (peaks["tensor_sustained_source"] if sus else peaks["tensor_source"])
                + (f" x {world} GPUs" if world > 1 else ""),
                "peak_burst": round(tens * world, 2), "frac_vs_burst": round(achieved / (tens * world), 4),
                "bf16_measured_tflops": peaks["bf16_tflops"]}
    else:
        achieved = dom_w.algo_bytes / (dom_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "unit": "GB/s", "peak": round(hbm * world, 1),
                "peak_source": peaks["source"] + (f" x {world} GPUs" if world > 1 else "")}
    traffic = ncu_traffic(dom_name) if world == 1 else None
    roof.update({"kernel": dom_name, "achieved": round(achieved, 2), "frac": round(achieved / roof["peak"], 4),
                 "traffic": traffic, "algo_bytes": dom_w.algo_bytes, "ms_per_launch": round(dom_ms, 4),
                 "share_of_step": round(dom_ms / ms_per_step, 3)})

    # ---- end to end through the public API with pinned host buffers
    e2e = None
    if not a.no_e2e:
        e2e_fns, h2d, d2h = [], 0, 0
        e2e_streams = E2EStreams(device)
        # ops that read the same input tensor (SHARED_INPUTS) form one group:
        # the input is uploaded once per step and every op of the group runs
        # on each uploaded block
        groups: dict[str, list] = {}
        for n, w, ins, _, out in runners:
            groups.setdefault(SHARED_INPUTS.get(n, n), []).append((n, w, ins, out))
        for lead, members in groups.items():
            n, w, ins, out = members[0]
            hin = []
            for t in ins:
                h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                h.copy_(t)
                hin.append(h)
            houts, extra = [], []
            for m_name, m_w, m_ins, m_out in members:
                hout = torch.empty(m_out.shape, dtype=m_out.dtype, pin_memory=True)
                houts.append(hout)
                d2h += bytes_of([hout])
                if m_name != n:
                    fwd = (_dist_forward(m_name, comm) if world > 1 and m_name in EXCHANGE
                           else load_candidate(m_w.problem).Model().to(device))
                    extra.append((fwd, len(m_ins), hout))
            fwd = None
            chunks = a.e2e_chunks
            if world > 1 and n in EXCHANGE:  # the sharded op with its exchange, whole
                fwd = _dist_forward(n, comm)
                chunks = 1
            e2e_fns.append(e2e_runner(n, w.problem, hin, houts[0], device, chunks, e2e_streams,
                                      dev_in=ins, forward=fwd, extra=extra))
            h2d += bytes_of(hin)
        e2e_streams.begin()
        for f in e2e_fns:
            f()
        e2e_streams.end()
        torch.cuda.synchronize(device)
        e2e_steps = max(1, min(a.steps, a.e2e_steps))
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
        e2e = {"value": round(roof_s / (e2e_ms * 1e-3), 6), "unit": unit,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
               "steps": e2e_steps, "gbs_algorithmic": round(sum(w.algo_bytes for _, w, *_ in runners)
                                                            / (e2e_ms * 1e-3) / 1e9, 2),
               "pipeline": (f"{a.e2e_chunks} row blocks per row-independent op: H2D, candidate "
                            "Model.forward, D2H on three streams; ops with a global result whole; an input "
                            "read by several ops of the step (x of sum/mean/argmax, of LayerNorm/RMSNorm, "
                            "of softmax/log-softmax) uploaded once" if a.e2e_chunks > 1 else "serial")}
        del e2e_fns, groups

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_reference(ops, a.cpu_steps, 1, host_cores(), peaks, budget_s=60.0)
        cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample", "gbs", "ms_per_step")}

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
        "metric": metric, "value": round(value, 4), "unit": unit, "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, generated on device)", "config": config,
        "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
        # kernels of ours in the timed step loop (the per-op pass after it runs as many again)
        "gpu_launches": a.steps * sum(launches(n, world, comm, ins) for n, _, ins, _, _ in runners),
        "peaks": peaks,
        "aggregate": {"hbm_ops_gbs": round(hbm_bytes / (hbm_ms * 1e-3) / 1e9, 1) if hbm_ms else None,
                      "hbm_ops_frac": round(hbm_bytes / (hbm_ms * 1e-3) / 1e9 / (hbm * world), 4) if hbm_ms else None,
                      "tensor_ops_tflops": round(tf_flops / (tf_ms * 1e-3) / 1e12, 2) if tf_ms else None,
                      "tensor_ops_frac": round(tf_flops / (tf_ms * 1e-3) / 1e12 / (tens * world), 4) if tf_ms else None},
        "per_op": per_op,
        "impl": "ours",
    }
    sink.emit(json.dumps(line))
    return 0


def _dist_forward(name: str, comm):
    """The sharded op with its exchange as a forward(inputs) -> output for
    the end-to-end pipeline (public API: kbb200.dist)."""
    from kbb200 import dist

    if name == "mse_loss":
        return lambda a, b: dist.mse_loss(a, b, comm=comm)
    if name == "frobenius_normalize":
        return lambda x: dist.frobenius_normalize(x, comm=comm)
    if name == "batch_norm_train":
        return lambda x, w, b: dist.batch_norm_train(x, w, b, comm=comm)
    if name == "matmul_splitk":
        return lambda A, B: dist.matmul_splitk(A, B, comm=comm)
    if name == "cross_entropy":
        return lambda lg, tg: dist.cross_entropy(lg, tg, comm=comm)
    raise KeyError(name)


if __name__ == "__main__":
    sys.exit(main())
