"""CPU: the bench's host-side pieces — the reference arm maps no library of
this repository, the CPU samples keep the workload's units, and the
roofline units of the value."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def test_reference_arm_maps_no_repo_library():
    """The CPU reference arm (torch-eager models on samples of every op)
    runs without loading libkbb200.so: its ratio against the GPU arm compares
    the reference with this library, not the library with itself."""
    code = f"""
import json, sys
sys.path.insert(0, {str(REPO)!r})
import bench
bench.MIN_SAMPLE_BYTES = 1 << 20      # small samples: a unit test, not a measurement
bench.SAMPLE_FLOPS = 1.0e8
bench.host_llc_bytes = lambda: (1 << 16, "test")
peaks = bench.load_peaks()
bench._tensor_peak(peaks, None)
r = bench.cpu_reference(["relu", "layer_norm", "mse_loss", "matmul"], 1, 0, 2, peaks, budget_s=60)
maps = open("/proc/self/maps").read()
print(json.dumps({{"value": r["value"], "unit": r["unit"], "lib": "libkbb200" in maps, "sample": r["sample"]}}))
"""
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    r = json.loads(out.stdout.strip().splitlines()[-1])
    assert r["lib"] is False, "the reference arm mapped libkbb200.so"
    assert r["value"] > 0 and r["unit"] == "B200 rooflines"
    assert "matmul[" in r["sample"] and "mse_loss[" in r["sample"]


def test_cpu_sample_cuts_the_shard_units():
    sys.path.insert(0, str(REPO))
    import bench
    from kbb200.workloads import WORKLOADS

    shapes, frac = bench.cpu_sample(WORKLOADS["layer_norm"], 256 << 20, 2e11)
    assert shapes["x"] == (4096, 8192) and frac == pytest.approx(4096 / 65536)
    shapes, frac = bench.cpu_sample(WORKLOADS["matmul_splitk"], 256 << 20, 2e11)
    assert shapes["A"][0] == 256 and shapes["B"][1] == 256 and shapes["A"][1] == shapes["B"][0]
    assert frac == pytest.approx(shapes["A"][1] / 4194304)
    shapes, frac = bench.cpu_sample(WORKLOADS["gemv"], 1 << 40, 2e11)
    assert frac == 1.0 and shapes["A"] == (4096, 1048576)


def test_value_units_scale_with_the_gpu_count():
    """The roofline time of an op is the larger of its bytes at the copy
    peak and (contractions) its FLOPs at the 3xTF32 ceiling; N GPUs at the
    same per-GPU speed give N times the one-GPU value."""
    from kbb200.workloads import FAMILIES, WORKLOADS, roofline_bound, roofline_seconds

    hbm, tens = 6448.7, 758.8 / 3
    mm = WORKLOADS["matmul"]
    assert roofline_bound(mm, hbm, tens) == "tensor"
    assert roofline_seconds(mm, hbm, tens) == pytest.approx(2 * 8192 ** 3 / (tens * 1e12))
    gv = WORKLOADS["gemv"]
    assert roofline_bound(gv, hbm, tens) == "hbm"
    roof = sum(roofline_seconds(WORKLOADS[n], hbm, tens) for n in FAMILIES["northstar"])
    assert len(FAMILIES["northstar"]) == 19
    assert 0.015 < roof < 0.02  # ~17.7 ms of one-B200 roofline time per step


def test_tensor_peak_sustained_denominator():
    """The in-step GEMM denominator is the burst 3xTF32 ceiling scaled by the
    live sustained / burst TF32 ratio, else by the pool's bf16 ratio, and is
    never above the burst ceiling."""
    sys.path.insert(0, str(REPO))
    import bench

    peaks = {"hbm_gbs": 6448.7, "bf16_tflops": 1676.2, "bf16_tflops_sustained": 1396.9, "source": "test"}
    bench._tensor_peak(peaks, {"burst": 760.0, "sustained": 608.0, "sustained_calls": 2000})
    burst = bench.TF32_CEILING_TFLOPS / 3.0
    assert peaks["tensor_tflops"] == round(burst, 2)
    assert peaks["tensor_tflops_sustained"] == round(round(burst, 2) * 0.8, 2)
    assert "live cuBLAS TF32" in peaks["tensor_sustained_source"]

    peaks = {"hbm_gbs": 6448.7, "bf16_tflops": 1676.2, "bf16_tflops_sustained": 1396.9, "source": "test"}
    bench._tensor_peak(peaks, None)
    assert peaks["tensor_tflops_sustained"] == round(round(burst, 2) * 1396.9 / 1676.2, 2)

    peaks = {"hbm_gbs": 6448.7, "bf16_tflops": 1676.2, "source": "test"}
    bench._tensor_peak(peaks, {"burst": 700.0, "sustained": 720.0, "sustained_calls": 10})
    assert peaks["tensor_tflops_sustained"] == peaks["tensor_tflops"]
