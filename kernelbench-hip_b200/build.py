"""Build libkbb200.so (the C-ABI operator library) for sm_100a.

Each csrc/*.cu is compiled by nvcc into _build/*.o in parallel, then linked
into kbb200/libkbb200.so with the CUDA runtime linked statically, so the
library needs only the driver at run time.  Rebuilds only what changed
(object older than its source or any header).

    python kernelbench-hip_b200/build.py [--clean] [-j N] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
CSRC = PKG_ROOT / "csrc"
BUILD = PKG_ROOT / "_build"
REPO = PKG_ROOT.parent
INCLUDE = REPO / "include"
LIB = PKG_ROOT / "kbb200" / "libkbb200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(INCLUDE), "-I", str(CSRC),
]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(f"== {src.name}\n{r.stdout}{r.stderr}", file=sys.stderr)
    return obj


def build(jobs: int | None = None, clean: bool = False, verbose: bool = False) -> Path:
    if clean and BUILD.exists():
        shutil.rmtree(BUILD)
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    hdr = _headers_mtime()
    stale = []
    for s in sources:
        o = BUILD / (s.stem + ".o")
        if verbose or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr):
            stale.append(s)
    jobs = jobs or min(len(stale) or 1, os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(lambda s: _compile(s, verbose), stale))
    objs = [BUILD / (s.stem + ".o") for s in sources]
    if stale or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill report")
    a = ap.parse_args()
    lib = build(a.j, a.clean, a.verbose)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
