"""Milestone / roofline table from eval_b200 verdicts (markdown + JSON).

The reference builds results/milestone-table.{md,json} from its verdicts
(scripts/milestone_table.py:27-84); this version adds the B200 columns:
the GPU count of the verdict, GB/s or TFLOP/s of the whole job, fraction of
the measured per-GPU roofline, and the torch-eager CPU estimate with its core
count.

    python -m kbb200.milestone_table verdicts/ [--md out.md] [--json out.json]
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path


def load(dir_: str) -> list[dict]:
    return [json.loads(p.read_text()) for p in sorted(Path(dir_).glob("*.json"))]


def rows(verdicts: list[dict]) -> list[dict]:
    out = []
    for v in verdicts:
        ct, et = v.get("cand_time") or {}, v.get("eager_time") or {}
        cpu = v.get("cpu") or {}
        r = {"problem": v.get("problem"), "ngpu": v.get("ngpu", 1), "milestone": v.get("milestone"),
             "cand_ms": ct.get("median_ms"), "eager_ms": et.get("median_ms"),
             "speedup_eager": v.get("speedup_eager"), "gbs": v.get("gbs"), "tflops": v.get("tflops"),
             "roofline_frac": v.get("roofline_frac"), "cpu_ms": cpu.get("full_ms_estimate"),
             "cpu_cores": cpu.get("cores"), "why": v.get("why")}
        if r["cand_ms"] and r["cpu_ms"]:
            r["x_cpu"] = round(r["cpu_ms"] / r["cand_ms"], 1)
        out.append(r)
    return out


def markdown(rs: list[dict]) -> str:
    head = ("| problem | ngpu | milestone | cand ms | eager ms | x eager | GB/s | TFLOP/s | roofline | "
            "CPU ms (est.) | x CPU |\n|---|---:|---:|---:|---:|---:|---:|---:|---:|---:|---:|\n")
    fmt = lambda x: "" if x is None else str(x)  # noqa: E731
    body = "".join(
        f"| {r['problem']} | {fmt(r['ngpu'])} | {fmt(r['milestone'])} | {fmt(r['cand_ms'])} | "
        f"{fmt(r['eager_ms'])} | "
        f"{fmt(r['speedup_eager'])} | {fmt(r['gbs'])} | {fmt(r['tflops'])} | {fmt(r['roofline_frac'])} | "
        f"{fmt(r['cpu_ms'])} | {fmt(r.get('x_cpu'))} |\n" for r in rs)
    return head + body


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("dir")
    ap.add_argument("--md")
    ap.add_argument("--json")
    a = ap.parse_args()
    rs = rows(load(a.dir))
    md = markdown(rs)
    if a.md:
        Path(a.md).write_text(md)
    if a.json:
        Path(a.json).write_text(json.dumps(rs, indent=1) + "\n")
    print(md)
    return 0


if __name__ == "__main__":
    sys.exit(main())
