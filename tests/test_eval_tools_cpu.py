"""CPU: the milestone table renders verdict files, and the strict eval's
static stage rejects a fallback candidate without a GPU."""
from __future__ import annotations

import json


def test_table_from_verdicts(tmp_path):
    from tests.milestone_table import load, markdown, rows

    (tmp_path / "a.json").write_text(json.dumps({
        "problem": "40_LayerNorm", "milestone": 2, "cand_time": {"median_ms": 0.63},
        "eager_time": {"median_ms": 1.9}, "speedup_eager": 3.0, "gbs": 6800.0,
        "roofline_frac": 1.04, "cpu": {"full_ms_estimate": 210.0, "cores": 16}}))
    (tmp_path / "b.json").write_text(json.dumps({"problem": "x", "milestone": -1, "why": "parity failed"}))
    rs = rows(load(str(tmp_path)))
    assert rs[0]["x_cpu"] == round(210.0 / 0.63, 1)
    md = markdown(rs)
    assert "| 40_LayerNorm | 2 |" in md and "| x | -1 |" in md
