"""CPU: the milestone table renders verdict files, and the strict eval's
static stage rejects a fallback candidate without a GPU."""
from __future__ import annotations

import json


def test_table_from_verdicts(tmp_path):
    from kbb200.milestone_table import load, markdown, rows

    (tmp_path / "a.json").write_text(json.dumps({
        "problem": "40_LayerNorm", "milestone": 2, "cand_time": {"median_ms": 0.63},
        "eager_time": {"median_ms": 1.9}, "speedup_eager": 3.0, "gbs": 6800.0,
        "roofline_frac": 1.04, "cpu": {"full_ms_estimate": 210.0, "cores": 16}, "ngpu": 2}))
    (tmp_path / "b.json").write_text(json.dumps({"problem": "x", "milestone": -1, "why": "parity failed"}))
    rs = rows(load(str(tmp_path)))
    assert rs[0]["x_cpu"] == round(210.0 / 0.63, 1)
    md = markdown(rs)
    # ngpu column: from the verdict, 1 for a single-GPU verdict without it
    assert "| 40_LayerNorm | 2 | 2 |" in md and "| x | 1 | -1 |" in md


def test_word_fingerprint_sees_single_changes_and_swaps():
    """The device-side R1 fingerprint (used for inputs of 64 MB and more)
    changes when one word changes, when two words swap, and across chunks."""
    import torch

    from tests.protocol import word_fingerprint

    g = torch.Generator().manual_seed(0)
    w = torch.randint(-2**31, 2**31 - 1, (10_000,), generator=g, dtype=torch.int32)
    base = word_fingerprint(w, chunk=4096)
    assert word_fingerprint(w.clone(), chunk=4096) == base
    v = w.clone()
    v[7777] ^= 1
    assert word_fingerprint(v, chunk=4096) != base
    v = w.clone()
    v[[10, 5000]] = v[[5000, 10]]
    assert word_fingerprint(v, chunk=4096) != base
    v = w.clone()
    v[[100, 101]] = v[[101, 100]]
    assert word_fingerprint(v, chunk=4096) != base
