"""GPU: the strict eval (tests/eval_b200.py) runs every candidate through the
reference's protocol at small shapes and every verdict reaches milestone >= 1
(parity 5/5 at both the reference's 1e-2 and the op's own tolerance, R1, R2);
the milestone table renders from those verdicts."""
from __future__ import annotations

import pytest

from oracle import problems

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", problems.SUBSET)
def test_eval_small(name, cuda_device, tmp_path):
    from tests.eval_b200 import evaluate

    v = evaluate(name, str(tmp_path / f"{name}.json"), small=True, trials=5, with_cpu=False)
    assert v["static_check"]["ok"], v["static_check"]
    assert v["parity"]["parity"], v["parity"]
    assert v["milestone"] >= 1, v.get("why")


def test_milestone_table(cuda_device, tmp_path):
    from tests.eval_b200 import evaluate
    from kbb200.milestone_table import load, markdown, rows

    for name in ("19_ReLU", "40_LayerNorm"):
        evaluate(name, str(tmp_path / f"{name}.json"), small=True, trials=3, with_cpu=False)
    md = markdown(rows(load(str(tmp_path))))
    assert "19_ReLU" in md and "40_LayerNorm" in md
