"""CPU: every candidate keeps the reference's candidate contract.

- ENTRY at column 0 names a function of kbb200.ext (the compiled entry);
- the AST rules of harness/antihack.py pass (restated in tests/protocol.py);
- when the reference checkout is present, its own antihack.static_check
  passes too;
- the candidate builds under the eval's restricted globals and defines Model
  (and the ModelNew alias).
"""
from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

from oracle import problems
from tests.protocol import build_candidate, candidate_entry, candidate_path, static_check

REF_ANTIHACK = Path("/root/reference/harness/antihack.py")


@pytest.mark.parametrize("name", problems.SUBSET)
def test_candidate_contract(name):
    src = candidate_path(name).read_text()
    entry = candidate_entry(src)
    assert entry, "no ENTRY constant"
    import kbb200.ext as EXT

    assert callable(getattr(EXT, entry, None)), f"ENTRY {entry} is not a kbb200.ext entry"
    res = static_check(src, entry)
    assert res["ok"], res["violations"]
    Model, e2 = build_candidate(src)
    assert e2 == entry and Model.__name__ == "Model"


@pytest.mark.skipif(not REF_ANTIHACK.exists(), reason="reference checkout not present")
@pytest.mark.parametrize("name", problems.SUBSET)
def test_reference_antihack_accepts_candidate(name):
    spec = importlib.util.spec_from_file_location("_ref_antihack", REF_ANTIHACK)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    src = candidate_path(name).read_text()
    res = mod.static_check(src, candidate_entry(src))
    assert res["ok"], res["violations"]


def test_static_check_catches_fallbacks():
    src = (
        'ENTRY = "relu_entry"\n'
        "import torch\n"
        "class Model(torch.nn.Module):\n"
        "    def forward(self, x):\n"
        "        torch.cuda.synchronize()\n"
        "        return torch.relu(x)\n"
    )
    v = static_check(src, "relu_entry")["violations"]
    assert any(s.startswith("S1") for s in v) and any(s.startswith("S2") for s in v)


def test_every_problem_has_a_candidate():
    for name in problems.SUBSET:
        assert candidate_path(name).exists(), name
