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
import os
import sys
from pathlib import Path

import pytest
import torch

from oracle import problems
from tests.protocol import build_candidate, candidate_entry, candidate_path, static_check

# a checkout of the reference (read-only); the tests that run its own harness
# code skip where there is none
REF_ROOT = Path(os.environ.get("KBB200_REFERENCE_DIR", "/root/reference"))
REF_ANTIHACK = REF_ROOT / "harness" / "antihack.py"
REF_EVAL = REF_ROOT / "harness" / "eval_protected.py"


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


@pytest.fixture(scope="module")
def reference_eval():
    """The reference's protected eval module, unmodified (its import pulls in
    its own antihack and problems modules from the same directory)."""
    if not REF_EVAL.exists():
        pytest.skip("reference checkout not present")
    saved = list(sys.path)
    spec = importlib.util.spec_from_file_location("_ref_eval_protected", REF_EVAL)
    mod = importlib.util.module_from_spec(spec)
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.path[:] = saved
    return mod


@pytest.mark.parametrize("name", problems.SUBSET)
def test_reference_eval_builds_candidate(name, reference_eval):
    """The reference eval's own candidate handling (harness/eval_protected.py:
    _candidate_entry :259-263, antihack.static_check :150-159, build_candidate
    :286-300 with its restricted globals) accepts every candidate, and the
    Model it returns constructs from the problem's init inputs.  The timed
    GPU part of evaluate() pins cuda:0 and is not run here (no GPU)."""
    src = candidate_path(name).read_text()
    entry = reference_eval._candidate_entry(src)
    assert entry and entry == candidate_entry(src)
    assert reference_eval.antihack.static_check(src, entry)["ok"]
    Model, e2 = reference_eval.build_candidate(src)
    assert e2 == entry
    _, _, get_init_inputs, _ = problems.load_problem(name)
    assert isinstance(Model(*get_init_inputs()), torch.nn.Module)


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


def _lib_symbols_of_entry(entry: str) -> set[str]:
    """The C-ABI symbols an ENTRY of kbb200.ext reaches: the kbb200.ops
    functions its body calls, and the LIB.kb_* functions (or "kb_*" names
    passed to getattr(LIB, ...)) those bodies call — read from the sources'
    syntax trees, so no GPU is needed."""
    import ast

    pkg = Path(__file__).resolve().parent.parent / "kernelbench-hip_b200" / "kbb200"

    def funcs(path):
        tree = ast.parse(path.read_text())
        return {n.name: n for n in tree.body if isinstance(n, ast.FunctionDef)}

    ext_f, ops_f = funcs(pkg / "ext.py"), funcs(pkg / "ops.py")

    def ops_called(fn):
        out = set()
        for n in ast.walk(fn):
            if isinstance(n, ast.Call) and isinstance(n.func, ast.Attribute) and \
                    isinstance(n.func.value, ast.Name) and n.func.value.id == "ops":
                out.add(n.func.attr)
        return out

    def lib_syms(name, seen):
        if name in seen or name not in ops_f:
            return set()
        seen.add(name)
        out = set()
        for n in ast.walk(ops_f[name]):
            if isinstance(n, ast.Attribute) and isinstance(n.value, ast.Name) and n.value.id == "LIB":
                out.add(n.attr)
            if isinstance(n, ast.Constant) and isinstance(n.value, str) and n.value.startswith("kb_"):
                out.add(n.value)
            if isinstance(n, ast.Call) and isinstance(n.func, ast.Name) and n.func.id in ops_f:
                out |= lib_syms(n.func.id, seen)
        return out

    def direct(fn):  # LIB.kb_* used (or named) in the function's own body
        out = set()
        for n in ast.walk(fn):
            if isinstance(n, ast.Attribute) and isinstance(n.value, ast.Name) and n.value.id == "LIB":
                out.add(n.attr)
            if isinstance(n, ast.Constant) and isinstance(n.value, str) and n.value.startswith("kb_"):
                out.add(n.value)
        return out

    def ext_syms(name, seen):
        if name in seen or name not in ext_f:
            return set()
        seen.add(name)
        fn = ext_f[name]
        out = direct(fn)
        for o in ops_called(fn):
            out |= lib_syms(o, set())
        for n in ast.walk(fn):  # entries that delegate to another entry
            if isinstance(n, ast.Call) and isinstance(n.func, ast.Name) and n.func.id in ext_f:
                out |= ext_syms(n.func.id, seen)
        return out

    return ext_syms(entry, set())


@pytest.mark.parametrize("name", problems.SUBSET)
def test_entry_reaches_exported_c_abi_symbols(name):
    """Every candidate's ENTRY resolves, through kbb200.ext and kbb200.ops, to
    compute entries of the C ABI that include/kbb200.h declares and
    libkbb200.so exports (not to a torch fallback)."""
    import subprocess

    from kbb200 import _lib

    entry = candidate_entry(candidate_path(name).read_text())
    syms = {s for s in _lib_symbols_of_entry(entry) if not s.endswith("_workspace_size")}
    assert syms, f"{entry} reaches no kb_* compute entry"
    header = (Path(__file__).resolve().parent.parent / "include" / "kbb200.h").read_text()
    exported = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                              text=True, check=True).stdout.split()
    for s in syms:
        assert s in exported, f"{entry} -> {s} is not exported by libkbb200.so"
        assert f" {s}(" in header, f"{entry} -> {s} is not declared in include/kbb200.h"
