"""The reference's evaluation protocol, restated for the tests.

- static_check: the AST rules of harness/antihack.py:18-65 (S1 forward calls
  the declared entry, S2 no compile/stream/event/graph/synchronize calls in
  forward, S3 no harness imports).
- build_candidate: exec a candidate file with the restricted globals of
  harness/eval_protected.py:286-300 and return (Model, ENTRY).
- parity_trials: seeds 0-4, fresh seeded inputs per seed, shape match and
  allclose, R1 input-immutability hashes and the R2 seed-0 recompute digest
  (harness/eval_protected.py:338-411, :316-335).
"""
from __future__ import annotations

import ast
import hashlib
import math
import re
from pathlib import Path

import torch

CANDIDATES = Path(__file__).resolve().parent.parent / "kernelbench-hip_b200" / "candidates"

BANNED_CALLS = {"compile", "Stream", "Event", "graph", "CUDAGraph", "make_graphed_callables",
                "set_stream", "current_stream", "synchronize"}
BANNED_MODULES = {"kernelbench", "harness", "eval_protected", "runner", "antihack", "problems"}


def candidate_path(problem: str) -> Path:
    return CANDIDATES / problem / "b200.py"


def candidate_entry(src: str) -> str:
    m = re.search(r'^ENTRY\s*=\s*["\']([\w]+)["\']', src, re.M)
    return m.group(1) if m else ""


def static_check(src: str, entry_symbol: str) -> dict:
    violations = []
    tree = ast.parse(src)
    forward = None
    for node in ast.walk(tree):
        if isinstance(node, ast.ClassDef) and node.name == "Model":
            for item in node.body:
                if isinstance(item, ast.FunctionDef) and item.name == "forward":
                    forward = item
        if isinstance(node, (ast.Import, ast.ImportFrom)):
            names = [a.name for a in node.names] if isinstance(node, ast.Import) else [node.module or ""]
            for m in names:
                if any(m == b or m.startswith(b + ".") for b in BANNED_MODULES):
                    violations.append(f"S3 imports harness module: {m}")
    if forward is None:
        return {"ok": False, "violations": violations + ["S1 no Model.forward found"]}
    calls = []
    for node in ast.walk(forward):
        if isinstance(node, ast.Call):
            f = node.func
            name = f.attr if isinstance(f, ast.Attribute) else getattr(f, "id", "")
            calls.append(name)
            if name in BANNED_CALLS:
                violations.append(f"S2 banned call in forward: {name}()")
    if not any(entry_symbol in c for c in calls):
        violations.append(f"S1 forward never calls the entry '{entry_symbol}'")
    return {"ok": not violations, "violations": violations}


def build_candidate(src: str):
    import torch.nn as nn

    g = {"__builtins__": __builtins__, "torch": torch, "nn": nn, "math": math}
    exec(compile(src, "<candidate>", "exec"), g)
    if "Model" not in g:
        raise RuntimeError("candidate defines no Model")
    return g["Model"], g.get("ENTRY", "")


_DEVICE_HASH_MIN_BYTES = 64 << 20
_HASH_CHUNK = 1 << 24  # 32-bit words per chunk (64 MB)


def hash_tensor(t: torch.Tensor) -> str:
    """R1 input fingerprint.  Host tensors and small device tensors: sha256
    of the bytes, as the reference's protected eval does.  Device tensors of
    64 MB and more (benchmark shapes reach 8 GB, whose host copy and sha256
    dominated a sweep) are fingerprinted on the device instead: per 64 MB
    chunk of 32-bit words w_i, sum(w_i), sum(w_i * (i + 1)) and
    sum(w_i XOR (w_i >> 11)) in wrapping int64, then sha256 of those sums.
    Any single changed word changes the position-weighted sum."""
    t = t.detach()
    nbytes = t.numel() * t.element_size()
    if not t.is_cuda or nbytes < _DEVICE_HASH_MIN_BYTES or nbytes % 4:
        return hashlib.sha256(t.cpu().contiguous().numpy().tobytes()).hexdigest()[:16]
    return word_fingerprint(t.contiguous().view(-1).view(torch.int32), str((tuple(t.shape), t.dtype)))


def word_fingerprint(words: torch.Tensor, tag: str = "", chunk: int = _HASH_CHUNK) -> str:
    """Chunked position-weighted checksum of int32 `words` (any device)."""
    idx = torch.arange(1, chunk + 1, device=words.device, dtype=torch.int64)
    sums = []
    for part in words.split(chunk):
        w = part.to(torch.int64)
        sums += [w.sum(), (w * idx[: w.numel()]).sum(), (w ^ (w >> 11)).sum()]
    host = torch.stack(sums).cpu().numpy().tobytes()
    return hashlib.sha256(host + tag.encode()).hexdigest()[:16]


def digest(t: torch.Tensor) -> list:
    return [tuple(t.shape), t.numel(), f"{t.min().item():.6e}", f"{t.max().item():.6e}"]


def digest_close(d1: list, d2: list) -> bool:
    if d1[:2] != d2[:2]:
        return False
    lo1, hi1, lo2, hi2 = float(d1[2]), float(d1[3]), float(d2[2]), float(d2[3])
    tol = 1e-4 * max(1e-30, hi1 - lo1, hi2 - lo2)
    return abs(lo1 - lo2) <= tol and abs(hi1 - hi2) <= tol
