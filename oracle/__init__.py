"""Oracle — TEST INFRASTRUCTURE ONLY, never part of the product path.

This package restates, on the CPU, what the reference operator library
computes, so the CUDA kernels can be checked against it:

  oracle.ops       numpy restatement of every op (fp64 internally, results
                   rounded to fp32), each citing the reference kernel it
                   follows.
  oracle.problems  the torch-eager fp32 reference models the reference's
                   protected eval compares candidates against
                   (harness/eval_protected.py:346-375 builds `Model_ref` from a
                   problem file and calls it), restated from the op semantics
                   at the benchmark shapes; the KernelBench problem files the
                   reference loads (harness/problems.py:12) are not vendored.
  oracle.cpu_baseline  times the torch-eager CPU models (the reference's
                   reference arm) on the host cores.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package.  The product (kernelbench-hip_b200/) never does.

Pinning: the reference ships no golden vectors.  tests/golden/make_golden.py
records seeded torch-eager CPU outputs (the reference arm itself) as
fixtures; tests check oracle.ops against them and against the reference's
own hand-checkable cases (argmax ties, NaN, empty inputs).
"""
