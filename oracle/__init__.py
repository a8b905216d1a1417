"""CPU oracle for the TensorLang execution path -- TEST INFRASTRUCTURE ONLY.

This package restates, in NumPy, what the TensorLang reference computes for a
lowered program: the per-op kernel semantics of
``tensorlang/kernel_generator.py``, the execution phases of
``tensorlang/compiler.py`` (``compile_and_execute`` and ``_execute_for_loop``)
and the reverse-mode rules of ``tensorlang/autograd.py``.  It runs in float64
(the correctness oracle) or float32 (the reference's own arithmetic width; the
timed CPU baseline).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs may import it.  The GPU backend never calls into it.

Parity status: pinned.  ``tests/test_oracle_golden.py`` checks this oracle
against every ``// @EXPECTED`` block of the reference's 106 test programs and
against every tensor the reference's own executor produced for them
(``tests/golden/ref_programs.json``), and checks the autograd restatement
against gradients from the reference's ``ComputationGraph``
(``tests/golden/autograd_cases.json``).
"""
from .tl_oracle import (  # noqa: F401
    OracleProgram,
    SEMANTICS_EXTENSIONS,
    op_forward,
    infer_shape,
)
