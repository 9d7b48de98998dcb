"""CPU oracle for the quantized-matvec decode path (test infrastructure only).

This package restates, in numpy and plain C, the arithmetic of the reference
AuraTensor Java engine for the decode hot path. It exists to CHECK the CUDA
implementation in ``auratensor_b200``: only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import
it. The product library never calls into this package.

Parity pin: the reference is Java and no JDK exists where this was written, so
the restatement is pinned against the known-answer tests the reference's own
JUnit suite holds for this path (fp16 decode, Q4_0 nibble order, kernel
formulas, sampler cases) via the fixtures under ``tests/golden/``. Full-model
logits have no reference-side golden vector ("parity unpinned" for the
whole forward pass beyond those KATs).
"""
