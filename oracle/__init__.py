"""CPU oracle for the int4 quantized-matmul path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's own algorithm for the hot path
(unpack, per-group dequant, GEMV, GEMM, lm_head argmax, weight-only decoder).
It is the checker: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The product path (``slang_b200``) never calls it and fails loudly when its CUDA
library is missing.

Parity of this restatement is pinned against vectors produced by running the
reference's own functions (``tests/golden/make_golden.py`` imports the
reference's ``gemma4.qat_loader``, ``gemma4.reference`` and
``gemma4_150.kernels_dsl`` sources and writes ``tests/golden/*.npz``), and
against the reference tests' known-answer vectors.
"""
