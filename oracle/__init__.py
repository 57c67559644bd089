"""CPU oracle for the mrun quantized decode hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (and torch on CPU where the reference itself computes with
torch), the reference algorithms that the B200 kernels replace. Each function cites the
reference file:line it follows (paths inside the mrun project, JHollenb/mrun-pub v0.1.2).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it, and only as the checker or the timed CPU baseline. The product path
(``mrun_b200``) never imports it and has no CPU fallback.

Pinning: ``tests/test_oracle_golden.py`` checks these functions against golden vectors
produced by the reference itself (``tests/golden/make_golden.py``, run where the reference
source is importable) and against the reference's own known-answer tests.
"""
