"""CPU oracle for the b200fp8 hot path — TEST INFRASTRUCTURE ONLY.

Plain torch-on-CPU restatements of the reference evaluators' own math (the code after
``# === CUTE_HARNESS_EVALUATOR_V1 ===`` in each reference ``tasks/*/starter.py``).  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import this package, and only as the checker or the timed CPU baseline.  The product path
(``b200fp8``) never imports it.

Pinning: ``tests/golden/make_golden.py`` runs the reference evaluators' own code (their
``main()`` functions, executed on CPU with the CUDA-only calls redirected) with these
oracle functions standing in for the candidate kernels; the evaluators' own thresholds
then accept or reject the oracle.  The recorded results live in
``tests/golden/reference_pass.json`` and the small golden vectors in ``tests/golden/*.pt``.
"""
