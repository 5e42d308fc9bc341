"""CPU oracle for the Maba v2 hot path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference algorithms (each function cites the
reference file:line it follows).  It is the checker: ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` may call
it; the product path (``maba_v2_architecture_b200``) never imports it and has no
CPU fallback.

Pinning: ``tests/test_oracle_golden.py`` checks every function here against the
golden vectors in ``tests/golden/`` that ``tests/golden/make_golden.py``
produced by running the reference implementation itself.
"""
