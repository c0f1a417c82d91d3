"""CPU oracle for minitp_b200's parity tests and CPU baseline (test infrastructure only).

This package restates, on the CPU, the reference algorithm of mini-TP's
tensor-parallel decode path (WJX3078/mini-tp v0.4, package ``minitp``). TP
is emulated in one process: each rank's shard computes its partial and the
partials are summed in rank order. Every function cites the reference
file:line it follows.

It is NOT part of the product. Only ``tests/``, ``__graft_entry__.smoke()``
(as the checker) and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it. The minitp_b200 package never imports it and
fails loudly instead of falling back to it.

Parity pin: ``tests/test_oracle_golden.py`` checks this oracle against
fixtures recorded from the reference itself (``tests/golden/make_golden.py``
imports the unmodified reference and records its outputs).
"""
