"""CPU oracle for the bound-propagation path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of vibecheck's batched bound kernels and input-split BaB
driver, each function citing the reference ``file:line`` it follows.  It is
the checker for the CUDA path: only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may use
it.  The product package never imports it.

Parity of this restatement is pinned against golden vectors produced by the
reference itself (``tests/golden/make_golden.py`` imports the reference's
Python sources and records its outputs; ``tests/test_oracle_golden.py``
checks this module against them).
"""
