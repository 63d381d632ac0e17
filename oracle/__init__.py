"""CPU oracle for the MoE verification path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package, and only as the checker or the timed CPU
baseline.  The product package ``specfit_b200`` never imports it.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against golden vectors produced by the SpecFit reference itself (see
``tests/golden/make_golden.py``).
"""
