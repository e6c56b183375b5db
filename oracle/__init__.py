"""CPU oracle of the block-sparse SpMM path (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs import this package, as the checker.  The ``kairo_b200`` package never
does.
"""
