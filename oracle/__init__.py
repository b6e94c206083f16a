"""CPU oracle for the sequence-loss path (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this package. The shipped library never does.
"""
