"""CPU oracle for the gated-delta path (test infrastructure only).

Importable only from ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg, as the checker. The product package
``gdn_b200`` never imports it.
"""
