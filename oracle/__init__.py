"""Test-only CPU oracle for the sparse-MLA forward (see ``oracle/sparse_mla.py``).

Nothing in the shipped package imports this; it is the checker for tests,
``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``.
"""
