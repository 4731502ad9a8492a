"""``import dsa`` for callers of CHNJZ/dsa (its dsa/__init__.py:2-5).

The reference's package exports ``forward``, ``Tuning``, ``CASE_SHAPES`` and
``SELECTED``; this module gives the same names from the B200 library, so
``import dsa; dsa.forward(q, kv, q_rope, k_rope, indices)`` runs the sm_100a
kernels unchanged. Everything else of ``dsa_b200`` is reachable here too.
"""
from dsa_b200 import *  # noqa: F401,F403
from dsa_b200 import CASE_SHAPES, SELECTED, Tuning, forward

__all__ = ["forward", "Tuning", "CASE_SHAPES", "SELECTED"]
