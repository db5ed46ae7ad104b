"""CPU oracle for the spmd-dialect hot path -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as
the checker.  The product (spmd-dialect_b200/) never imports it.
"""
from .oracle import *  # noqa: F401,F403
