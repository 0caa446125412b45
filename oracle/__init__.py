"""CPU oracle for parity tests -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs may import this package; the product never does.
"""
from .layer_stack import attention, block, forward

__all__ = ["attention", "block", "forward"]
