"""Parity checker for the B200 MoE layer (test infrastructure, never shipped).

Only tests/, __graft_entry__.smoke() and bench.py's CPU arm import this package.
"""
from . import moe_oracle  # noqa: F401
