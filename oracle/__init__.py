"""CPU oracle for the ZoomKV sparse decode-attention hot path.

TEST INFRASTRUCTURE ONLY.  tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py use it as the checker;
the product package never imports it.
"""
from .oracle import *  # noqa: F401,F403
