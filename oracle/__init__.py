"""CPU oracle for the oblivious-tree training path (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this package, and only as the checker or the timed CPU
baseline.  The product (catboost_rs_b200) never imports it.
"""
from .oracle import *  # noqa: F401,F403
