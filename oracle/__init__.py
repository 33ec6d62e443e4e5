"""CPU oracle of the ouroboros-kernelsmith op suite — TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this package, and only as the checker or the timed CPU
baseline.  The product package (b200k) never imports it: every b200k op runs
its CUDA kernel or raises.
"""
from . import numerics, ops, regimes  # noqa: F401
