"""CPU oracle for the VQ-MoE expert layer (test infrastructure only).

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline legs
import this package; the product path never does.
"""
