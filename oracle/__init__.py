"""CPU oracle for Hale-Token's MoE / sampling path (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this package, and only as the checker. The CUDA library never depends on it.
"""
