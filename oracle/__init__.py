"""Test infrastructure only: the CPU checker for the GEMM operator family.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this package, and only as the checker (or the timed CPU baseline) — never as
the product path.
"""
