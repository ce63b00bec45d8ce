"""TEST INFRASTRUCTURE: the CPU oracle for the GEMM path and the reference arm's loader.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and reference legs.
"""
