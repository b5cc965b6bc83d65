"""Oracle: CPU restatement of the reference's NumPy verifier.

Test infrastructure only: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the kernel library or the tuner.
"""
