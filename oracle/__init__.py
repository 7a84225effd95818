"""Test infrastructure: the CPU restatement of the reference Oracle (see oracle.py).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm use this package.
"""
