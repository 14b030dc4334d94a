"""Oracle for the decode / verify path: TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import this package, and only as the checker (or the timed CPU
restatement).  The product library never depends on it.
"""
