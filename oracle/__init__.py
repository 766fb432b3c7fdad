"""CPU checker for the batched geometric-product path (test infrastructure only).

Imported only by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
and reference legs; the product library never uses it.
"""
