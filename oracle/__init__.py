"""CPU oracle for the attention-forward hot path (test infrastructure only).

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs.
"""
