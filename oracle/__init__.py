"""CPU oracle (test infrastructure only): a restatement of the reference algorithms used as the checker.

Importable only from tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs.
"""
