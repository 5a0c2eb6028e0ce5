"""CPU oracle for the reduce / broadcast hot path: test infrastructure only.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, never by the product
(matrix_b200/).  See oracle/oracle.cpp (the restatement) and oracle/build_ref.py (the reference's own
CPU code, compiled from its tree).
"""
