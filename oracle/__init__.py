"""Test oracle for the PyFlameRT MatMul/Gemm/QuantizedMatMul/SpMM hot path.

TEST INFRASTRUCTURE ONLY: a CPU restatement of the reference's arithmetic
(oracle.c) and the reference's own sources compiled into oracle/_ref.  Only
tests/, __graft_entry__.smoke() and bench.py's CPU baseline use it; the
product path never imports it.
"""
