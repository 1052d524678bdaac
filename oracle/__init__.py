"""CPU oracle for tests -- TEST INFRASTRUCTURE ONLY.

Loads ``oracle/_build/libhs_oracle.so`` (the C restatement in hs_oracle.c) and,
when it was built here, ``oracle/_ref/libhs_ref.so`` (the reference's own CPU
code compiled from its sources).  Only tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py import this package, as a checker; the product
path never does.
"""
