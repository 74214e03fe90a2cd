"""ORACLE - TEST INFRASTRUCTURE ONLY.

CPU restatement (h3_oracle.c + oracle.py) of the reference's INT8 linear path
arithmetic, used by tests/, __graft_entry__.smoke() and bench.py's CPU baseline as
the checker.  The product (the h3tp package and libh3b200.so) never imports it.
"""
