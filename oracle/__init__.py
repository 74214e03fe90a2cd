"""ORACLE - TEST INFRASTRUCTURE ONLY.

CPU restatement (h3_oracle.c + oracle.py) of the reference's INT8 linear path
arithmetic, used by tests/, __graft_entry__.smoke() and bench.py (its CPU baseline,
its reference arm and the sampled-row check after the timed region) as the checker.
tilelang_ref.py builds the reference's own TileLang kernels into _ref/ for the GPU
parity tests.  The product (the h3tp package and libh3b200.so) never imports either.
"""
