"""CPU checker for the affine 4-bit weight-product path (test infrastructure only).

See oracle/oracle.py. Nothing in the product package imports this package.
"""
