"""CPU oracle of the StarVector decode-sampling step: test infrastructure only.

Imported by tests/, __graft_entry__.smoke() (as the checker) and bench.py's CPU
baseline leg.  Never imported by the product package.
"""
