"""CPU oracle of the reference's compression path -- test infrastructure only.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs,
never by the bitsparse_b200 package.
"""
