"""CPU oracle for the sampling path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may import
this package.  The product (tinygpt_b200) never does.
"""
