"""TEST INFRASTRUCTURE ONLY: CPU oracle of flexkv_b200 (see oracle.c).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs may import this package; the product never does.
"""
