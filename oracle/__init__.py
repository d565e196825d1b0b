"""CPU oracle for the selective-scan hot path.

TEST INFRASTRUCTURE ONLY: the checker, never the product.  Only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / reference arm import
this package.  The CUDA library in saccade_v1_b200/ never imports it.
"""
