"""Test infrastructure: the CPU oracle of the quantized-matmul hot path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package; the product (libnxq.so and the nxq binding) never does.
"""
