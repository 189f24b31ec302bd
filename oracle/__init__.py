"""Checkers for the bitcache B200 kernels -- TEST INFRASTRUCTURE ONLY.

oracle.py: numpy front end of the C restatement (bitcache_oracle.c).
refgpu.py: the reference's own kernels compiled from their sources (oracle/_ref).
build.py:  build recipe for both.
Nothing in the product (bitcache_b200/) imports this package.
"""
