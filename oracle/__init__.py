"""CPU oracle for tinyvllm's attention hot path -- TEST INFRASTRUCTURE, not product.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm import this package.  The product (``tinyvllm_b200``) never does.

Pinning: the reference (tinygrad) cannot run in this image, so the oracle is
pinned to the reference tests' own known answers and self-consistency checks
(tests/test_oracle.py), not to recorded tinygrad outputs.
"""
