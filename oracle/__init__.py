"""CPU oracle for the fused EM path -- test infrastructure, never the product.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs
import this package, and only as the checker / the timed CPU reference.
"""
