"""CPU oracle of the memory-layer hot path.

TEST INFRASTRUCTURE: imported only by ``tests/``, ``__graft_entry__.smoke``
and the CPU-baseline legs of ``bench.py``, as the checker.  The product
(``model_b200``) never imports it and has no CPU fallback.
"""
