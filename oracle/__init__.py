"""CPU oracle for the algx kernels: test infrastructure, never the product.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package, and only as the checker or the timed CPU
baseline. The shipped code under ``algebraic-extra_b200/`` never calls it.
"""
