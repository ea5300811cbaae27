"""CPU oracle for the AWQ W4A16 path: test infrastructure only, never the product.

Importable only from ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline and reference legs.
"""
