"""CPU parity oracle for the Sinkhorn hot path (test infrastructure only).

Importable by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py``; the product package never imports it.
"""
