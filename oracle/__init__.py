"""Parity oracle (TEST INFRASTRUCTURE ONLY).

CPU restatements of the reference algorithm on the hot path, plus a harness for
the reference's own kernels rebuilt under ``oracle/_ref/``.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg and the
``--impl reference`` arm) may use anything here, and only as the checker — the
product package never imports this directory.
"""
