"""Parity oracle: CPU restatements of the reference's low-bit path (TEST INFRASTRUCTURE ONLY).

Nothing under ``torch-intel-npu_b200/`` imports this package.  Tests, ``smoke()`` and the
CPU-baseline legs of ``bench.py`` use it as the checker and as the timed CPU baseline.
"""
