"""CPU oracle — TEST INFRASTRUCTURE ONLY.

A restatement of the reference's CPU IR evaluator (test/_eval.ts) and of the
per-step worker logic around it. Imported only by ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg, as the checker
or the timed CPU baseline; nothing under ``tensorgrad_b200/`` imports it.
"""
