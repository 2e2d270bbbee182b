"""CPU oracle for the flicker DiT attention hot path (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this package, and only as a checker or as the timed
CPU baseline. The product path (``flicker_b200``) never imports it.
"""
