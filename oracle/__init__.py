"""Test infrastructure: the CPU oracle for the decode-attention path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this package, and only as the checker or the timed CPU baseline; the
product package never does.
"""
