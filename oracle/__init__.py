"""TEST INFRASTRUCTURE ONLY -- the CPU oracle of the tree-attention path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg (and its ``--impl reference`` arm) import this package, always as the
checker or the timed CPU baseline, never as part of the product path.  The
product (``tree-attention-scheduling_b200/tree_attention``) never imports it.

Parity pins: the functions here are checked against golden vectors generated
from the reference implementation itself (``tests/golden/make_golden.py``
imports the reference's own ``src/tree_attention`` and records its outputs),
see ``tests/test_oracle.py``.
"""
