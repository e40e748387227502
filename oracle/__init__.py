"""CPU oracle for the multi-LoRA shrink/expand path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package, and only as the checker (or the timed CPU baseline).
The product (``loraforge_b200``) never imports it and has no CPU fallback.

Parity pins: the restatements here are checked against golden vectors generated
from the reference's own test oracles and known answers (``tests/golden/``,
made by ``tests/golden/make_golden.py``), see ``tests/test_oracle_golden.py``.
"""
