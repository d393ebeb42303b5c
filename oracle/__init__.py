"""CPU oracle for the shared last-layer KV attention path (test infrastructure).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import this package, and only as the checker or as the timed
CPU baseline.  The product path (``lastkv_b200``) never imports it.
"""

from . import lastkv_oracle  # noqa: F401
