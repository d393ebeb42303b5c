"""lastkv_b200 - B200 (sm_100a) kernels for LastKV's shared last-layer KV attention.

The hot path is attention against one shared final-layer K/V history plus a
bounded per-layer ring (the merged paged pool of the reference's vLLM fast
path).  Kernels live in ``csrc/`` and are reached through the C ABI declared
in ``include/lastkv_b200.h``; this package is the thin Python host side.
"""

from .contract import PAGE_SIZE, RMarinBackendContractError  # noqa: F401

__all__ = ["PAGE_SIZE", "RMarinBackendContractError"]
