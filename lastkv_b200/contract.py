"""Fail-closed runtime contract of the shared last-layer KV path.

Mirrors the reference's envelope
(vllm/src/lastkv/vllm/backends/rmarin_flashinfer/runtime_contract.py:27-168):
block (page) size 16, chunk sizes dividing into pages, bf16 only, and a
single exception type for every violation.
"""

from __future__ import annotations

PAGE_SIZE = 16
SUPPORTED_CHUNK_SIZES = frozenset({16, 32, 64, 128, 256, 512, 1024, 2048, 4096})
SUPPORTED_HEAD_DIMS = frozenset({64, 128})
SUPPORTED_GQA_GROUPS = frozenset({1, 2, 4, 8})


class RMarinBackendContractError(RuntimeError):
    """Raised when a call could silently violate the recurrent semantics."""


def require_chunk_size(chunk: int) -> int:
    if isinstance(chunk, bool) or not isinstance(chunk, int) or chunk < PAGE_SIZE or chunk % PAGE_SIZE:
        raise RMarinBackendContractError(f"chunk_size must be a positive multiple of {PAGE_SIZE}, got {chunk!r}")
    return chunk


def require_heads(num_q_heads: int, num_kv_heads: int, head_dim: int) -> int:
    if head_dim not in SUPPORTED_HEAD_DIMS:
        raise RMarinBackendContractError(f"head_dim must be one of {sorted(SUPPORTED_HEAD_DIMS)}, got {head_dim}")
    if num_kv_heads < 1 or num_q_heads % num_kv_heads:
        raise RMarinBackendContractError("num_attention_heads must be divisible by num_key_value_heads")
    group = num_q_heads // num_kv_heads
    if group not in SUPPORTED_GQA_GROUPS:
        raise RMarinBackendContractError(f"GQA group {group} not in {sorted(SUPPORTED_GQA_GROUPS)}")
    return group
