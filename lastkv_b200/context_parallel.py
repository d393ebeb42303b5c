"""Context-parallel (sequence-sharded) decode over the shared history.

For very long contexts (the 128K-token case) every sequence's shared
final-layer pages are split into contiguous slices, one per rank; the last
rank also holds the per-layer rings (the previous and current chunk).  Per
layer each rank runs the split-KV decode kernel on its slice in partial mode,
producing a normalised fp32 output and a natural-log LSE per (sequence, query
head); the partials are all-gathered over NCCL and merged exactly with the
LSE-merge kernel, which also applies s_l, so every rank ends with the full
attention output for its replicated O projection and MLP.

The reference has no context parallelism (CP = 1 is enforced,
vllm/src/lastkv/vllm/backends/rmarin_flashinfer/runtime_contract.py:124-133);
the combine is the same exact two-partial merge the reference uses between
its source and local passes (flashinfer_executor.py:185-231), applied to G
partials.  Payload per rank and layer: batch * Hq * (D + 1) * 4 bytes.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from .contract import RMarinBackendContractError


def shard_range(num_items: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous near-even split of ``num_items`` pages over ``world`` ranks."""
    if world < 1 or not 0 <= rank < world:
        raise RMarinBackendContractError("invalid rank / world size")
    base, extra = divmod(num_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass
class ShardPlan:
    """This rank's keys of one sequence: shared pages [p0, p1) and, on the last rank, the ring window."""

    p0: int
    p1: int
    ring_pages: int
    seq_k: int


def plan_shard(nsrc_pages: int, window_tokens: int, page: int, world: int, rank: int) -> ShardPlan:
    p0, p1 = shard_range(nsrc_pages, world, rank)
    last = rank == world - 1
    ring_pages = -(-window_tokens // page) if last else 0
    return ShardPlan(p0, p1, ring_pages, (p1 - p0) * page + (window_tokens if last else 0))


class ContextParallelDecode:
    """Sequence-sharded decode for one process group (NCCL on GPUs, gloo for host tests)."""

    def __init__(self, group=None, *, partial_fn=None, merge_fn=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.partial_fn = partial_fn or self._partial_kernel
        self.merge_fn = merge_fn or self._merge_kernel
        self._bufs = {}

    @staticmethod
    def _partial_kernel(q, pool_k, pool_v, block_table, seq_k, workspace, max_pages):
        return ops.decode_paged(q, pool_k, pool_v, block_table, seq_k, workspace=workspace, max_pages=max_pages,
                                partial=True)

    @staticmethod
    def _merge_kernel(o_all, lse_all, out_scale, out):
        return ops.merge_partials(o_all, lse_all, out_scale=out_scale, out=out)

    def _gather_buffers(self, shape_o, shape_l, device):
        """Concatenated [world * B, ...] receive buffers (the form every backend accepts)."""
        key = (tuple(shape_o), str(device))
        if key not in self._bufs:
            self._bufs[key] = (torch.empty((self.world * shape_o[0], *shape_o[1:]), dtype=torch.float32,
                                           device=device),
                               torch.empty((self.world * shape_l[0], *shape_l[1:]), dtype=torch.float32,
                                           device=device))
        return self._bufs[key]

    def layer(self, q, pool_k, pool_v, block_table, seq_k, *, out_scale=None, out=None, workspace=None,
              max_pages=None):
        """One layer: local partial over this rank's keys, all-gather, exact merge."""
        o, lse = self.partial_fn(q, pool_k, pool_v, block_table, seq_k, workspace, max_pages)
        if self.world == 1:
            o_all, lse_all = o.unsqueeze(0), lse.unsqueeze(0)
        else:
            o_flat, lse_flat = self._gather_buffers(o.shape, lse.shape, o.device)
            self.dist.all_gather_into_tensor(o_flat, o.contiguous(), group=self.group)
            self.dist.all_gather_into_tensor(lse_flat, lse.contiguous(), group=self.group)
            o_all = o_flat.view(self.world, *o.shape)
            lse_all = lse_flat.view(self.world, *lse.shape)
        return self.merge_fn(o_all.contiguous(), lse_all.contiguous(), out_scale, out)
