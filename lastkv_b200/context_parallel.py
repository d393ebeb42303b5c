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
    """This rank's keys: the last rank holds the ring window, so its shared-page
    share is its even share of all pages minus the ring pages (every rank then
    streams about the same number of pages); the other ranks split the rest."""
    ring = -(-window_tokens // page)
    last_src = nsrc_pages if world == 1 else min(nsrc_pages, max(0, round((nsrc_pages + ring) / world) - ring))
    first = nsrc_pages - last_src
    last = rank == world - 1
    if last:
        p0, p1 = first, nsrc_pages
    else:
        if not 0 <= rank < world:
            raise RMarinBackendContractError("invalid rank / world size")
        p0, p1 = shard_range(first, world - 1, rank)
    return ShardPlan(p0, p1, ring if last else 0, (p1 - p0) * page + (window_tokens if last else 0))


class ContextParallelDecode:
    """Sequence-sharded decode for one process group (NCCL on GPUs, gloo for host tests).

    ``combine`` picks how the ranks' partials (o, lse) meet:

    * ``"p2p"`` (default with more than one CUDA rank): ``lkv_decode_paged_cp``
      - the decode kernel itself, as each (sequence, KV head) finishes, merges
      its splits and pushes the merged rows into every rank's receive buffer
      over NVLink peer memory (torch symmetric memory), so the transfer overlaps
      the rest of the decode; one poll-and-merge launch then combines the ranks
      in rank order - no collective call and no split-merge launch;
    * ``"nccl"``: the decode's partial into one packed send buffer
      [B*Hq*D | B*Hq | pad], one ``all_gather_into_tensor``, then the merge
      kernel over the gathered parts in place.

    Both merge the same partials in the same order (identical outputs).
    ``partial_fn`` and ``merge_fn`` can be injected (host tests) and then use
    separate o / lse tensors over the process group's all-gather.
    """

    def __init__(self, group=None, *, partial_fn=None, merge_fn=None, combine: str | None = None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.injected = partial_fn is not None or merge_fn is not None
        self.partial_fn = partial_fn or self._partial_kernel
        self.merge_fn = merge_fn or self._merge_kernel
        if combine is None:
            combine = "p2p" if self.world > 1 and not self.injected else "nccl"
        if combine not in ("p2p", "nccl"):
            raise RMarinBackendContractError(f"unknown combine {combine!r}")
        if combine == "p2p" and self.injected:
            raise RMarinBackendContractError("the p2p combine runs the CUDA kernels only")
        self.combine = combine
        self._bufs = {}
        self._p2p = {}

    def _p2p_state(self, B, Hq, D, device, Hkv=1):
        """Receive buffers in symmetric memory (allocated and exchanged once per shape)."""
        key = (B, Hq, D, Hkv, str(device))
        st = self._p2p.get(key)
        if st is None:
            import torch.distributed._symmetric_memory as symm

            group = self.group if self.group is not None else self.dist.group.WORLD
            sizes = ops.cp_combine_sizes(B * Hq, D, self.world)
            recv = symm.empty(sizes["recv_words"], dtype=torch.int64, device=device)
            recv.zero_()
            torch.cuda.synchronize(device)
            h_recv = symm.rendezvous(recv, group)
            h_recv.barrier()  # every rank's receive words are zero before anyone pushes
            st = {"recv": recv, "handle": h_recv, "recv_ptrs": [int(x) for x in h_recv.buffer_ptrs],
                  "send": torch.empty(sizes["send_floats"], dtype=torch.float32, device=device),
                  "state": torch.zeros(2, dtype=torch.int32, device=device),
                  "error": torch.zeros(4, dtype=torch.int32, device=device)}
            # fused path: epoch, done counter and per-(sequence, KV head) arrivals
            st["cp_state"] = torch.zeros(ops.decode_cp_state_words(B, Hkv), dtype=torch.int32, device=device)
            self._p2p[key] = st
        return st

    def check_errors(self):
        """Raise if a device-side wait gave up (a peer did not push in time).  The ranks'
        epoch and arrival state is then inconsistent: rebuild this object on every rank
        (fresh, zeroed state and receive buffers) before the next layer call."""
        for st in self._p2p.values():
            e = st["error"].cpu().tolist()
            if e[0]:
                raise RMarinBackendContractError(f"context-parallel combine error word set: {e}")

    @staticmethod
    def _partial_kernel(q, pool_k, pool_v, block_table, seq_k, workspace, max_pages):
        return ops.decode_paged(q, pool_k, pool_v, block_table, seq_k, workspace=workspace, max_pages=max_pages,
                                partial=True)

    @staticmethod
    def _merge_kernel(o_all, lse_all, out_scale, out):
        return ops.merge_partials(o_all, lse_all, out_scale=out_scale, out=out)

    def _buffers(self, key, make):
        if key not in self._bufs:
            self._bufs[key] = make()
        return self._bufs[key]

    def layer(self, q, pool_k, pool_v, block_table, seq_k, *, out_scale=None, out=None, workspace=None,
              max_pages=None, tables_ready=False, l2_keep=False):
        """One layer: local partial over this rank's keys, all-gather, exact merge.
        ``tables_ready`` and ``l2_keep`` as for ``ops.decode_paged``."""
        if self.injected:
            return self._layer_generic(q, pool_k, pool_v, block_table, seq_k, out_scale, out, workspace, max_pages)
        B, Hq, D = q.shape
        if self.combine == "p2p":
            # the decode kernel pushes every unit's merged rows as it finishes; one poll-and-merge launch follows
            st = self._p2p_state(B, Hq, D, q.device, pool_k.shape[2])
            return ops.decode_paged_cp(q, pool_k, pool_v, block_table, seq_k, st["recv_ptrs"], self.rank, self.world,
                                       st["cp_state"], out=out, out_scale=out_scale, workspace=workspace,
                                       max_pages=max_pages, error_word=st["error"], tables_ready=tables_ready,
                                       l2_keep=l2_keep)
        n = -(-(B * Hq * (D + 1)) // 4) * 4  # o | lse | pad to a multiple of 4 floats (float4 reads)
        send, recv = self._buffers(("packed", n, str(q.device)), lambda: (
            torch.empty(n, dtype=torch.float32, device=q.device),
            torch.empty(self.world * n, dtype=torch.float32, device=q.device)))
        o_view = send[: B * Hq * D].view(B, Hq, D)
        l_view = send[B * Hq * D: B * Hq * (D + 1)].view(B, Hq)
        ops.decode_paged(q, pool_k, pool_v, block_table, seq_k, workspace=workspace, max_pages=max_pages,
                         partial=True, partial_out=(o_view, l_view), tables_ready=tables_ready, l2_keep=l2_keep)
        if self.world == 1:
            parts = send.view(1, n)
        else:
            self.dist.all_gather_into_tensor(recv, send, group=self.group)
            parts = recv.view(self.world, n)
        return ops.merge_partials_packed(parts, B, Hq, D, out_scale=out_scale, out=out)

    def _layer_generic(self, q, pool_k, pool_v, block_table, seq_k, out_scale, out, workspace, max_pages):
        o, lse = self.partial_fn(q, pool_k, pool_v, block_table, seq_k, workspace, max_pages)
        if self.world == 1:
            o_all, lse_all = o.unsqueeze(0), lse.unsqueeze(0)
        else:
            o_flat, lse_flat = self._buffers(("split", tuple(o.shape), str(o.device)), lambda: (
                torch.empty((self.world * o.shape[0], *o.shape[1:]), dtype=torch.float32, device=o.device),
                torch.empty((self.world * lse.shape[0], *lse.shape[1:]), dtype=torch.float32, device=o.device)))
            self.dist.all_gather_into_tensor(o_flat, o.contiguous(), group=self.group)
            self.dist.all_gather_into_tensor(lse_flat, lse.contiguous(), group=self.group)
            o_all = o_flat.view(self.world, *o.shape)
            lse_all = lse_flat.view(self.world, *lse.shape)
        return self.merge_fn(o_all.contiguous(), lse_all.contiguous(), out_scale, out)
