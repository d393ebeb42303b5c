"""B200 form of the reference's vLLM CUSTOM attention backend (merged fast path).

Mirrors, class for class, the serving-side hot path of
vllm/src/lastkv/vllm/backends/rmarin_flashinfer/:

* ``SharedKVPool``       - the merged K/V page pool and its session slots
                           (``RMarinSessionPool._reserve_fused_slabs``,
                           batching.py:1971-2122): shared final-layer pages per
                           slot, one 2C ring per (layer, slot), one scratch page
                           for padded rows, bound per-layer parameters.
* ``SharedKVFastPath``   - ``RMarinDecodeFastPath`` (fastpath.py:32-734): a host
                           prologue per step (``prepare``: boundary commits,
                           per-row plans, index buffers, per-layer block tables)
                           and a static per-layer op sequence (``run_layer``):
                           fused RoPE/QK-norm/V-scale append -> split-KV decode
                           (uniform single-token steps) or tcgen05 prefill
                           (chunk spans), with s_l folded into the epilogue.
* ``SharedKVAttentionImpl`` / ``SharedKVBackend`` - the attention-impl forward
                           signature and backend class surface vLLM binds
                           (vllm_backend.py:637-750).
* ``chunk_aligned_new_tokens`` / ``sliver_deferred_new_tokens`` - the span rules
                           of the chunk-aligned scheduler (batching.py:88-133).

vLLM itself is not imported: this module is the B200 implementation of the
operations the reference's backend performs, with the same buffers and
contracts, for a serving engine to bind.  Everything after ``prepare`` reads
device buffers only and is CUDA-graph capturable.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass

import numpy as np
import torch

from . import ops
from .contract import PAGE_SIZE, RMarinBackendContractError, require_chunk_size, require_heads


def chunk_aligned_new_tokens(num_computed_tokens: int, num_new_tokens: int, chunk_size: int) -> int:
    """Cap a scheduled span at the request's next chunk boundary (batching.py:88-105)."""
    if num_computed_tokens < 0 or chunk_size < 1:
        raise RMarinBackendContractError("chunk_aligned_new_tokens received invalid scheduling state")
    if num_new_tokens < 1:
        return num_new_tokens
    next_boundary = ((num_computed_tokens // chunk_size) + 1) * chunk_size
    return min(num_new_tokens, next_boundary - num_computed_tokens)


def sliver_deferred_new_tokens(num_computed_tokens: int, num_new_tokens: int, chunk_size: int,
                               num_tokens: int) -> int:
    """Chunk-aligned span that waits instead of splitting a chunk (batching.py:108-133)."""
    span = chunk_aligned_new_tokens(num_computed_tokens, num_new_tokens, chunk_size)
    if span < 1:
        return span
    next_boundary = ((num_computed_tokens // chunk_size) + 1) * chunk_size
    reaches = num_computed_tokens + span >= next_boundary
    final = num_computed_tokens + span >= num_tokens
    return span if reaches or final else 0


@dataclass(frozen=True)
class Span:
    """One request's work in a step: ``num_query_tokens`` new tokens from ``num_computed_tokens``."""

    slot: int
    num_computed_tokens: int
    num_query_tokens: int


class SharedKVPool:
    """Merged K/V page pool with per-slot shared pages and per-(layer, slot) rings.

    Page ids: ``[0, pages_per_slot * num_slots)`` shared final-layer pages (raw K,
    raw V; slot s owns ``src_table[s]``), then ``scratch_src_page``; layer l's
    ring region starts at ``ring_base(l)`` and holds ``ring_pages`` pages per slot
    plus one scratch page (batching.py:2005-2013).
    """

    def __init__(self, *, num_layers: int, num_slots: int, max_sequence_tokens: int, chunk_size: int,
                 num_kv_heads: int, head_dim: int, device=None, page_order=None):
        require_chunk_size(chunk_size)
        if head_dim not in (64, 128):
            raise RMarinBackendContractError("head_dim must be 64 or 128")
        self.num_layers, self.num_slots, self.chunk_size = num_layers, num_slots, chunk_size
        self.hkv, self.d = num_kv_heads, head_dim
        self.device = torch.device(device or "cuda")
        self.max_sequence_tokens = max_sequence_tokens
        self.pages_per_slot = -(-max_sequence_tokens // PAGE_SIZE)
        self.padded_tokens = self.pages_per_slot * PAGE_SIZE
        self.scratch_src_page = self.pages_per_slot * num_slots
        self.src_pages = self.scratch_src_page + 1
        self.ring_pages = 2 * chunk_size // PAGE_SIZE
        self.ring_tokens = 2 * chunk_size
        self.ring_stride = self.ring_pages * num_slots + 1
        self.scratch_ring_page = self.ring_pages * num_slots  # layer-relative
        self.num_pages = self.src_pages + num_layers * self.ring_stride
        shape = (self.num_pages, PAGE_SIZE, num_kv_heads, head_dim)
        self.pool_k = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.pool_v = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        n = self.pages_per_slot * num_slots
        order = np.arange(n) if page_order is None else np.asarray(page_order)
        if sorted(order.tolist()) != list(range(n)):
            raise RMarinBackendContractError("page_order must permute the shared pages")
        self.src_table = order.reshape(num_slots, self.pages_per_slot).astype(np.int32)
        self.ring_base_host = self.src_pages + np.arange(num_layers, dtype=np.int64) * self.ring_stride
        self.ring_base_dev = torch.from_numpy(self.ring_base_host.astype(np.int32)).to(self.device)
        self.committed = [0] * num_slots
        self._free = list(range(num_slots))[::-1]
        self.alpha = self.scale = self.inv_scale = self.out_scale = None

    # -- slots
    def acquire(self) -> int:
        if not self._free:
            raise RMarinBackendContractError("no free session slot")
        slot = self._free.pop()
        self.committed[slot] = 0
        return slot

    def release(self, slot: int) -> None:
        self.committed[slot] = 0
        self._free.append(slot)

    # -- parameters (bound after weights load, fastpath.py:254-269)
    def bind_parameters(self, alpha_logits, value_scales, num_q_heads: int) -> None:
        """alpha_logits / value_scales: [L, Hkv]; stored bf16-exact as the pool sees them."""
        a = torch.as_tensor(alpha_logits, dtype=torch.float32).reshape(self.num_layers, self.hkv)
        s = torch.as_tensor(value_scales, dtype=torch.float32).reshape(self.num_layers, self.hkv)
        s = s.to(torch.bfloat16).float()
        if not bool(torch.isfinite(s).all()) or bool((s == 0).any()):
            raise RMarinBackendContractError("value scales must be finite and non-zero for merged attention")
        require_heads(num_q_heads, self.hkv, self.d)
        self.alpha = a.to(torch.bfloat16).sigmoid().float().contiguous().to(self.device)
        self.scale = s.contiguous().to(self.device)
        self.inv_scale = (1.0 / s).contiguous().to(self.device)
        self.out_scale = s.repeat_interleave(num_q_heads // self.hkv, dim=1).contiguous().to(self.device)

    # -- addressing
    def ring_base(self, layer: int) -> int:
        return int(self.ring_base_host[layer])

    def layer_ring_view(self, pool: torch.Tensor, layer: int) -> torch.Tensor:
        """Flat token view [ring_stride * 16, Hkv, D] of layer l's ring region."""
        base = self.ring_base(layer)
        return pool[base:base + self.ring_stride].view(-1, self.hkv, self.d)

    def src_view(self, pool: torch.Tensor) -> torch.Tensor:
        return pool[: self.src_pages].view(-1, self.hkv, self.d)


class SharedKVFastPath:
    """Per-step prologue + per-layer op sequence on the merged pool."""

    NSETS = 4  # rotating pinned staging sets (the host may run ahead of the GPU)

    def __init__(self, pool: SharedKVPool, *, max_batch: int, max_tokens: int, num_q_heads: int,
                 sm_scale: float | None = None):
        self.pool = pool
        self.max_batch = max(1, int(max_batch))
        self.max_tokens = max(self.max_batch, int(max_tokens))
        self.hq = num_q_heads
        require_heads(num_q_heads, pool.hkv, pool.d)
        self.scale = float(sm_scale) if sm_scale is not None else pool.d ** -0.5
        dev, mb, mt = pool.device, self.max_batch, self.max_tokens
        self.W = pool.pages_per_slot + pool.ring_pages
        self.ring_idx = torch.zeros(mt, dtype=torch.int64, device=dev)
        self.src_idx = torch.zeros(mt, dtype=torch.int64, device=dev)
        self.positions = torch.zeros(mt, dtype=torch.int64, device=dev)
        self.cu_q = torch.zeros(mb + 1, dtype=torch.int32, device=dev)
        self.seq_k = torch.ones(mb, dtype=torch.int32, device=dev)
        self.nsrc = torch.zeros(mb, dtype=torch.int32, device=dev)
        self.bt = torch.zeros((mb, self.W), dtype=torch.int32, device=dev)
        # contiguous [L, batch, W] view of this flat buffer per step (batch varies)
        self._bt_all_flat = torch.zeros(pool.num_layers * mb * self.W, dtype=torch.int32, device=dev)
        self.bt_all = self._bt_all_flat.view(pool.num_layers, mb, self.W)
        self.q_out = torch.empty((mt, num_q_heads, pool.d), dtype=torch.bfloat16, device=dev)
        self.error_word = torch.zeros(4, dtype=torch.int32, device=dev)
        # boundary commits of a step: page lists + a device row count read by layer 0's fused
        # append (lkv_rope_norm_append_commit), so captured decode graphs carry them too.
        # fuse_commit False: one blend launch in prepare instead.
        ppc = pool.chunk_size // PAGE_SIZE
        self.c_raw = torch.zeros((mb, ppc), dtype=torch.int32, device=dev)
        self.c_ring = torch.zeros((mb, ppc), dtype=torch.int32, device=dev)
        self.c_count = torch.zeros(1, dtype=torch.int32, device=dev)
        self.fuse_commit = True
        # commit blocks in the fused launch: 0 = one wave of 8 per SM striding over the page
        # items (a step without a boundary pays well under a microsecond for them)
        self.commit_blocks = 0
        self.workspace = ops.Workspace.for_decode(mb, num_q_heads, pool.d, self.W, device=dev)
        pin = torch.cuda.is_available() and dev.type == "cuda"
        def host(shape, dtype):
            t = torch.zeros(shape, dtype=dtype)
            return t.pin_memory() if pin else t
        self._h = [{"ring": host(mt, torch.int64), "src": host(mt, torch.int64), "pos": host(mt, torch.int64),
                    "cu": host(mb + 1, torch.int32), "seqk": host(mb, torch.int32), "nsrc": host(mb, torch.int32),
                    "bt": host((mb, self.W), torch.int32), "craw": host((mb, ppc), torch.int32),
                    "cring": host((mb, ppc), torch.int32), "ccount": host(1, torch.int32)}
                   for _ in range(self.NSETS)]
        # per set: an event recorded after the last copies that read it (None = never used)
        self._h_done = [None] * self.NSETS
        self._set = 0
        self.layers = None
        self.cos_sin = None
        self.batch = self.tokens = self.max_q = 0
        self.uniform = True
        self.active = False
        # RMARIN_MERGED_CHECK=1 (the reference's switch, fastpath.py:199-203): recompute every
        # layer two-pass from the same pool and report the deviation (eager diagnostics only)
        self.check = os.environ.get("RMARIN_MERGED_CHECK") == "1"
        self.check_steps = 0
        self.check_log: list[dict] = []

    def register_layers(self, norm_weights, cos_sin_cache: torch.Tensor, eps: float) -> None:
        """Per-layer (q_norm.weight, k_norm.weight) and the bf16 [max_pos, D] cos|sin cache
        (register_fused_qkv / _bind_fused_qkv, fastpath.py:219-252).  Weights may be None
        (use_qk_norm=False); cos_sin_cache None means use_nope."""
        if len(norm_weights) != self.pool.num_layers:
            raise RMarinBackendContractError("fused qkv needs one norm pair per layer")
        if cos_sin_cache is not None and (cos_sin_cache.dtype != torch.bfloat16 or cos_sin_cache.shape[-1] != self.pool.d):
            raise RMarinBackendContractError("fused qkv expects a bf16 [max_pos, head_dim] rotary cache")
        self.layers = [(None if q is None else q.to(torch.bfloat16).contiguous(),
                        None if k is None else k.to(torch.bfloat16).contiguous()) for q, k in norm_weights]
        self.cos_sin = None if cos_sin_cache is None else cos_sin_cache.contiguous()
        self.eps = float(eps)

    # ------------------------------------------------------------------ host prologue
    def plan_rows(self, spans: list[Span], num_reqs_padded: int | None = None) -> dict:
        """Per-row plan (``_row_plan`` + ``_merged_fill``, fastpath.py:373-454) as numpy arrays."""
        pool = self.pool
        C, P = pool.chunk_size, PAGE_SIZE
        uniform = all(s.num_query_tokens == 1 for s in spans)
        batch = max(int(num_reqs_padded or 0), len(spans)) if uniform else len(spans)
        total = batch if uniform else sum(s.num_query_tokens for s in spans)
        if batch > self.max_batch or total > self.max_tokens:
            raise RMarinBackendContractError(f"step of {batch} rows / {total} tokens exceeds the fast path")
        ring = np.zeros(total, np.int64)
        src = np.zeros(total, np.int64)
        pos = np.zeros(total, np.int64)
        cu = np.zeros(batch + 1, np.int32)
        seqk = np.ones(batch, np.int32)
        nsrc = np.zeros(batch, np.int32)
        bt = np.zeros((batch, self.W), np.int32)
        commits = []
        tok = 0
        max_q = 1
        for row, sp in enumerate(spans):
            p0, n, slot = sp.num_computed_tokens, sp.num_query_tokens, sp.slot
            last = p0 + n - 1
            if p0 // C != last // C:
                raise RMarinBackendContractError("a span may not cross a chunk boundary")
            if last >= pool.max_sequence_tokens:
                raise RMarinBackendContractError("span beyond the slot's capacity")
            cur = (last // C) * C
            rec = max(0, cur - C)
            if cur > 0 and pool.committed[slot] < cur:
                if pool.committed[slot] != cur - C:
                    raise RMarinBackendContractError("boundary commits must be contiguous and exactly one chunk")
                commits.append((slot, cur))
            window = last + 1 - rec
            npages = -(-window // P)
            first = (rec // P) % pool.ring_pages
            ns = rec // P
            bt[row, :ns] = pool.src_table[slot, :ns]
            bt[row, ns:ns + npages] = slot * pool.ring_pages + (first + np.arange(npages)) % pool.ring_pages
            nsrc[row] = ns
            seqk[row] = last + 1
            tp = p0 + np.arange(n)
            ring[tok:tok + n] = slot * pool.ring_tokens + tp % pool.ring_tokens
            src[tok:tok + n] = pool.src_table[slot, tp // P].astype(np.int64) * P + tp % P
            pos[tok:tok + n] = tp
            tok += n
            cu[row + 1] = tok
            max_q = max(max_q, n)
        for row in range(len(spans), batch):  # padded rows read/write the scratch pages
            ring[tok] = pool.scratch_ring_page * P
            src[tok] = pool.scratch_src_page * P
            bt[row, 0] = pool.scratch_ring_page
            tok += 1
            cu[row + 1] = tok
        return {"uniform": uniform, "batch": batch, "tokens": tok, "max_q": max_q, "ring": ring, "src": src,
                "pos": pos, "cu": cu, "seqk": seqk, "nsrc": nsrc, "bt": bt, "commits": commits}

    def prepare_dummy(self, num_reqs: int) -> bool:
        """A uniform decode step whose rows all read and write the scratch pages
        (``prepare_dummy``, fastpath.py:584-600): vLLM's warm-up and CUDA-graph
        capture runs, which have no real requests."""
        return self.prepare([], max(1, int(num_reqs)), dummy=True)

    def prepare(self, spans: list[Span], num_reqs_padded: int | None = None, *, dummy: bool = False) -> bool:
        """Host prologue of one step (``prepare_real``, fastpath.py:456-582)."""
        if not spans and not dummy:
            self.active = False
            return False
        if self.pool.alpha is None or self.layers is None:
            raise RMarinBackendContractError("bind_parameters and register_layers must run before prepare")
        plan = self.plan_rows(spans, num_reqs_padded)
        if not self.fuse_commit:
            self._commit(plan["commits"])
        self._set = (self._set + 1) % self.NSETS
        h = self._h[self._set]
        if self._h_done[self._set] is not None:
            # the non_blocking copies that last read this set must have run before it is refilled
            self._h_done[self._set].synchronize()
        T, B = plan["tokens"], plan["batch"]
        h["ring"][:T] = torch.from_numpy(plan["ring"])
        h["src"][:T] = torch.from_numpy(plan["src"])
        h["pos"][:T] = torch.from_numpy(plan["pos"])
        h["cu"][:B + 1] = torch.from_numpy(plan["cu"])
        h["seqk"][:B] = torch.from_numpy(plan["seqk"])
        h["nsrc"][:B] = torch.from_numpy(plan["nsrc"])
        h["bt"][:B] = torch.from_numpy(plan["bt"])
        self.ring_idx[:T].copy_(h["ring"][:T], non_blocking=True)
        self.src_idx[:T].copy_(h["src"][:T], non_blocking=True)
        self.positions[:T].copy_(h["pos"][:T], non_blocking=True)
        self.cu_q[:B + 1].copy_(h["cu"][:B + 1], non_blocking=True)
        self.seq_k[:B].copy_(h["seqk"][:B], non_blocking=True)
        self.nsrc[:B].copy_(h["nsrc"][:B], non_blocking=True)
        self.bt[:B].copy_(h["bt"][:B], non_blocking=True)
        if self.fuse_commit:
            k = self._stage_commits(plan["commits"], h)
            if k:
                self.c_raw[:k].copy_(h["craw"][:k], non_blocking=True)
                self.c_ring[:k].copy_(h["cring"][:k], non_blocking=True)
            self.c_count.copy_(h["ccount"], non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        self._h_done[self._set] = done
        L = self.pool.num_layers
        self.bt_all = self._bt_all_flat[: L * B * self.W].view(L, B, self.W)
        ops.build_layer_block_tables(self.bt[:B], self.nsrc[:B], self.pool.ring_base_dev, out=self.bt_all)
        self.batch, self.tokens, self.max_q, self.uniform = B, T, plan["max_q"], plan["uniform"]
        self.active = True
        return True

    def _commit_pages(self, commits):
        """Shared pages and layer-0 ring pages [commits, C/16] of each finished chunk."""
        pool = self.pool
        C, P = pool.chunk_size, PAGE_SIZE
        raw = np.stack([pool.src_table[s, (end - C) // P:end // P] for s, end in commits]).astype(np.int32)
        ring = np.stack([pool.ring_base(0) + s * pool.ring_pages + ((end - C) % pool.ring_tokens) // P
                         + np.arange(C // P) for s, end in commits]).astype(np.int32)
        return raw, ring

    def _commit(self, commits) -> None:
        """Blend finished chunks into every layer ring in one launch (batching.py:1099-1144)."""
        if not commits:
            return
        pool = self.pool
        raw, ring = self._commit_pages(commits)
        ops.blend_chunk(pool.pool_k, pool.pool_v, torch.from_numpy(raw).to(pool.device),
                        torch.from_numpy(ring).to(pool.device), pool.ring_stride, pool.alpha,
                        error_word=self.error_word)
        for s, end in commits:
            pool.committed[s] = end

    def _stage_commits(self, commits, h) -> int:
        """The step's commits into staging set ``h`` for layer 0's fused append; returns their count.
        The commits count as done here: every later step's attention runs after that append."""
        k = len(commits)
        if k:
            raw, ring = self._commit_pages(commits)
            h["craw"][:k] = torch.from_numpy(raw)
            h["cring"][:k] = torch.from_numpy(ring)
            for s, end in commits:
                self.pool.committed[s] = end
        h["ccount"][0] = k
        return k

    # ------------------------------------------------------------------ per-layer ops
    def run_layer(self, layer_index: int, query, key, value, output):
        """Static per-layer op sequence (fastpath.py:619-651): append, attention, s_l."""
        pool, T, B = self.pool, self.tokens, self.batch
        qw, kw = self.layers[layer_index]
        top = layer_index == pool.num_layers - 1
        q = ops.rope_norm_append(
            query[:T].reshape(T, -1), key[:T].reshape(T, -1), value[:T].reshape(T, -1), self.positions[:T],
            self.cos_sin, qw, kw, self.eps, pool.inv_scale[layer_index], self.ring_idx[:T],
            pool.layer_ring_view(pool.pool_k, layer_index), pool.layer_ring_view(pool.pool_v, layer_index),
            self.src_idx[:T] if top else None, pool.src_view(pool.pool_k) if top else None,
            pool.src_view(pool.pool_v) if top else None, q_out=self.q_out[:T], error_word=self.error_word,
            commit=ops.Commit(pool.pool_k, pool.pool_v, self.c_raw, self.c_ring, pool.ring_stride, pool.alpha,
                              count=self.c_count, blocks=self.commit_blocks)
            if layer_index == 0 and self.fuse_commit else None)
        out = output[:T]
        if self.uniform:
            ops.decode_paged(q, pool.pool_k, pool.pool_v, self.bt_all[layer_index, :B], self.seq_k[:B],
                             softmax_scale=self.scale, out=out, out_scale=pool.out_scale[layer_index],
                             workspace=self.workspace, max_pages=self.W, l2_keep=True)
        else:
            ops.prefill_paged(q, pool.pool_k, pool.pool_v, self.bt_all[layer_index, :B], self.seq_k[:B],
                              self.cu_q[:B + 1], self.max_q, softmax_scale=self.scale, out=out,
                              out_scale=pool.out_scale[layer_index], error_word=self.error_word, max_pages=self.W)
        if self.check:
            self.merged_check(layer_index, q, out)
        return output

    def merged_check(self, layer_index: int, q, out) -> dict:
        """Two-pass recomputation of one layer from the same pool (the reference's
        _merged_check_impl, fastpath.py:737-766): causal attention over the layer's ring
        pages, non-causal attention over the older shared pages, LSE merge (x s_l); the
        relative L2 deviation of the merged single call from it is logged and printed for
        the first 192 layer calls and whenever it exceeds 0.02."""
        pool, B, T = self.pool, self.batch, self.tokens
        bt = self.bt_all[layer_index, :B]
        nsrc = self.nsrc[:B]
        seqk = self.seq_k[:B]
        cu = self.cu_q[:B + 1]
        idx = (nsrc.unsqueeze(1).long() + torch.arange(pool.ring_pages, device=bt.device).unsqueeze(0)).clamp_(
            max=self.W - 1)
        bt_loc = torch.gather(bt, 1, idx).to(torch.int32).contiguous()
        seq_loc = (seqk - nsrc * PAGE_SIZE).to(torch.int32)
        seq_src = torch.clamp(nsrc * PAGE_SIZE, min=1).to(torch.int32)
        lse_loc = torch.empty((T, self.hq), dtype=torch.float32, device=q.device)
        lse_src = torch.empty_like(lse_loc)
        lo = ops.prefill_paged(q, pool.pool_k, pool.pool_v, bt_loc, seq_loc, cu, self.max_q, causal=True,
                               softmax_scale=self.scale, lse=lse_loc, error_word=self.error_word,
                               max_pages=pool.ring_pages, kv_splits=1)
        so = ops.prefill_paged(q, pool.pool_k, pool.pool_v, bt.contiguous(), seq_src, cu, self.max_q, causal=False,
                               softmax_scale=self.scale, lse=lse_src, error_word=self.error_word,
                               max_pages=self.W, kv_splits=1)
        # sequences without older shared pages: the source pass saw a placeholder key
        tok_seq = torch.repeat_interleave(torch.arange(B, device=q.device), (cu[1:] - cu[:-1]).long(),
                                          output_size=T)
        lse_src.masked_fill_((nsrc[tok_seq] == 0).unsqueeze(1), float("-inf"))
        ref = ops.merge_partials(torch.stack([so.float(), lo.float()]), torch.stack([lse_src, lse_loc]),
                                 out_scale=pool.out_scale[layer_index])
        diff = float((ref.float() - out.float()).norm() / ref.float().norm().clamp(min=1e-6))
        self.check_steps += 1
        rec = {"layer": layer_index, "batch": B, "tokens": T, "rel": round(diff, 5),
               "out_absmax": round(float(out.float().abs().max()), 2), "ref_absmax": round(float(ref.float().abs().max()), 2)}
        self.check_log.append(rec)
        if self.check_steps <= 32 * 6 or diff > 0.02:
            print({"rmarin_merged_check": rec}, flush=True)
        return rec

    def check_errors(self) -> None:
        e, w = self.error_word.cpu().tolist(), self.workspace.error()
        if e[0] or w[0]:
            raise RMarinBackendContractError(f"device error word set: {e} / decode {w}")


class SharedKVAttentionImpl:
    """The attention-impl forward contract (vllm_backend.py:637-717)."""

    can_return_lse_for_decode = False

    def __init__(self, fast_path: SharedKVFastPath, num_heads: int, head_size: int):
        self.fast = fast_path
        self.num_heads, self.head_size = num_heads, head_size

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None):
        del kv_cache  # the shared pool belongs to the fast path
        if attn_metadata is None:
            return output.fill_(0)
        if output_scale is not None or output_block_scale is not None:
            raise RMarinBackendContractError("fused output quantization is not supported")
        if not self.fast.active:
            raise RMarinBackendContractError("fast path was not prepared for this step")
        self.fast.run_layer(int(layer.rmarin_layer_index), query.view(-1, self.num_heads, self.head_size),
                            key, value, output.view(-1, self.num_heads, self.head_size))
        if int(output.shape[0]) > self.fast.tokens:
            output[self.fast.tokens:].fill_(0)
        return output


class SharedKVBackend:
    """Backend class surface (vllm_backend.py:719-750)."""

    supported_dtypes = [torch.bfloat16]
    supported_kv_cache_dtypes = ["auto", "bfloat16"]
    forward_includes_kv_cache_update = True

    @staticmethod
    def get_name() -> str:
        return "CUSTOM"

    @staticmethod
    def get_impl_cls():
        return SharedKVAttentionImpl

    @classmethod
    def supports_non_causal(cls) -> bool:
        return False

    @classmethod
    def supports_sink(cls) -> bool:
        return False


def rope_cos_sin_cache(max_pos: int, head_dim: int, theta: float, scaling: dict | None = None, device=None):
    """bf16 [max_pos, D] cos|sin cache in vLLM's layout (cos half then sin half)."""
    from .hf import _llama3_inv_freq

    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    if scaling and scaling.get("rope_type", scaling.get("type")) == "llama3":
        inv = _llama3_inv_freq(inv, scaling)
    t = torch.arange(max_pos, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.cat((t.cos(), t.sin()), dim=-1).to(torch.bfloat16).to(device or "cuda")


__all__ = ["Span", "SharedKVPool", "SharedKVFastPath", "SharedKVAttentionImpl", "SharedKVBackend",
           "chunk_aligned_new_tokens", "sliver_deferred_new_tokens", "rope_cos_sin_cache", "math"]
