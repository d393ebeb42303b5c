"""CUDA-graph greedy decoding for ``LastKVForCausalLM`` on the paged shared-KV cache.

One decode step (embedding, rotary, every layer's fused append + split-KV
decode + dense layers, final norm, LM head, argmax) is captured once into a
CUDA graph over static buffers.  Before each replay the host prologue
(``PagedLastKVCache.plan_host``, the equivalent of the reference's
``prepare_real``, vllm/src/lastkv/vllm/backends/rmarin_flashinfer/fastpath.py:456-582)
fills pinned staging buffers that are copied to the static device buffers on
the same stream; the argmax of a step feeds the next step on the device.  The
chunk-boundary commit runs inside the first layer's append of the next step:
a second graph, captured with that fused launch over static page lists,
replays for the step after each boundary.  All sequences of the batch advance
together (equal positions), as in ``generate``.
"""

from __future__ import annotations

import torch

from . import ops
from .contract import PAGE_SIZE, RMarinBackendContractError
from .hf import LastKVForCausalLM, PagedLastKVCache


class GraphDecodeRunner:
    NSETS = 4

    def __init__(self, model: LastKVForCausalLM, cache: PagedLastKVCache):
        self.model, self.cache = model, cache
        dev = cache.device
        B, L = cache.batch, cache.num_layers
        self.B, self.L = B, L
        self.W = cache.pages_per_seq + cache.ring_pages
        self.ids = torch.zeros((B, 1), dtype=torch.int64, device=dev)
        self.pos = torch.zeros((1, 1), dtype=torch.int64, device=dev)
        self.bt = torch.zeros((B, self.W), dtype=torch.int32, device=dev)
        self.nsrc = torch.zeros(B, dtype=torch.int32, device=dev)
        self.bt_all = torch.zeros((L, B, self.W), dtype=torch.int32, device=dev)
        self.seq_k = torch.ones(B, dtype=torch.int32, device=dev)
        self.ring_tok = torch.zeros(B, dtype=torch.int64, device=dev)
        self.src_slot = torch.zeros(B, dtype=torch.int64, device=dev)
        self.local_pos = torch.zeros(B, dtype=torch.int64, device=dev)
        self.cu_q = torch.arange(B + 1, dtype=torch.int32, device=dev)
        self._h = [{"bt": torch.zeros((B, self.W), dtype=torch.int32).pin_memory(),
                    "nsrc": torch.zeros(B, dtype=torch.int32).pin_memory(),
                    "seqk": torch.zeros(B, dtype=torch.int32).pin_memory(),
                    "ring": torch.zeros(B, dtype=torch.int64).pin_memory(),
                    "src": torch.zeros(B, dtype=torch.int64).pin_memory(),
                    "pos": torch.zeros((1, 1), dtype=torch.int64).pin_memory(),
                    "done": None} for _ in range(self.NSETS)]
        self._set = 0
        self.graph = None
        self.graph_commit = None  # the step after a chunk boundary (bf16 caches)
        self.alpha = model.model.blend_alpha(cache.dtype)
        ppc = cache.chunk_size // PAGE_SIZE
        self.c_raw = torch.zeros((B, ppc), dtype=torch.int32, device=dev)
        self.c_ring = torch.zeros((B, ppc), dtype=torch.int32, device=dev)

    def _prepare(self):
        """Host plan of the next token -> static device buffers (stream-ordered copies)."""
        cache = self.cache
        h = cache.plan_host(1)
        self._set = (self._set + 1) % self.NSETS
        st = self._h[self._set]
        if st["done"] is not None:
            st["done"].synchronize()  # the copy that last used this staging set has run
        st["bt"].zero_()
        st["bt"][:, : h["W"]] = torch.from_numpy(h["bt"])
        st["nsrc"].fill_(h["nsrc"])
        st["seqk"].fill_(h["seq_k"])
        st["ring"].copy_(torch.from_numpy(h["ring_tok"]))
        st["src"].copy_(torch.from_numpy(h["src_tok"]))
        st["pos"].fill_(cache.seen_tokens)
        self.bt.copy_(st["bt"], non_blocking=True)
        self.nsrc.copy_(st["nsrc"], non_blocking=True)
        self.seq_k.copy_(st["seqk"], non_blocking=True)
        self.ring_tok.copy_(st["ring"], non_blocking=True)
        self.src_slot.copy_(st["src"], non_blocking=True)
        self.pos.copy_(st["pos"], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        st["done"] = ev
        ops.build_layer_block_tables(self.bt, self.nsrc, cache.ring_base_dev, out=self.bt_all)
        self._fresh_meta()

    def _fresh_meta(self, tables_ready=True):
        """The span metadata over the static buffers, without the per-span values the
        layers memoise (so a capture records the kernels that compute them).

        ``tables_ready``: the block tables and sequence lengths are written before the
        graph starts (copies + the table kernel in ``_prepare``), and a graph's first
        kernel waits for all earlier stream work, so every decode in the step may start
        its page loads before its PDL wait (LKV_DECODE_TABLES_READY).  Not in the step
        after a boundary: its first append launch rewrites the finished chunk's ring
        pages of every layer, so those decodes load pages after their wait."""
        self.cache._meta = {"n": 1, "W": self.W, "bt_all": self.bt_all, "seq_k": self.seq_k, "cu_q": self.cu_q,
                            "local_pos": self.local_pos, "ring_tok": self.ring_tok, "src_slot": self.src_slot,
                            "tables_ready": tables_ready}

    def _body(self):
        m = self.model.model
        hidden = m.embed_tokens(self.ids)
        pe = m.rotary_emb(hidden, self.pos)
        logits = self.model.lm_head(m.run_layers(hidden, pe, self.cache)[:, -1])
        if logits.dtype == torch.bfloat16 and logits.shape[-1] % 8 == 0:
            ops.argmax_rows(logits, out=self.ids.view(-1))  # torch.argmax order, one launch
        else:
            self.ids.copy_(logits.float().argmax(-1, keepdim=True))

    def capture(self):
        """Capture one decode step at the current position (the warm-up runs do not advance),
        and for bf16 caches the same step with a boundary commit fused into layer 0's append."""
        cache = self.cache
        cache.flush_commit()
        saved = self.ids.clone()
        self._prepare()
        fused = cache.fuse_commit
        empty = torch.zeros((0, self.c_raw.shape[1]), dtype=torch.int32, device=self.ids.device)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for i in range(3 if fused else 2):
                self.ids.copy_(saved)
                self._fresh_meta()
                if i == 2:  # loads the fused append kernel before its capture; commits nothing
                    cache._pending = ops.Commit(cache.pool_k, cache.pool_v, empty, empty, cache.ring_stride,
                                                self.alpha)
                self._body()
        torch.cuda.current_stream().wait_stream(s)
        self.ids.copy_(saved)
        self._fresh_meta()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._body()
        self.graph = g
        if fused:
            self._fresh_meta(tables_ready=False)
            cache._pending = ops.Commit(cache.pool_k, cache.pool_v, self.c_raw, self.c_ring, cache.ring_stride,
                                        self.alpha)
            gc = torch.cuda.CUDAGraph()
            try:
                with torch.cuda.graph(gc, pool=g.pool()):
                    self._body()
            finally:
                cache._pending = None
            self.graph_commit = gc
        self.ids.copy_(saved)

    def step(self):
        """One greedy token for every sequence; returns the device tensor of new ids [B, 1]."""
        if self.graph is None:
            raise RMarinBackendContractError("capture() must run before step()")
        cache = self.cache
        pending = cache.take_commit()
        if pending is not None and (self.graph_commit is None or pending.pool_k is not cache.pool_k
                                    or pending.alpha is not self.alpha
                                    or pending.raw_pages.shape != self.c_raw.shape):
            cache._pending = pending  # not the captured form: run it on its own
            cache.flush_commit()
            pending = None
        self._prepare()
        if pending is not None:
            self.c_raw.copy_(pending.raw_pages)
            self.c_ring.copy_(pending.ring_pages)
            self.graph_commit.replay()
        else:
            self.graph.replay()
        cache.seen_tokens += 1
        cache._meta = None
        if cache.seen_tokens % cache.chunk_size == 0:
            cache.commit(self.alpha)
        return self.ids

    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor, call_tokens: int) -> torch.Tensor:
        """Eager chunked prefill in calls of ``call_tokens`` (split at chunk boundaries inside);
        sets the first generated token into the static id buffer."""
        logits = None
        for start in range(0, prompt.shape[1], call_tokens):
            logits, _ = self.model(prompt[:, start:start + call_tokens], self.cache, logits_to_keep=1)
        self.ids.copy_(logits[:, -1].float().argmax(-1, keepdim=True))
        return self.ids


def init_random_(model: torch.nn.Module, std: float = 0.02, seed: int = 0, scale_range=(0.1, 2.0)) -> None:
    """Random weights in place: Linear/Embedding ~ N(0, std), norms = 1, blend logits ~ N(0, 1),
    value scales ~ U(scale_range) (bf16-exact after the model's cast)."""
    g = torch.Generator(device=next(model.parameters()).device).manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.fill_(1.0)
            elif name.endswith("prev_chunk_alphas"):
                p.normal_(0.0, 1.0, generator=g)
            elif name.endswith("deep_v_scale"):
                p.uniform_(*scale_range, generator=g)
            else:
                p.normal_(0.0, std, generator=g)


__all__ = ["GraphDecodeRunner", "init_random_"]
