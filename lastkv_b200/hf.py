"""Drop-in LastKV language model whose attention runs on the B200 kernels.

Mirrors the reference's HF implementation (llm/src/lastkv/llm/modeling.py)
module for module and parameter name for parameter name, so a reference
state dict loads strictly:

* ``LastKVConfig``        - the config fields the path reads (configuration.py:13-48)
* ``PagedLastKVCache``    - ``LastKVCache`` (modeling.py:37-67) backed by the merged
                            paged pool: shared final-layer pages + per-layer 2C rings
* ``LastKVAttention``     - ``LastKVAttention.forward(hidden, (cos, sin), cache)``
                            (modeling.py:98-148): q/k/v projection, then one fused
                            RoPE -> Q/K RMSNorm -> V/s -> paged-append kernel, then
                            the split-KV decode kernel (one new token) or the tcgen05
                            prefill kernel (a chunk), output scaled by s_l in-kernel
* ``LastKVModel`` / ``LastKVForCausalLM`` - the chunk loop and commit
                            (modeling.py:173-212): spans never cross a chunk
                            boundary, and a completed chunk is blended into every
                            layer ring by the blend kernel.

Dense layers (projections, MLP, norms, embedding, LM head) are plain torch
(cuBLAS); everything on the shared-KV path goes through ``lastkv_b200.ops``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch
from torch import nn
from torch.nn import functional as F

from . import ops
from .contract import PAGE_SIZE, RMarinBackendContractError, require_chunk_size, require_heads


@dataclass
class LastKVConfig:
    hidden_size: int
    intermediate_size: int
    num_attention_heads: int
    num_key_value_heads: int
    num_hidden_layers: int
    head_dim: int
    vocab_size: int
    chunk_size: int = 1024
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_scaling: dict | None = None
    max_position_embeddings: int = 8192
    deep_kv_rescale: bool = True
    deep_v_scale_init: object = 1.0
    use_qk_norm: bool = True
    use_nope: bool = False
    attention_bias: bool = False
    tie_word_embeddings: bool = False
    initializer_range: float = 0.02
    extra: dict = field(default_factory=dict)

    def __post_init__(self):
        require_chunk_size(self.chunk_size)
        require_heads(self.num_attention_heads, self.num_key_value_heads, self.head_dim)

    @classmethod
    def from_dict(cls, d: dict) -> "LastKVConfig":
        known = {f for f in cls.__dataclass_fields__ if f != "extra"}
        kw = {k: v for k, v in d.items() if k in known}
        return cls(**kw, extra={k: v for k, v in d.items() if k not in known})


def _llama3_inv_freq(inv_freq: torch.Tensor, scaling: dict) -> torch.Tensor:
    """Llama-3.1 frequency scaling (the published rule: keep high frequencies,
    divide low ones by ``factor``, interpolate smoothly in between)."""
    factor = scaling["factor"]
    low, high = scaling.get("low_freq_factor", 1.0), scaling.get("high_freq_factor", 4.0)
    old_len = scaling.get("original_max_position_embeddings", 8192)
    low_wl, high_wl = old_len / low, old_len / high
    wavelen = 2 * math.pi / inv_freq
    scaled = torch.where(wavelen > low_wl, inv_freq / factor, inv_freq)
    smooth = (old_len / wavelen - low) / (high - low)
    mid = (1 - smooth) * scaled / factor + smooth * scaled
    is_mid = (wavelen >= high_wl) & (wavelen <= low_wl)
    return torch.where(is_mid, mid, scaled)


class RotaryEmbedding(nn.Module):
    """NeoX rotary frequencies; returns (cos, sin) [1, L, D] like the HF module."""

    def __init__(self, config: LastKVConfig, device=None):
        super().__init__()
        self.config = config
        self.register_buffer("inv_freq", self._frequencies(device or "cpu"), persistent=False)

    def _frequencies(self, device) -> torch.Tensor:
        """fp32 frequencies, computed on the host (as the reference's module is built) and moved."""
        config, d = self.config, self.config.head_dim
        inv = 1.0 / (config.rope_theta ** (torch.arange(0, d, 2, dtype=torch.int64, device="cpu").float() / d))
        if config.rope_scaling and config.rope_scaling.get("rope_type", config.rope_scaling.get("type")) == "llama3":
            inv = _llama3_inv_freq(inv, config.rope_scaling)
        return inv.to(device)

    def _apply(self, fn, recurse=True):
        # dtype casts of the model and meta-device materialisation leave the
        # frequencies fp32 and exact: recompute them on the buffer's new device
        super()._apply(fn, recurse)
        self.inv_freq = self._frequencies(self.inv_freq.device)
        return self

    @torch.no_grad()
    def forward(self, x, position_ids):
        freqs = position_ids[..., None].float() * self.inv_freq.to(x.device)[None, None, :]
        emb = torch.cat((freqs, freqs), dim=-1)
        return emb.cos().to(x.dtype), emb.sin().to(x.dtype)


class RMSNorm(nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.variance_epsilon = eps

    def forward(self, x):
        dt = x.dtype
        h = x.float()
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + self.variance_epsilon)
        return self.weight * h.to(dt)

    def fused(self, x, residual=None):
        """``(h, norm(h))`` with ``h = x + residual`` (or ``x``): one kernel for bf16 CUDA rows."""
        H = x.shape[-1]
        if x.is_cuda and x.dtype == torch.bfloat16 and self.weight.dtype == torch.bfloat16 and H % 8 == 0 \
                and H <= 8192:
            w = self.weight.detach()
            if residual is None:
                return x, ops.rmsnorm(x, w, self.variance_epsilon)
            return ops.rmsnorm(x, w, self.variance_epsilon, residual)
        h = x if residual is None else x + residual
        return h, self(h)


def _fuse_linears(linears) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Concatenate the weights (and biases) of ``linears`` along the output dim and
    re-point each module's parameters at its slice, so one GEMM computes all of
    them and state-dict loads still write through the original names."""
    w = torch.cat([lin.weight.detach() for lin in linears], 0)
    has_bias = linears[0].bias is not None
    b = torch.cat([lin.bias.detach() for lin in linears], 0) if has_bias else None
    start = 0
    for lin in linears:
        n = lin.out_features
        rg = lin.weight.requires_grad
        lin.weight = nn.Parameter(w[start:start + n], requires_grad=rg)
        if has_bias:
            lin.bias = nn.Parameter(b[start:start + n], requires_grad=lin.bias.requires_grad)
        start += n
    return w, b


def _fused_ok(fused, linears) -> bool:
    """The fused buffers still back every module's parameters (a later .to() or
    parameter replacement breaks the aliasing; then the modules run separately)."""
    if fused is None:
        return False
    w, b = fused
    start = 0
    for lin in linears:
        n = lin.out_features
        if lin.weight.data_ptr() != w[start:start + n].data_ptr() or lin.weight.dtype != w.dtype:
            return False
        if b is not None and (lin.bias is None or lin.bias.data_ptr() != b[start:start + n].data_ptr()):
            return False
        start += n
    return True


def _decode_linear(x, weight, bias=None, silu_mul=False):
    """``F.linear`` (or, with ``silu_mul``, ``silu(x @ gate.T) * (x @ up.T)`` for
    weight = [gate | up]) on the tcgen05 decode GEMM for at most 16 bf16 rows
    without bias - the decode-step shapes, where every projection of a layer is
    one weight stream chained to its neighbours by PDL; None otherwise."""
    if bias is None and ops.decode_gemm_supported(x, weight):
        return ops.decode_gemm(x, weight, silu_mul=silu_mul)
    return None


class MLP(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.gate_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.down_proj = nn.Linear(config.intermediate_size, config.hidden_size, bias=False)
        self._gate_up = None

    def fuse_(self):
        """One [gate | up] GEMM + the SiLU-and-mul kernel instead of two GEMMs and two elementwise ops."""
        self._gate_up = _fuse_linears([self.gate_proj, self.up_proj])
        return self

    def forward(self, x):
        if x.is_cuda and x.dtype == torch.bfloat16 and _fused_ok(self._gate_up, [self.gate_proj, self.up_proj]):
            w = self._gate_up[0]
            h = _decode_linear(x, w, silu_mul=True)
            if h is None:
                h = ops.silu_mul(F.linear(x, w))
            y = _decode_linear(h, self.down_proj.weight, self.down_proj.bias)
            return y if y is not None else self.down_proj(h)
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


# ----------------------------------------------------------------------- cache


class PagedLastKVCache:
    """``LastKVCache`` on the merged paged pool, for ``batch`` unpadded sequences.

    Layout (batching.py:1999-2016): pages ``[0, src)`` hold each sequence's shared
    final-layer history (raw K, raw V), ``pages_per_seq`` per sequence (the
    page order may be shuffled); layer ``l`` owns ``2C/16`` ring pages per
    sequence at ``ring_base[l] + b * ring_pages`` holding K and V / s_l.
    ``seen_tokens``, ``get_seq_length`` and ``reorder_cache`` keep the
    reference's meaning (modeling.py:56-67).
    """

    def __init__(self, config: LastKVConfig, batch: int, max_tokens: int, device=None, *, page_order=None,
                 dtype=torch.bfloat16):
        if dtype not in (torch.bfloat16, torch.float32):
            raise RMarinBackendContractError("the paged cache holds bf16 or fp32 keys and values")
        self.dtype = dtype
        self.num_layers = config.num_hidden_layers
        self.chunk_size = config.chunk_size
        self.batch = batch
        self.max_tokens = max_tokens
        self.hkv, self.d = config.num_key_value_heads, config.head_dim
        self._hq = config.num_attention_heads
        self.seen_tokens = 0
        self.committed = 0
        device = torch.device(device or "cuda")
        self.device = device
        C = self.chunk_size
        self.pages_per_seq = -(-max_tokens // PAGE_SIZE)
        self.ring_pages = 2 * C // PAGE_SIZE
        self.ring_tokens = 2 * C
        self.src_pages = batch * self.pages_per_seq
        self.ring_stride = self.ring_pages * batch + 1
        self.num_pages = self.src_pages + self.num_layers * self.ring_stride
        shape = (self.num_pages, PAGE_SIZE, self.hkv, self.d)
        self.pool_k = torch.zeros(shape, dtype=dtype, device=device)
        self.pool_v = torch.zeros(shape, dtype=dtype, device=device)
        order = np.arange(self.src_pages) if page_order is None else np.asarray(page_order)
        if sorted(order.tolist()) != list(range(self.src_pages)):
            raise RMarinBackendContractError("page_order must permute the shared pages")
        self.src_table = order.reshape(batch, self.pages_per_seq).astype(np.int32)
        self.src_table_dev = torch.from_numpy(self.src_table).to(device)
        self.ring_base = self.src_pages + np.arange(self.num_layers) * self.ring_stride
        self.ring_base_dev = torch.from_numpy(self.ring_base.astype(np.int32)).to(device)
        self.error_word = torch.zeros(4, dtype=torch.int32, device=device)
        # the split-KV partials of the bf16 decode (the fp32 attention needs no scratch)
        self.workspace = ops.Workspace.for_decode(batch, config.num_attention_heads, self.d,
                                                  self.pages_per_seq + self.ring_pages, device=device) \
            if dtype == torch.bfloat16 else None
        self._meta = None
        # bf16: a boundary commit waits for the next span's first-layer append and runs inside
        # that launch (lkv_rope_norm_append_commit); False: one blend launch at the boundary
        self.fuse_commit = dtype == torch.bfloat16
        self._pending = None

    # -- capacity
    def reserve(self, max_tokens: int) -> None:
        """Grow the cache to hold ``max_tokens`` tokens per sequence, keeping its contents:
        a new pool with ``ceil(max_tokens / 16)`` shared pages per sequence (in sequence
        order), the old shared pages and every layer ring copied over (for callers that
        do not know the final length up front, such as ``generate``).  Allocates; not
        for use inside a CUDA-graph capture."""
        if max_tokens <= self.max_tokens:
            return
        self.flush_commit()
        B, L, P = self.batch, self.num_layers, PAGE_SIZE
        pps = -(-max_tokens // P)
        src_pages = B * pps
        num_pages = src_pages + L * self.ring_stride
        table = np.arange(src_pages, dtype=np.int32).reshape(B, pps)
        ring_base = src_pages + np.arange(L) * self.ring_stride
        old_idx = [self.src_table.reshape(-1)] + [self.ring_base[l] + np.arange(self.ring_stride) for l in range(L)]
        new_idx = [table[:, : self.pages_per_seq].reshape(-1)] + [ring_base[l] + np.arange(self.ring_stride)
                                                                   for l in range(L)]
        o = torch.from_numpy(np.concatenate(old_idx).astype(np.int64)).to(self.device)
        n = torch.from_numpy(np.concatenate(new_idx).astype(np.int64)).to(self.device)
        shape = (num_pages, P, self.hkv, self.d)
        for name in ("pool_k", "pool_v"):
            old = getattr(self, name)
            new = torch.zeros(shape, dtype=self.dtype, device=self.device)
            new[n] = old.index_select(0, o)
            setattr(self, name, new)
        self.max_tokens = max_tokens
        self.pages_per_seq = pps
        self.src_pages = src_pages
        self.num_pages = num_pages
        self.src_table = table
        self.src_table_dev = torch.from_numpy(table).to(self.device)
        self.ring_base = ring_base
        self.ring_base_dev = torch.from_numpy(ring_base.astype(np.int32)).to(self.device)
        if self.workspace is not None:
            self.workspace = ops.Workspace.for_decode(B, self._hq, self.d, pps + self.ring_pages, device=self.device)
        self._meta = None

    # -- reference API
    def get_seq_length(self, layer_idx=0):
        return self.seen_tokens

    def reorder_cache(self, beam_idx):
        """Reorder sequences (beam search): gather shared pages and rings by beam index."""
        self.flush_commit()
        idx = beam_idx.to("cpu").long().numpy()
        src_old = self.src_table[idx].reshape(-1)
        src_new = self.src_table.reshape(-1)
        ring_old = (idx[:, None] * self.ring_pages + np.arange(self.ring_pages)[None]).reshape(-1)
        ring_new = (np.arange(self.batch)[:, None] * self.ring_pages + np.arange(self.ring_pages)[None]).reshape(-1)
        old = [src_old] + [self.ring_base[l] + ring_old for l in range(self.num_layers)]
        new = [src_new] + [self.ring_base[l] + ring_new for l in range(self.num_layers)]
        o = torch.from_numpy(np.concatenate(old)).to(self.device)
        n = torch.from_numpy(np.concatenate(new)).to(self.device)
        for pool in (self.pool_k, self.pool_v):
            pool[n] = pool.index_select(0, o)
        self._meta = None

    # -- per-span metadata (shared by all layers of one chunk piece)
    def plan_host(self, n_new: int) -> dict:
        """Host part of the span plan (fastpath.py:427-454 / 373-424) as numpy arrays."""
        C, P = self.chunk_size, PAGE_SIZE
        start = self.seen_tokens
        last = start + n_new - 1
        if last >= self.max_tokens:
            raise RMarinBackendContractError(f"cache capacity {self.max_tokens} exceeded")
        if (start // C) != (last // C):
            raise RMarinBackendContractError("a span may not cross a chunk boundary")
        cur = (last // C) * C
        rec = max(0, cur - C)
        nsrc = rec // P
        window = last + 1 - rec
        npages = -(-window // P)
        first = (rec // P) % self.ring_pages
        B = self.batch
        W = nsrc + npages
        bt = np.zeros((B, W), np.int32)
        for b in range(B):
            bt[b, :nsrc] = self.src_table[b, :nsrc]
            bt[b, nsrc:] = b * self.ring_pages + (first + np.arange(npages)) % self.ring_pages
        pos = start + np.arange(n_new)
        ring_tok = (np.arange(B)[:, None] * self.ring_tokens + (pos % self.ring_tokens)[None, :]).reshape(-1)
        src_tok = (self.src_table[:, pos // P] * P + (pos % P)[None, :]).reshape(-1)
        return {"bt": bt, "nsrc": nsrc, "W": W, "seq_k": last + 1, "ring_tok": ring_tok.astype(np.int64),
                "src_tok": src_tok.astype(np.int64)}

    def plan(self, n_new: int):
        h = self.plan_host(n_new)
        B, dev = self.batch, self.device
        # block tables are padded to the maximum width, so the decode kernel's
        # split plan is the same at every position (and in captured graphs)
        w_max = self.pages_per_seq + self.ring_pages
        bt = np.zeros((B, w_max), np.int32)
        bt[:, : h["W"]] = h["bt"]
        bt_d = torch.from_numpy(bt).to(dev)
        nsrc_d = torch.full((B,), h["nsrc"], dtype=torch.int32, device=dev)
        meta = {
            "n": n_new, "W": w_max,
            "bt_all": ops.build_layer_block_tables(bt_d, nsrc_d, self.ring_base_dev),
            "seq_k": torch.full((B,), h["seq_k"], dtype=torch.int32, device=dev),
            "cu_q": torch.arange(0, (B + 1) * n_new, n_new, dtype=torch.int32, device=dev),
            "local_pos": torch.arange(n_new, device=dev, dtype=torch.int64).repeat(B),
            "ring_tok": torch.from_numpy(h["ring_tok"]).to(dev),
            "src_slot": torch.from_numpy(h["src_tok"]).to(dev),
        }
        self._meta = meta
        return meta

    def advance(self, n_new: int):
        self.seen_tokens += n_new
        self._meta = None

    def commit(self, alpha: torch.Tensor):
        """Blend the chunk that just completed into every layer ring (modeling.py:203-207).

        With ``fuse_commit`` the blend is queued and runs inside the next span's
        first-layer append (the next attention to read a ring comes after it);
        ``flush_commit`` runs a queued blend on its own."""
        C, P = self.chunk_size, PAGE_SIZE
        end = self.seen_tokens
        if end % C or end == self.committed:
            return
        if end != self.committed + C:
            raise RMarinBackendContractError("boundary commits must be contiguous and exactly one chunk")
        pages = np.arange((end - C) // P, end // P)
        raw = self.src_table[:, pages]
        ring_first = ((end - C) % self.ring_tokens) // P
        ring = (self.ring_base[0] + np.arange(self.batch)[:, None] * self.ring_pages
                + ring_first + np.arange(C // P)[None, :])
        raw_d = torch.from_numpy(np.ascontiguousarray(raw, dtype=np.int32)).to(self.device)
        ring_d = torch.from_numpy(np.ascontiguousarray(ring, dtype=np.int32)).to(self.device)
        self.flush_commit()
        if self.fuse_commit:
            self._pending = ops.Commit(self.pool_k, self.pool_v, raw_d, ring_d, self.ring_stride, alpha)
        else:
            ops.blend_chunk(self.pool_k, self.pool_v, raw_d, ring_d, self.ring_stride, alpha,
                            error_word=self.error_word)
        self.committed = end

    def take_commit(self):
        """The queued boundary commit (an ``ops.Commit``) for the caller's append, or None."""
        c, self._pending = self._pending, None
        return c

    def flush_commit(self) -> None:
        """Run a queued boundary commit now (before the pools are read or moved outside a span)."""
        c = self.take_commit()
        if c is not None:
            ops.blend_chunk(c.pool_k, c.pool_v, c.raw_pages, c.ring_pages, c.ring_layer_stride, c.alpha,
                            error_word=self.error_word)

    def check_errors(self):
        e = self.error_word.cpu().tolist()
        w = self.workspace.error() if self.workspace is not None else [0, 0, 0, 0]
        if e[0] or w[0]:
            raise RMarinBackendContractError(f"device error word set: append/blend {e}, decode {w}")


# ----------------------------------------------------------------------- attention


class LastKVAttention(nn.Module):
    """Same parameters and call signature as the reference (modeling.py:70-148)."""

    def __init__(self, config: LastKVConfig, layer_idx: int):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.head_dim = config.head_dim
        self.num_heads = config.num_attention_heads
        self.num_key_value_heads = config.num_key_value_heads
        h, d = config.hidden_size, config.head_dim
        self.q_proj = nn.Linear(h, self.num_heads * d, bias=config.attention_bias)
        self.k_proj = nn.Linear(h, self.num_key_value_heads * d, bias=config.attention_bias)
        self.v_proj = nn.Linear(h, self.num_key_value_heads * d, bias=config.attention_bias)
        self.o_proj = nn.Linear(self.num_heads * d, h, bias=config.attention_bias)
        self.prev_chunk_alphas = nn.Parameter(torch.zeros(self.num_key_value_heads))
        if config.deep_kv_rescale:
            init = config.deep_v_scale_init
            value = init[layer_idx] if isinstance(init, (list, tuple)) else init
            values = value if isinstance(value, (list, tuple)) else [value] * self.num_key_value_heads
            if len(values) != self.num_key_value_heads:
                raise ValueError("deep_v_scale_init must match the number of KV heads")
            self.deep_v_scale = nn.Parameter(torch.tensor(values, dtype=torch.float32))
        if config.use_qk_norm:
            self.q_norm = RMSNorm(d, config.rms_norm_eps)
            self.k_norm = RMSNorm(d, config.rms_norm_eps)
        self._qkv = None
        self._consts = (None, None)

    def fuse_qkv_(self):
        """One [q | k | v] GEMM per call; the three projections become views of its weight."""
        self._qkv = _fuse_linears([self.q_proj, self.k_proj, self.v_proj])
        return self

    def _layer_constants(self, kv_dtype=torch.bfloat16):
        """(s, 1/s, s per query head, q-norm weight, k-norm weight) for the kernels of a
        ``kv_dtype`` cache, rebuilt only when a parameter they derive from changes
        (in-place loads bump the version)."""
        params = [p for p in (getattr(self, "deep_v_scale", None),
                              getattr(getattr(self, "q_norm", None), "weight", None),
                              getattr(getattr(self, "k_norm", None), "weight", None)) if p is not None]
        key = tuple((p.data_ptr(), p._version, p.dtype) for p in params) + (str(self.q_proj.weight.device),
                                                                             kv_dtype)
        if self._consts[0] != key:
            s = self.value_scale(kv_dtype)
            qn = getattr(self, "q_norm", None)
            kn = getattr(self, "k_norm", None)
            self._consts = (key, (s, (1.0 / s).contiguous(),
                                  s.repeat_interleave(self.num_heads // self.num_key_value_heads).contiguous(),
                                  qn.weight.detach().to(kv_dtype).contiguous() if qn is not None else None,
                                  kn.weight.detach().to(kv_dtype).contiguous() if kn is not None else None))
        return self._consts[1]

    def value_scale(self, kv_dtype=torch.bfloat16) -> torch.Tensor:
        """s_l per KV head as the pool sees it, in fp32: bf16-exact values for a bf16 cache
        (batching.py:1070-1080), the parameter itself for an fp32 one (``_scale``,
        modeling.py:93-96, in the value dtype)."""
        if not self.config.deep_kv_rescale:
            return torch.ones(self.num_key_value_heads, device=self.q_proj.weight.device)
        return self.deep_v_scale.detach().to(kv_dtype).float()

    def blend_alpha(self, kv_dtype=torch.bfloat16) -> torch.Tensor:
        """The blend weight a = sigmoid(prev_chunk_alphas) in the cache's dtype, as fp32:
        the sigmoid of the bf16 logits rounded to bf16 for a bf16 cache
        (batching.py:1067-1079), the fp32 sigmoid for an fp32 one (modeling.py:115)."""
        return self.prev_chunk_alphas.detach().to(kv_dtype).sigmoid().float()

    def forward(self, hidden_states, position_embeddings, cache: PagedLastKVCache):
        B, L, _ = hidden_states.shape
        D, Hq, Hkv = self.head_dim, self.num_heads, self.num_key_value_heads
        meta = cache._meta if cache._meta is not None and cache._meta["n"] == L else cache.plan(L)
        fast = _fused_ok(self._qkv, [self.q_proj, self.k_proj, self.v_proj])
        if fast:
            qkv = _decode_linear(hidden_states, *self._qkv)
            if qkv is None:
                qkv = F.linear(hidden_states, *self._qkv)
            qkv = qkv.reshape(B * L, (Hq + 2 * Hkv) * D)
            q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:]
        else:
            q = self.q_proj(hidden_states).reshape(B * L, Hq * D)
            k = self.k_proj(hidden_states).reshape(B * L, Hkv * D)
            v = self.v_proj(hidden_states).reshape(B * L, Hkv * D)
        kv_dtype = cache.dtype  # bf16: the tensor-core kernels; fp32: the fp32 configuration's kernels
        if q.dtype != kv_dtype:
            q, k, v = q.to(kv_dtype), k.to(kv_dtype), v.to(kv_dtype)
        cs = None
        if not self.config.use_nope:
            cos, sin = position_embeddings
            # the (cos | sin) table is the same for every layer of a span: build it once
            if meta.get("cs_of") is not cos:
                meta["cs"] = torch.cat((cos[0, :, : D // 2], sin[0, :, : D // 2]), dim=-1).to(
                    torch.bfloat16 if kv_dtype == torch.bfloat16 else torch.float32).contiguous()
                meta["cs_of"] = cos
            cs = meta["cs"]
        s, inv, out_scale, q_w, k_w = self._layer_constants(kv_dtype)
        top = self.layer_idx == cache.num_layers - 1
        flat_k = cache.pool_k.view(-1, Hkv, D)
        flat_v = cache.pool_v.view(-1, Hkv, D)
        if "ring_slot_all" not in meta:  # every layer's ring slots of the span, one launch
            meta["ring_slot_all"] = meta["ring_tok"][None, :] + cache.ring_base_dev.to(torch.int64)[:, None] * PAGE_SIZE
        ring_slot = meta["ring_slot_all"][self.layer_idx]
        q_out = ops.rope_norm_append(
            q, k, v, meta["local_pos"], cs, q_w, k_w,
            self.config.rms_norm_eps, inv, ring_slot, flat_k, flat_v,
            meta["src_slot"] if top else None, flat_k if top else None, flat_v if top else None,
            error_word=cache.error_word, commit=cache.take_commit() if self.layer_idx == 0 else None)
        bt = meta["bt_all"][self.layer_idx]
        if kv_dtype == torch.float32:  # decode and spans alike (lkv_attention_paged_f32)
            out = ops.attention_paged_f32(q_out, cache.pool_k, cache.pool_v, bt, meta["seq_k"], meta["cu_q"],
                                          out_scale=out_scale, error_word=cache.error_word, max_pages=meta["W"])
        elif L == 1:
            out = ops.decode_paged(q_out, cache.pool_k, cache.pool_v, bt, meta["seq_k"], out_scale=out_scale,
                                   workspace=cache.workspace, max_pages=meta["W"],
                                   tables_ready=meta.get("tables_ready", False), l2_keep=True)
        else:
            out = ops.prefill_paged(q_out, cache.pool_k, cache.pool_v, bt, meta["seq_k"], meta["cu_q"], L,
                                    out_scale=out_scale, error_word=cache.error_word, max_pages=meta["W"])
        out = out.view(B, L, Hq * D).to(hidden_states.dtype)
        y = _decode_linear(out, self.o_proj.weight, self.o_proj.bias) if fast else None
        return y if y is not None else self.o_proj(out)


class LastKVDecoderLayer(nn.Module):
    def __init__(self, config, layer_idx):
        super().__init__()
        self.self_attn = LastKVAttention(config, layer_idx)
        self.mlp = MLP(config)
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)

    def forward(self, hidden_states, position_embeddings, cache):
        h, delta = self.forward_residual(hidden_states, None, position_embeddings, cache)
        return h + delta

    def forward_residual(self, residual, delta, position_embeddings, cache):
        """``(residual stream, pending delta) -> (residual stream, MLP output)``.

        The same arithmetic as ``forward`` (h = h + attn(norm(h)); h + mlp(norm(h))),
        with each residual add done inside the following RMSNorm kernel; the MLP
        output is returned un-added so the next layer's norm can absorb it.
        """
        h, x = self.input_layernorm.fused(residual, delta)
        h, x = self.post_attention_layernorm.fused(h, self.self_attn(x, position_embeddings, cache))
        return h, self.mlp(x)

    def fuse_projections_(self):
        self.self_attn.fuse_qkv_()
        self.mlp.fuse_()
        return self


class LastKVModel(nn.Module):
    def __init__(self, config: LastKVConfig):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList(LastKVDecoderLayer(config, i) for i in range(config.num_hidden_layers))
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.rotary_emb = RotaryEmbedding(config)

    def forward(self, input_ids, cache: PagedLastKVCache, *, inputs_embeds=None, position_ids=None):
        """Chunk loop of modeling.py:194-208: split at chunk boundaries, commit after all layers.
        ``position_ids`` [1 or B, length] (default: the cache positions) drive the rotary
        tables only, as in the reference (modeling.py:188-195)."""
        hidden = self.embed_tokens(input_ids) if inputs_embeds is None else inputs_embeds
        B, length, _ = hidden.shape
        if not length:
            raise ValueError("At least one new token is required")
        if cache.chunk_size != self.config.chunk_size or cache.num_layers != len(self.layers):
            raise ValueError("Cache architecture does not match this model")
        if position_ids is not None:
            position_ids = position_ids[None, :] if position_ids.ndim == 1 else position_ids
            if position_ids.shape[-1] != length or position_ids.shape[0] not in (1, B):
                raise ValueError("position_ids must describe the new input tokens")
            if position_ids.shape[0] != 1 and not bool((position_ids == position_ids[:1]).all()):
                raise RMarinBackendContractError("the paged cache advances all sequences together: "
                                                 "position_ids must be equal across the batch")
        C = self.config.chunk_size
        outputs = []
        start = 0
        while start < length:
            take = min(length - start, C - cache.seen_tokens % C)
            chunk = hidden[:, start:start + take]
            if position_ids is None:
                pos = torch.arange(cache.seen_tokens, cache.seen_tokens + take, device=hidden.device)[None]
            else:
                pos = position_ids[:1, start:start + take].to(hidden.device)
            position_embeddings = self.rotary_emb(chunk, pos)
            cache.plan(take)
            outputs.append(self.run_layers(chunk, position_embeddings, cache))
            cache.advance(take)
            if cache.seen_tokens % C == 0:
                cache.commit(self.blend_alpha(cache.dtype))
            start += take
        return outputs[0] if len(outputs) == 1 else torch.cat(outputs, dim=1)

    def run_layers(self, hidden, position_embeddings, cache):
        """All decoder layers and the final norm over one planned span."""
        residual, delta = hidden, None
        for layer in self.layers:
            residual, delta = layer.forward_residual(residual, delta, position_embeddings, cache)
        return self.norm.fused(residual, delta)[1]

    def blend_alpha(self, kv_dtype=torch.bfloat16) -> torch.Tensor:
        """Every layer's blend weights [L, Hkv] for a ``kv_dtype`` cache (cached; a state-dict
        load through ``load_reference_state_dict`` resets it)."""
        cached = getattr(self, "_alpha", None)
        if cached is None or cached[0] != kv_dtype:
            cached = (kv_dtype, torch.stack([l.self_attn.blend_alpha(kv_dtype) for l in self.layers]).contiguous())
            self._alpha = cached
        return cached[1]


class LastKVForCausalLM(nn.Module):
    """``CustomRecurrentMarinAKV254ReuseKVForCausalLM`` (modeling.py:215-293) on the B200 path."""

    def __init__(self, config: LastKVConfig):
        super().__init__()
        self.config = config
        self.model = LastKVModel(config)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)

    def fuse_projections_(self):
        """Inference fast path: each layer's q/k/v and gate/up projections become one
        GEMM each, and decode-sized calls (<= 16 rows) of every projection run on the
        tcgen05 decode GEMM (gate/up with the SiLU-and-mul in its epilogue).
        Parameter names and state-dict loading are unchanged; call after moving the
        model (a later move falls back to the module path)."""
        for layer in self.model.layers:
            layer.fuse_projections_()
        return self

    def new_cache(self, batch: int, max_tokens: int, **kw) -> PagedLastKVCache:
        """A paged cache for this model: fp32 keys and values for an fp32 model (the
        reference's fp32 arithmetic end to end), bf16 otherwise."""
        kw.setdefault("dtype", torch.float32 if self.lm_head.weight.dtype == torch.float32 else torch.bfloat16)
        return PagedLastKVCache(self.config, batch, max_tokens, device=self.lm_head.weight.device, **kw)

    def forward(self, input_ids, past_key_values: PagedLastKVCache, logits_to_keep: int = 0):
        if not isinstance(past_key_values, PagedLastKVCache):
            raise TypeError("Use a PagedLastKVCache created by this model")
        hidden = self.model(input_ids, past_key_values)
        if logits_to_keep:
            hidden = hidden[:, -logits_to_keep:]
        return self.lm_head(hidden), past_key_values

    @torch.no_grad()
    def generate_greedy(self, prompt, max_new_tokens: int, cache: PagedLastKVCache | None = None):
        cache = cache or self.new_cache(prompt.shape[0], prompt.shape[1] + max_new_tokens)
        logits, _ = self(prompt, cache, logits_to_keep=1)
        out = [prompt]
        nxt = logits[:, -1].float().argmax(-1, keepdim=True)
        for _ in range(max_new_tokens):
            out.append(nxt)
            if len(out) - 1 == max_new_tokens:
                break
            logits, _ = self(nxt, cache, logits_to_keep=1)
            nxt = logits[:, -1].float().argmax(-1, keepdim=True)
        return torch.cat(out, dim=1)

    def load_reference_state_dict(self, state: dict, strict: bool = True):
        """Load the reference's tensor names (strict, as modeling.py:243-249 requires)."""
        missing, unexpected = self.load_state_dict(state, strict=False)
        if strict and (missing or unexpected):
            raise ValueError(f"Checkpoint is not a strict LastKV model match: missing={missing}, "
                             f"unexpected={unexpected}")
        self.model._alpha = None
        return self
