"""ORACLE (test infrastructure, not product code).

A CPU restatement of LastKV's shared last-layer-KV attention path, written in
numpy (float64 accumulation unless stated).  It is the checker for the CUDA
kernels of ``lastkv_b200`` and the timed CPU baseline of ``bench.py``; the
product path never imports it.

Parity pin: ``tests/test_oracle_golden.py`` checks every function here that
has a counterpart in the reference against golden vectors produced by the
reference's own HF implementation (``tests/golden/make_golden.py`` imports
``lastkv.llm`` from the reference tree and records every attention call of
its cached chunk recurrence).  The vLLM fast path's Triton/FA3 arithmetic has
no shipped test vectors; its bf16 rounding points are restated from source
below and cross-checked only through the merged == HF equivalence.

Reference files are cited relative to the reference project root:
  HF path      llm/src/lastkv/llm/modeling.py
  vLLM path    vllm/src/lastkv/vllm/backends/rmarin_flashinfer/{fastpath,fused_qkv,batching}.py
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

# --------------------------------------------------------------------------
# bf16 helpers (round to nearest even, as torch/CUDA ``__float2bfloat16_rn``)
# --------------------------------------------------------------------------


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even); returns float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.float32("nan")
    return out


def bf16_bits(x) -> np.ndarray:
    """uint16 bit patterns of ``bf16_round(x)``."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits) -> np.ndarray:
    """float32 values of uint16 bf16 bit patterns."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def _fma32(a, b, c) -> np.ndarray:
    """fp32 fused multiply-add emulated in float64 (a*b is exact in float64)."""
    return (_f32(a).astype(np.float64) * _f32(b).astype(np.float64) + _f32(c).astype(np.float64)).astype(np.float32)


# --------------------------------------------------------------------------
# Cache append epilogue: RoPE -> Q/K RMSNorm -> V/s -> paged stores
# --------------------------------------------------------------------------


def rope_neox(x, cos, sin, *, bf16: bool = True) -> np.ndarray:
    """NeoX rotary over the full head: ``[x1*c - x2*s, x2*c + x1*s]``.

    HF form: ``apply_rotary_pos_emb`` (modeling.py:105, rotate_half).  vLLM
    fused form (fused_qkv.py:36-41): fp32 math, ``x*c - y*s`` contracted to one
    FMA, then a single bf16 rounding.  ``cos``/``sin`` hold the D/2 distinct
    frequencies, broadcastable to ``x[..., :D/2]``.
    """
    x = _f32(x)
    half = x.shape[-1] // 2
    xf, yf = x[..., :half], x[..., half:]
    c, s = _f32(cos), _f32(sin)
    r1 = _fma32(xf, c, -(yf * s))
    r2 = _fma32(yf, c, xf * s)
    out = np.concatenate([r1, r2], axis=-1)
    return bf16_round(out) if bf16 else out


def rms_norm(x, weight, eps: float, *, bf16: bool = True) -> np.ndarray:
    """RMSNorm over the last dim: ``x * rsqrt(mean(x^2) + eps) * w``.

    vLLM order (fused_qkv.py:42-55): fp32 sum of squares, one rounding of
    ``x * inv * w``.  HF ``LlamaRMSNorm`` (modeling.py:90-91,106) rounds
    ``x * inv`` to the input dtype before ``* w``; both agree in fp32.
    """
    x = _f32(x)
    var = (x.astype(np.float64) ** 2).sum(-1, keepdims=True) / x.shape[-1]
    inv = (1.0 / np.sqrt(var.astype(np.float32) + np.float32(eps))).astype(np.float32)
    out = x * inv * _f32(weight)
    return bf16_round(out) if bf16 else out


def v_over_s(v, inv_scale) -> np.ndarray:
    """Ring V in ``V/s`` units: ``bf16(v * fp32(1/s))`` (fused_qkv.py:83-86, fastpath.py:266)."""
    return bf16_round(_f32(v) * _f32(inv_scale))


def rope_norm_append(q, k, v, positions, cos_sin, q_w, k_w, eps, inv_scale,
                     ring_slot, ring_k, ring_v, src_slot=None, src_k=None, src_v=None):
    """Restates ``_fused_qkv_kernel`` (fused_qkv.py:58-90) on flat token views.

    q [T, Hq*D], k/v [T, Hkv*D] (bf16 values); cos_sin [maxpos, D] (cos | sin);
    ring_k/ring_v/src_k/src_v [slots, Hkv, D] are updated in place.
    Returns q_out [T, Hq, D].
    """
    q, k, v = _f32(q), _f32(k), _f32(v)
    T = q.shape[0]
    D = cos_sin.shape[-1]
    half = D // 2
    Hq, Hkv = q.shape[1] // D, k.shape[1] // D
    pos = np.asarray(positions, dtype=np.int64)
    cs = _f32(cos_sin)[pos]  # [T, D]
    cos = cs[:, None, :half]
    sin = cs[:, None, half:]
    q_out = rms_norm(rope_neox(q.reshape(T, Hq, D), cos, sin), q_w, eps)
    kn = rms_norm(rope_neox(k.reshape(T, Hkv, D), cos, sin), k_w, eps)
    v3 = v.reshape(T, Hkv, D)
    slots = np.asarray(ring_slot, dtype=np.int64)
    ring_k[slots] = kn
    ring_v[slots] = v_over_s(v3, _f32(inv_scale)[None, :, None])
    if src_slot is not None:
        ss = np.asarray(src_slot, dtype=np.int64)
        src_k[ss] = kn
        src_v[ss] = v3
    return q_out


def head_scale(x, scale) -> np.ndarray:
    """``x[t, h, :] *= s[h]`` with one bf16 rounding (fused_qkv.py:129-155)."""
    return bf16_round(_f32(x) * _f32(scale)[None, :, None])


# --------------------------------------------------------------------------
# Boundary commit: blend the finished chunk of every layer ring
# --------------------------------------------------------------------------


def blend_chunk(ring, raw, alpha) -> np.ndarray:
    """``ring = a*raw + (1-a)*ring`` with each torch op rounded to bf16.

    Restates ``_blend_kernel`` (fused_qkv.py:158-201) and the eager commit
    (batching.py:1135-1141): ``t1 = bf16(a*raw)``, ``ia = bf16(1-a)``,
    ``t3 = bf16(ia*ring)``, ``bf16(t1 + t3)``.  ring [L, C, H, D], raw [C, H, D],
    alpha [L, H] (bf16-exact sigmoid values).  V is blended in ``V/s`` units
    (rings hold V/s and the shared slab holds raw V, batching.py:1127-1129).
    """
    a = _f32(alpha)[:, None, :, None]
    ia = bf16_round(np.float32(1.0) - a)
    t1 = bf16_round(a * _f32(raw)[None])
    t3 = bf16_round(ia * _f32(ring))
    return bf16_round(t1 + t3)


def rope_hf_f32(x, cos, sin) -> np.ndarray:
    """fp32 ``apply_rotary_pos_emb`` as the HF module evaluates it (modeling.py:105):
    ``x*cos + rotate_half(x)*sin``, each product and the sum rounded to fp32.
    ``cos``/``sin`` hold the D/2 distinct frequencies."""
    x = _f32(x)
    half = x.shape[-1] // 2
    xf, yf = x[..., :half], x[..., half:]
    c, s = _f32(cos), _f32(sin)
    return np.concatenate([xf * c + (-yf) * s, yf * c + xf * s], axis=-1).astype(np.float32)


def rms_norm_hf_f32(x, weight, eps: float) -> np.ndarray:
    """fp32 ``LlamaRMSNorm`` (modeling.py:90-91, 106): ``w * (x * (1/sqrt(mean(x^2) + eps)))``
    in fp32 (the mean summed in float64 here; the kernel's fp32 order differs by an ulp)."""
    x = _f32(x)
    var = ((x.astype(np.float64) ** 2).sum(-1, keepdims=True) / x.shape[-1]).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    return (_f32(weight) * (x * inv)).astype(np.float32)


def blend_chunk_f32(ring, raw, alpha) -> np.ndarray:
    """fp32 recent-chunk blend ``a*top + (1-a)*layer`` (modeling.py:115-119 in fp32): the two
    products and their sum each rounded to fp32.  ring [L, C, H, D], raw [C, H, D], alpha [L, H]."""
    a = _f32(alpha)[:, None, :, None]
    return (a * _f32(raw)[None] + (np.float32(1.0) - a) * _f32(ring)).astype(np.float32)


def alpha_from_logits(logits) -> np.ndarray:
    """``sigmoid`` evaluated on bf16 logits and rounded to bf16 (batching.py:1067-1079)."""
    x = bf16_round(logits).astype(np.float64)
    return bf16_round((1.0 / (1.0 + np.exp(-x))).astype(np.float32))


# --------------------------------------------------------------------------
# Paged attention (the merged one-call-per-layer form)
# --------------------------------------------------------------------------


def gather_pages(pool, pages, n):
    """Token-major ``[n, Hkv, D]`` view of the first n tokens of a page list."""
    pool = np.asarray(pool)
    page = pool.shape[1]
    npages = -(-n // page)
    flat = pool[np.asarray(pages[:npages], dtype=np.int64)].reshape(npages * page, *pool.shape[2:])
    return flat[:n]


def attention(q, k, v, *, scale: float, causal: bool = True, dtype=np.float64):
    """softmax(q k^T * scale) v with GQA broadcast and bottom-right causal mask.

    q [Lq, Hq, D], k/v [Lk, Hkv, D].  Query i sits at key position
    ``Lk - Lq + i`` (modeling.py:124-130); decode (Lq=1) is unmasked.
    Returns (out [Lq, Hq, D], lse [Lq, Hq]) with lse in natural log.
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    Lq, Hq, D = q.shape
    Lk, Hkv, _ = k.shape
    g = Hq // Hkv
    qg = q.reshape(Lq, Hkv, g, D)
    s = np.einsum("qhgd,khd->hgqk", qg, k) * dtype(scale)
    if causal and Lq > 1:
        qpos = np.arange(Lq)[:, None] + (Lk - Lq)
        mask = np.arange(Lk)[None, :] > qpos
        s = np.where(mask[None, None], -np.inf, s)
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(-1, keepdims=True)
    o = np.einsum("hgqk,khd->qhgd", p / l, v).reshape(Lq, Hq, D)
    lse = (m + np.log(l))[..., 0]  # [Hkv, g, Lq]
    return o, lse.reshape(Hq, Lq).T


def paged_attention(q, pool_k, pool_v, block_table, seq_k, cu_q, *, scale: float,
                    out_scale=None, causal: bool = True, dtype=np.float64):
    """Varlen paged attention over ``[older shared pages | ring pages]``.

    Restates the merged call ``flash_attn_varlen_func(q, pool_k, pool_v,
    cu_seqlens_q, seqused_k, causal=True, block_table=bt_all[l])`` followed by
    ``head_scale_`` (fastpath.py:643-650).  q [T, Hq, D]; pool [P, page, Hkv, D];
    block_table [B, W]; seq_k [B]; cu_q [B+1]; out_scale [Hq] or None.
    Returns (out [T, Hq, D], lse [T, Hq]); lse excludes out_scale.
    """
    q = np.asarray(q)
    T, Hq, D = q.shape
    out = np.zeros((T, Hq, D), dtype=dtype)
    lse = np.full((T, Hq), -np.inf, dtype=dtype)
    for b in range(len(seq_k)):
        q0, q1 = int(cu_q[b]), int(cu_q[b + 1])
        n = int(seq_k[b])
        if q1 == q0 or n == 0:
            continue
        kb = gather_pages(pool_k, block_table[b], n)
        vb = gather_pages(pool_v, block_table[b], n)
        o, l = attention(q[q0:q1], kb, vb, scale=scale, causal=causal, dtype=dtype)
        out[q0:q1] = o
        lse[q0:q1] = l
    if out_scale is not None:
        out = out * np.asarray(out_scale, dtype=dtype)[None, :, None]
    return out, lse


def merge_states(o_a, lse_a, o_b, lse_b):
    """Exact LSE merge of two attention partials over disjoint key sets.

    Restates ``flashinfer.cascade.merge_state`` / ``vllm merge_attn_states`` as
    used at flashinfer_executor.py:185-231 and fastpath.py:719.  o [T, H, D],
    lse [T, H] (natural log; -inf marks an empty partial).
    """
    o_a, o_b = np.asarray(o_a, np.float64), np.asarray(o_b, np.float64)
    lse_a, lse_b = np.asarray(lse_a, np.float64), np.asarray(lse_b, np.float64)
    m = np.maximum(lse_a, lse_b)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    wa = np.where(np.isfinite(lse_a), np.exp(lse_a - m_safe), 0.0)
    wb = np.where(np.isfinite(lse_b), np.exp(lse_b - m_safe), 0.0)
    tot = wa + wb
    tot_safe = np.where(tot > 0, tot, 1.0)
    o = (o_a * wa[..., None] + o_b * wb[..., None]) / tot_safe[..., None]
    lse = np.where(tot > 0, m_safe + np.log(tot_safe), -np.inf)
    return o, lse


def merge_many(os_, lses):
    """Fold ``merge_states`` over a list of partials (the context-parallel combine)."""
    o, l = os_[0], lses[0]
    for o2, l2 in zip(os_[1:], lses[1:]):
        o, l = merge_states(o, l, o2, l2)
    return o, l


# --------------------------------------------------------------------------
# HF chunk-recurrence history (what the merged form must reproduce)
# --------------------------------------------------------------------------


def hf_history(deep_k, deep_v, prev_k, prev_v, cur_k, cur_v, alpha_logits, v_scale, chunk):
    """Compose [older*s | blend(recent) | current] for one layer (modeling.py:109-122).

    Shapes [Hkv, T, D] (batch dimension dropped).  deep_* hold the final
    layer's K/V of every completed chunk (or None); prev_* the same layer's
    previous chunk.  fp32 math, as the golden vectors are fp32.
    """
    keys, values = [], []
    s = _f32(v_scale)[:, None, None]
    if deep_k is not None:
        old = deep_k.shape[1] - chunk
        if old:
            keys.append(deep_k[:, :old])
            values.append(deep_v[:, :old] * s)
        a = (1.0 / (1.0 + np.exp(-_f32(alpha_logits).astype(np.float64)))).astype(np.float32)[:, None, None]
        keys.append(a * deep_k[:, old:] + (1 - a) * prev_k)
        values.append(a * (deep_v[:, old:] * s) + (1 - a) * prev_v)
    keys.append(cur_k)
    values.append(cur_v)
    return np.concatenate(keys, axis=1), np.concatenate(values, axis=1)


# --------------------------------------------------------------------------
# Pool layout and per-row page plan (vLLM merged pool)
# --------------------------------------------------------------------------


@dataclass
class PoolLayout:
    """Merged K/V page pool (batching.py:1999-2016, fastpath.py:153-161).

    Pages ``[0, src_pages)`` hold the shared final-layer history (raw K, raw V);
    layer ``l`` owns ring pages ``src_pages + l*ring_stride + slot*ring_pages +
    j`` with ``ring_pages = 2C/page`` and one scratch page at the end of each
    layer's stride.  Rings hold K and ``V/s_l``.
    """

    num_layers: int
    chunk: int
    page: int
    num_slots: int
    src_pages: int

    @property
    def ring_pages(self) -> int:
        return 2 * self.chunk // self.page

    @property
    def ring_tokens(self) -> int:
        return 2 * self.chunk

    @property
    def ring_stride(self) -> int:
        return self.ring_pages * self.num_slots + 1

    @property
    def total_pages(self) -> int:
        return self.src_pages + self.num_layers * self.ring_stride

    def ring_base(self, layer: int) -> int:
        return self.src_pages + layer * self.ring_stride


def row_plan(layout: PoolLayout, slot: int, position: int, n: int, src_page_list):
    """Per-row plan of one span of n query tokens starting at ``position``.

    Restates ``_row_plan`` (fastpath.py:427-454) with the older pages taken
    from the sequence's shared-history page list.  Returns
    (ring_token_of_first, local_pages (layer-relative), nsrc, seq_k).
    """
    C, P = layout.chunk, layout.page
    last = position + n - 1
    cur = (last // C) * C
    rec = max(0, cur - C)
    ring_tok = slot * layout.ring_tokens + (position % layout.ring_tokens)
    window = last + 1 - rec
    npages = -(-window // P)
    first = (rec // P) % layout.ring_pages
    local = [slot * layout.ring_pages + ((first + j) % layout.ring_pages) for j in range(npages)]
    nsrc = rec // P
    seq_k = (nsrc + npages - 1) * P + (window - (npages - 1) * P)
    return ring_tok, local, nsrc, seq_k, list(src_page_list[:nsrc])


def merged_block_table(layout: PoolLayout, layer: int, src_pages, local_pages) -> list[int]:
    """One row of ``bt_all[layer]`` = older pages | layer ring pages (fastpath.py:407-424)."""
    base = layout.ring_base(layer)
    return list(src_pages) + [base + p for p in local_pages]


@dataclass
class PagedLastKV:
    """Oracle-side state machine of the merged paged pool for B sequences.

    Drives the same writes as the vLLM fast path: per-layer append of K and
    ``V/s_l`` into the ring (fused_qkv.py:80-86), the top layer's raw K/V into
    the shared pages (fused_qkv.py:87-90), and the boundary blend of every ring
    chunk when a chunk completes (batching.py:1099-1144).  ``bf16`` selects
    whether stores are rounded like the bf16 pool.
    """

    layout: PoolLayout
    hkv: int
    d: int
    batch: int
    alpha: np.ndarray  # [L, Hkv] blend weights (already sigmoid'ed)
    v_scale: np.ndarray  # [L, Hkv]
    bf16: bool = False
    src_page_lists: list = field(default_factory=list)
    seen: list = field(default_factory=list)

    def __post_init__(self):
        lay = self.layout
        self.pool_k = np.zeros((lay.total_pages, lay.page, self.hkv, self.d), np.float32)
        self.pool_v = np.zeros_like(self.pool_k)
        if not self.src_page_lists:
            per = lay.src_pages // self.batch
            self.src_page_lists = [list(range(b * per, (b + 1) * per)) for b in range(self.batch)]
        self.seen = [0] * self.batch
        self.committed = [0] * self.batch

    def _round(self, x):
        return bf16_round(x) if self.bf16 else _f32(x)

    def _flat(self, pool):
        lay = self.layout
        return pool.reshape(lay.total_pages * lay.page, self.hkv, self.d)

    def _src_token(self, b, pos):
        P = self.layout.page
        return self.src_page_lists[b][pos // P] * P + pos % P

    def _ring_token(self, layer, b, pos):
        lay = self.layout
        rt = b * lay.ring_tokens + pos % lay.ring_tokens
        return lay.ring_base(layer) * lay.page + rt

    def append(self, layer: int, b: int, k, v, start: int):
        """Store n new tokens (k, v [n, Hkv, D], post RoPE/norm) of sequence b."""
        fk, fv = self._flat(self.pool_k), self._flat(self.pool_v)
        inv = (1.0 / _f32(self.v_scale[layer]).astype(np.float32)).astype(np.float32)
        for i in range(k.shape[0]):
            rt = self._ring_token(layer, b, start + i)
            fk[rt] = self._round(k[i])
            vs = _f32(v[i]) * inv[:, None]
            fv[rt] = self._round(vs)
            if layer == self.layout.num_layers - 1:
                st = self._src_token(b, start + i)
                fk[st] = self._round(k[i])
                fv[st] = self._round(v[i])

    def commit_if_boundary(self, b: int, seen_after: int):
        """Blend the chunk that just completed into every layer ring."""
        C = self.layout.chunk
        if seen_after % C or seen_after == self.committed[b]:
            return
        end = seen_after
        fk, fv = self._flat(self.pool_k), self._flat(self.pool_v)
        src = [self._src_token(b, p) for p in range(end - C, end)]
        raw_k, raw_v = fk[src], fv[src]
        for layer in range(self.layout.num_layers):
            rows = [self._ring_token(layer, b, p) for p in range(end - C, end)]
            a = _f32(self.alpha[layer])
            if self.bf16:
                ring = np.stack([fk[rows], fv[rows]])[:, None]  # [2, 1, C, H, D]
                fk[rows] = blend_chunk(ring[0], raw_k, a[None])[0]
                fv[rows] = blend_chunk(ring[1], raw_v, a[None])[0]
            else:
                aa = a[None, :, None]
                fk[rows] = aa * raw_k + (1 - aa) * fk[rows]
                fv[rows] = aa * raw_v + (1 - aa) * fv[rows]
        self.committed[b] = end

    def block_table(self, layer: int, b: int, position: int, n: int):
        lay = self.layout
        _, local, nsrc, seq_k, src = row_plan(lay, b, position, n, self.src_page_lists[b])
        return merged_block_table(lay, layer, src, local), seq_k

    def attend(self, layer: int, b: int, q, position: int, *, scale: float):
        """Merged attention of n queries (q [n, Hq, D]) at ``position``, times s_l."""
        n = q.shape[0]
        bt, seq_k = self.block_table(layer, b, position, n)
        hq = q.shape[1]
        s_q = np.repeat(_f32(self.v_scale[layer]), hq // self.hkv)
        out, _ = paged_attention(q, self.pool_k, self.pool_v, [bt], [seq_k], [0, n],
                                 scale=scale, out_scale=s_q)
        return out


def chunk_aligned_new_tokens(num_computed: int, num_new: int, chunk: int) -> int:
    """Cap a span at the next chunk boundary (batching.py:88-105)."""
    if num_computed < 0 or chunk < 1:
        raise ValueError("invalid scheduling state")
    if num_new < 1:
        return num_new
    nxt = (num_computed // chunk + 1) * chunk
    return min(num_new, nxt - num_computed)


# --------------------------------------------------------------------------
# Wan causal block attention over a shared final-layer history
# --------------------------------------------------------------------------


def wan_rope_angles(frames: int, fh: int, fw: int, start_frame: int, head_dim: int, theta: float = 10000.0):
    """Angles [T, D/2] of Wan's causal 3-D RoPE for a block of ``frames`` frames.

    Restates ``rope_params`` (videogen/src/lastkv/videogen/layers.py:24-31), the
    frequency table split (model.py:568; layers.py:135-136) and
    ``causal_rope_apply`` (layers.py:126-154): complex pair i of a token at
    (frame f, row h, col w) rotates by f*inv_t[i] (i < c - 2(c//3)), then
    h*inv_h, then w*inv_w, with each table over its own sub-dimension.
    """
    d = head_dim
    dims = [d - 4 * (d // 6), 2 * (d // 6), 2 * (d // 6)]
    inv = [1.0 / theta ** (np.arange(0, dd, 2, dtype=np.float64) / dd) for dd in dims]
    f, h, w = np.meshgrid(np.arange(frames) + start_frame, np.arange(fh), np.arange(fw), indexing="ij")
    return np.concatenate([f.reshape(-1, 1) * inv[0][None], h.reshape(-1, 1) * inv[1][None],
                           w.reshape(-1, 1) * inv[2][None]], axis=1)


def rope_interleaved(x, angles) -> np.ndarray:
    """Rotate pairs (2i, 2i+1) of x [T, H, D] by angles [T, D/2] in float64 (layers.py:141-150)."""
    x = np.asarray(x, dtype=np.float64)
    c = np.cos(angles)[:, None, :]
    s = np.sin(angles)[:, None, :]
    out = np.empty_like(x)
    out[..., 0::2] = x[..., 0::2] * c - x[..., 1::2] * s
    out[..., 1::2] = x[..., 0::2] * s + x[..., 1::2] * c
    return out


class WanHistory:
    """Per-layer history of one sequence, composed as the reference composes it.

    ``history(layer, start)`` restates ``_compose_history_kv`` (model.py:217-272)
    with ``history_kv`` (cache.py:58-65) and ``_blend_first_local_kv_segment``
    (model.py:173-195): [per-layer prefix | shared final-layer K/V | previous
    block = a*shared + (1-a)*layer-local, first-frame tokens kept local].
    ``commit(start, kvs)`` restates ``_update_caches_akv`` (model.py:716-729).
    Arrays are [T, H, D]; ``alpha`` [L, H] are the sigmoid'ed block weights.
    """

    def __init__(self, num_layers: int, prefix_tokens: int, block_tokens: int, alpha):
        self.L, self.P, self.BT = num_layers, prefix_tokens, block_tokens
        self.alpha = np.asarray(alpha, dtype=np.float64)
        self.prefix = [None] * num_layers
        self.shared = None
        self.curr = [None] * num_layers

    def history(self, layer: int, start: int):
        if start <= 0:
            return None
        P = self.P
        sk, sv = self.shared
        pk, pv = self.prefix[layer]
        keep = min(start, P)
        deep_k = np.concatenate([pk[:keep], sk[keep:start]]) if start > keep else pk[:start]
        deep_v = np.concatenate([pv[:keep], sv[keep:start]]) if start > keep else pv[:start]
        prev_start = start - min(self.BT, start)
        ck, cv = self.curr[layer]
        a = self.alpha[layer][None, :, None]
        bk = a * deep_k[prev_start:start] + (1 - a) * ck
        bv = a * deep_v[prev_start:start] + (1 - a) * cv
        keep_n = min(max(P - prev_start, 0), start - prev_start)
        if keep_n:
            bk[:keep_n], bv[:keep_n] = ck[:keep_n], cv[:keep_n]
        return (np.concatenate([deep_k[:prev_start], bk]), np.concatenate([deep_v[:prev_start], bv]))

    def commit(self, start: int, kvs):
        top_k, top_v = kvs[-1]
        end = start + top_k.shape[0]
        if self.shared is None:
            self.shared = (top_k.copy(), top_v.copy())
        else:
            self.shared = (np.concatenate([self.shared[0], top_k]), np.concatenate([self.shared[1], top_v]))
        for layer, (k, v) in enumerate(kvs):
            if start < self.P:
                n = min(end, self.P) - start
                pk = k[:n] if self.prefix[layer] is None else np.concatenate([self.prefix[layer][0], k[:n]])
                pv = v[:n] if self.prefix[layer] is None else np.concatenate([self.prefix[layer][1], v[:n]])
                self.prefix[layer] = (pk, pv)
            self.curr[layer] = (k.copy(), v.copy())


# --------------------------------------------------------------------------
# CPU baseline: the reference's own per-layer computation (torch, CPU)
# --------------------------------------------------------------------------


def reference_layer_step_cpu(query, deep_k, deep_v, prev_k, prev_v, cur_k, cur_v,
                             alpha_logits, v_scale, chunk):
    """One decode layer-step exactly as the HF reference computes it on CPU.

    Compose [older*s | blend(recent) | current] with ``torch.cat``
    (modeling.py:109-122), then ``F.scaled_dot_product_attention(...,
    enable_gqa=True)`` (modeling.py:143-146).  Inputs are torch tensors
    [B, H, T, D]; used only to time the reference's CPU path in ``bench.py``.
    """
    import torch
    import torch.nn.functional as F

    scale = v_scale.to(deep_v.dtype).view(1, -1, 1, 1)
    old = deep_k.shape[2] - chunk
    keys = [deep_k[:, :, :old]]
    values = [deep_v[:, :, :old] * scale]
    a = alpha_logits.sigmoid().to(cur_k.dtype).view(1, -1, 1, 1)
    keys.append(a * deep_k[:, :, old:] + (1 - a) * prev_k)
    values.append(a * (deep_v[:, :, old:] * scale) + (1 - a) * prev_v)
    keys.append(cur_k)
    values.append(cur_v)
    full_k, full_v = torch.cat(keys, dim=2), torch.cat(values, dim=2)
    causal = query.shape[2] == full_k.shape[2]
    return F.scaled_dot_product_attention(query, full_k, full_v, is_causal=causal,
                                          enable_gqa=query.shape[1] != full_k.shape[1])


def rope_cos_sin(max_pos: int, dim: int, theta: float) -> np.ndarray:
    """Plain (unscaled) NeoX cos|sin cache ``[max_pos, D]`` in fp32."""
    inv = 1.0 / (theta ** (np.arange(0, dim, 2, dtype=np.float64) / dim))
    t = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.concatenate([np.cos(t), np.sin(t)], axis=-1).astype(np.float32)


__all__ = [name for name in dir() if not name.startswith("_")] + ["math"]
