"""Wan causal block attention over the shared final-layer history on B200.

Reference: the AKV2541 reuse-KV Wan model (videogen/src/lastkv/videogen/):
a block of ``frames_per_block`` latent frames attends, non-causally, to
[per-layer first-frame prefix | shared final-layer K/V | previous block blended
``a*shared + (1-a)*layer`` (first-frame tokens kept local)] followed by its own
K/V (model.py:217-272, 372-390), and after the clean pass every layer's block is
committed (model.py:716-729, cache.py:39-65).

Layout (bf16 pool ``[pages, 16, H, D]``, pages of 16 tokens):
* shared pages  - final-layer K/V of every token of every sequence;
* prefix pages  - per (layer, sequence): keys [0, 16*PP), the layer's own first
  frame followed by shared values up to the page boundary;
* window pages  - per (layer, sequence), two buffers used by alternate blocks:
  keys [Pw, S + block) with Pw = the page-aligned start at or below the previous
  block: shared values up to the previous block, the blended previous block,
  then the current block written by the append kernel.
Block n's key list is [prefix pages | shared pages | window pages]; every
segment boundary that is not a multiple of 16 (1560-token frames,
4680-token blocks) lives inside a per-layer page, so no K/V is ever composed
with ``torch.cat``.  The commit is one token-level gather/blend launch.
"""

from __future__ import annotations

import numpy as np
import torch

from . import ops
from .contract import PAGE_SIZE, RMarinBackendContractError


def wan_rope_table(frames: int, fh: int, fw: int, start_frame: int, head_dim: int,
                   theta: float = 10000.0) -> np.ndarray:
    """fp32 [frames*fh*fw, D] = cos | sin of Wan's causal 3-D RoPE angles.

    Pair i of a token at (frame f, row h, col w) rotates by f*inv_t[i] for the
    first D/2 - 2*(D/2//3) pairs, then h*inv_h, then w*inv_w, each inverse
    frequency table over its own sub-dimension (videogen layers.py:24-31,
    126-154; model.py:568).  Angles in float64, cos/sin rounded once to fp32.
    """
    d = head_dim
    dims = [d - 4 * (d // 6), 2 * (d // 6), 2 * (d // 6)]
    inv = [1.0 / theta ** (np.arange(0, dd, 2, dtype=np.float64) / dd) for dd in dims]
    f, h, w = np.meshgrid(np.arange(frames) + start_frame, np.arange(fh), np.arange(fw), indexing="ij")
    ang = np.concatenate([f.reshape(-1, 1) * inv[0][None], h.reshape(-1, 1) * inv[1][None],
                          w.reshape(-1, 1) * inv[2][None]], axis=1)
    return np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(np.float32)


class WanSharedKVCache:
    """Paged shared-history cache of a Wan model for ``batch`` videos."""

    def __init__(self, *, num_layers: int, batch: int, num_heads: int, head_dim: int, frame_h: int, frame_w: int,
                 frames_per_block: int, max_frames: int, prefix_tokens: int, device=None, page_order=None):
        P = PAGE_SIZE
        self.L, self.B, self.H, self.D = num_layers, batch, num_heads, head_dim
        self.fh, self.fw, self.fpb = frame_h, frame_w, frames_per_block
        self.frame_tokens = frame_h * frame_w
        self.block = self.frame_tokens * frames_per_block
        self.max_tokens = self.frame_tokens * max_frames
        self.prefix = prefix_tokens
        self.pp = -(-prefix_tokens // P)  # prefix pages
        if self.pp * P > (self.block // P) * P:
            raise RMarinBackendContractError("the prefix must end (page-rounded) inside the first block")
        self.wp = -(-(2 * self.block + P - 1) // P)  # window pages per buffer
        self.src_pp = -(-self.max_tokens // P)
        self.device = torch.device(device or "cuda")
        n_src = batch * self.src_pp
        order = np.arange(n_src) if page_order is None else np.asarray(page_order)
        self.src_table = order.reshape(batch, self.src_pp).astype(np.int64)
        self.prefix_base = n_src                                         # [L, B, pp]
        self.window_base = self.prefix_base + num_layers * batch * self.pp  # [L, B, 2, wp]
        self.num_pages = self.window_base + num_layers * batch * 2 * self.wp
        shape = (self.num_pages, P, num_heads, head_dim)
        self.pool_k = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.pool_v = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.error_word = torch.zeros(4, dtype=torch.int32, device=self.device)
        self.n = -1
        self.committed = -1

    # -- addressing (host)
    def prefix_page(self, layer, b, j):
        return self.prefix_base + (layer * self.B + b) * self.pp + j

    def window_page(self, layer, b, parity, j):
        return self.window_base + ((layer * self.B + b) * 2 + parity) * self.wp + j

    def window_start(self, n: int) -> int:
        """First key of block n's window buffer (page-aligned, at or below the previous block)."""
        return 0 if n <= 1 else ((n - 1) * self.block // PAGE_SIZE) * PAGE_SIZE

    def _src_slot(self, b, t):
        return self.src_table[b, t // PAGE_SIZE] * PAGE_SIZE + t % PAGE_SIZE

    def _win_slot(self, layer, b, n, t):
        w = t - self.window_start(n)
        return self.window_page(layer, b, n % 2, w // PAGE_SIZE) * PAGE_SIZE + w % PAGE_SIZE

    # -- per block
    def begin_block(self, n: int):
        """Block tables, append slots and RoPE table for block n (start = n * block tokens)."""
        if n != self.committed + 1:
            raise RMarinBackendContractError("blocks must be processed in order, each committed before the next")
        P, S, BT = PAGE_SIZE, n * self.block, self.block
        if S + BT > self.max_tokens:
            raise RMarinBackendContractError("cache capacity exceeded")
        pw = self.window_start(n)
        n_win = -(-(S + BT - pw) // P)
        if n >= 2:
            n_src = (pw - self.pp * P) // P
            width = self.pp + n_src + n_win
        else:
            n_src, width = 0, n_win
        bt = np.zeros((self.L, self.B, width), np.int32)
        toks = np.arange(S, S + BT)
        ring = np.zeros((self.L, self.B * BT), np.int64)
        src = np.zeros(self.B * BT, np.int64)
        for b in range(self.B):
            src[b * BT:(b + 1) * BT] = self._src_slot(b, toks)
            for layer in range(self.L):
                row = []
                if n >= 2:
                    row += [self.prefix_page(layer, b, j) for j in range(self.pp)]
                    row += list(self.src_table[b, self.pp:self.pp + n_src])
                row += [self.window_page(layer, b, n % 2, j) for j in range(n_win)]
                bt[layer, b] = row
                ring[layer, b * BT:(b + 1) * BT] = self._win_slot(layer, b, n, toks)
        dev = self.device
        cs = wan_rope_table(self.fpb, self.fh, self.fw, n * self.fpb, self.D)
        self.meta = {
            "n": n, "W": width,
            "bt": torch.from_numpy(bt).to(dev),
            "ring": torch.from_numpy(ring).to(dev),
            "src": torch.from_numpy(src).to(dev),
            "seq_k": torch.full((self.B,), S + BT, dtype=torch.int32, device=dev),
            "cu_q": torch.arange(0, (self.B + 1) * BT, BT, dtype=torch.int32, device=dev),
            "pos": torch.arange(BT, dtype=torch.int64, device=dev).repeat(self.B),
            "cos_sin": torch.from_numpy(cs).to(dev),
        }
        self.n = n
        return self.meta

    def commit_block(self, alpha: torch.Tensor):
        """After the clean pass of block n: prefix (block 0) and block n+1's window buffer.

        alpha: fp32 [L, H] = sigmoid of the per-layer, per-head block weights.
        """
        n = self.n
        P, S, BT, pre = PAGE_SIZE, n * self.block, self.block, self.prefix
        dst, sa, sb, row = [], [], [], []
        nxt = n + 1
        pw_next = self.window_start(nxt)
        for layer in range(self.L):
            for b in range(self.B):
                if n == 0:  # per-layer prefix: own first frame, then shared values to the page boundary
                    t = np.arange(self.pp * P)
                    dst.append(self.prefix_base * P + ((layer * self.B + b) * self.pp) * P + t)
                    local = t < pre
                    sa.append(np.where(local, -1, self._src_slot(b, t)))
                    sb.append(np.where(local, self._win_slot(layer, b, n, t), -1))
                    row.append(np.full(t.size, layer))
                if S + BT >= self.max_tokens:
                    continue
                # window buffer of block n+1: shared values [pw_next, S), blended block n [S, S+BT)
                t = np.arange(pw_next, S + BT)
                d = self._win_slot(layer, b, nxt, t)
                in_block = t >= S
                first_frame = t < pre
                a = np.where(first_frame, -1, self._src_slot(b, t))
                bb = np.where(in_block, self._win_slot(layer, b, n, np.maximum(t, S)), -1)
                bb = np.where(in_block, bb, -1)
                dst.append(d)
                sa.append(a)
                sb.append(bb)
                row.append(np.full(t.size, layer))
        if dst:
            dev = self.device
            ops.gather_blend(self.pool_k, self.pool_v, torch.from_numpy(np.concatenate(dst)).to(dev),
                             torch.from_numpy(np.concatenate(sa)).to(dev), torch.from_numpy(np.concatenate(sb)).to(dev),
                             torch.from_numpy(np.concatenate(row).astype(np.int32)).to(dev),
                             alpha.float().contiguous(), error_word=self.error_word)
        self.committed = n

    def check_errors(self):
        e = self.error_word.cpu().tolist()
        if e[0]:
            raise RMarinBackendContractError(f"device error word set: {e}")


def wan_block_attention(qn, kn, v, cache: WanSharedKVCache, layer: int):
    """One layer of block attention.

    qn, kn: [B, T, H*D] bf16, already RMS-normalised over the model dim (Wan
    norms before RoPE, model.py:277-279); v: [B, T, H*D].  Applies the 3-D RoPE,
    stores this block's K/V (the last layer also into the shared pages) and
    attends non-causally over the block's key list.  Returns [B, T, H, D] bf16.
    """
    m = cache.meta
    B, T, _ = qn.shape
    H, D = cache.H, cache.D
    flat_k = cache.pool_k.view(-1, H, D)
    flat_v = cache.pool_v.view(-1, H, D)
    top = layer == cache.L - 1
    q = ops.rope_norm_append(
        qn.reshape(B * T, H * D), kn.reshape(B * T, H * D), v.reshape(B * T, H * D), m["pos"], m["cos_sin"],
        None, None, 0.0, None, m["ring"][layer], flat_k, flat_v,
        m["src"] if top else None, flat_k if top else None, flat_v if top else None,
        error_word=cache.error_word, interleaved=True)
    out = ops.prefill_paged(q, cache.pool_k, cache.pool_v, m["bt"][layer], m["seq_k"], m["cu_q"], T, causal=False,
                            error_word=cache.error_word, max_pages=m["W"])
    return out.view(B, T, H, D)
