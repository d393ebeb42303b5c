"""Torch-facing wrappers of the CUDA kernels (device tensors in, device tensors out).

Every function validates shapes/dtypes on the host, passes raw pointers to the
C ABI on the current torch stream and raises ``RMarinBackendContractError`` on
any nonzero status.  None of them allocates inside a CUDA-graph capture when
the caller passes ``out``/``workspace`` buffers.
"""

from __future__ import annotations

import ctypes
import functools
import os
from typing import NamedTuple, Optional

import torch

from . import _capi
from .contract import PAGE_SIZE, RMarinBackendContractError, require_heads


# lkv_decode_paged / lkv_decode_paged_cp flags (include/lastkv_b200.h): the tables predate the PDL chain;
# the oldest pages of each sequence stay in L2 for the next call over the same history
DECODE_TABLES_READY = 1
DECODE_L2_KEEP = 2
# lkv_rope_norm_append flag: every tensor fp32 (the fp32 model configuration)
APPEND_FP32 = 4


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RMarinBackendContractError(msg)


# LKV_NVTX=1: every kernel-launching op runs inside an NVTX range "lkv.<op>" (for timeline
# and ncu --nvtx captures); off by default, so the ops carry no range overhead.
_NVTX = os.environ.get("LKV_NVTX") == "1"


def _traced(fn):
    if not _NVTX:
        return fn
    name = "lkv." + fn.__name__

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        with torch.cuda.nvtx.range(name):
            return fn(*args, **kwargs)

    return wrapper


def _check_pool_f32(pool_k, pool_v):
    _require(pool_k.is_cuda and pool_v.is_cuda, "pools must be CUDA tensors")
    _require(pool_k.dtype == torch.float32 and pool_v.dtype == torch.float32, "pools must be fp32")
    _require(pool_k.dim() == 4 and pool_k.shape == pool_v.shape, "pools must be [pages, 16, Hkv, D] and equal")
    _require(pool_k.shape[1] == PAGE_SIZE, f"page size must be {PAGE_SIZE}")
    _require(pool_k.is_contiguous() and pool_v.is_contiguous(), "pools must be contiguous")


def _check_pool(pool_k, pool_v):
    _require(pool_k.is_cuda and pool_v.is_cuda, "pools must be CUDA tensors")
    _require(pool_k.dtype == torch.bfloat16 and pool_v.dtype == torch.bfloat16, "pools must be bf16")
    _require(pool_k.dim() == 4 and pool_k.shape == pool_v.shape, "pools must be [pages, 16, Hkv, D] and equal")
    _require(pool_k.shape[1] == PAGE_SIZE, f"page size must be {PAGE_SIZE}")
    _require(pool_k.is_contiguous() and pool_v.is_contiguous(), "pools must be contiguous")


class Workspace:
    """Caller-owned scratch for the split-KV partials (+ the int32[4] error word).

    Allocate once (outside graph capture) for the largest batch / context and
    reuse it; ``error()`` reads the device-side error word (synchronises).
    """

    def __init__(self, nbytes: int, device=None):
        self.buf = torch.zeros(int(nbytes) + 256, dtype=torch.uint8, device=device or "cuda")
        self.nbytes = int(nbytes)

    @classmethod
    def for_decode(cls, batch: int, num_q_heads: int, head_dim: int, max_pages: int, device=None):
        lib = _capi.lib()
        return cls(lib.lkv_decode_workspace_bytes(batch, num_q_heads, head_dim, max_pages), device)

    def ptr(self) -> int:
        return self.buf.data_ptr()

    def error(self) -> list[int]:
        out = (_capi.I32 * 4)()
        _capi.check(_capi.lib().lkv_read_error_word(self.ptr(), out, _stream()), "lkv_read_error_word")
        return list(out)

    def clear_error(self) -> None:
        _capi.check(_capi.lib().lkv_clear_error_word(self.ptr(), _stream()), "lkv_clear_error_word")


@_traced
def decode_paged(q, pool_k, pool_v, block_table, seq_k, *, softmax_scale=None, out=None, lse=None,
                 out_scale=None, workspace: Workspace | None = None, max_pages: int | None = None,
                 partial: bool = False, partial_out=None, tables_ready: bool = False, l2_keep: bool = False):
    """One query token per sequence against its paged history.

    q [B, Hq, D] bf16 (row-strided views allowed); block_table int32 [B, W];
    seq_k int32 [B]; out_scale fp32 [Hq] or None.  Returns out [B, Hq, D] bf16,
    or with ``partial=True`` a pair (o fp32 [B, Hq, D], lse fp32 [B, Hq]) for
    ``merge_partials``.  ``tables_ready=True`` (LKV_DECODE_TABLES_READY) promises
    that seq_k, the block table and all but each sequence's last page were
    written before the stream's most recent non-PDL operation (a copy, a torch
    kernel, a graph start), so the kernel may start loading pages before the
    preceding kernel finishes.  ``l2_keep=True`` (LKV_DECODE_L2_KEEP): the call is
    one of several over the same history (a step's layers), so the oldest pages
    of each sequence, a quarter of the L2 in all, are loaded to stay in L2.
    """
    _check_pool(pool_k, pool_v)
    B, Hq, D = q.shape
    Hkv = pool_k.shape[2]
    require_heads(Hq, Hkv, D)
    _require(pool_k.shape[3] == D, "head_dim mismatch between q and pools")
    _require(q.dtype == torch.bfloat16 and q.stride(2) == 1 and q.stride(1) == D, "q must be bf16 [B, Hq, D] rows")
    _require(block_table.dtype == torch.int32 and block_table.dim() == 2 and block_table.stride(1) == 1,
             "block_table must be int32 [B, W] with unit column stride")
    _require(block_table.shape[0] >= B and seq_k.dtype == torch.int32 and seq_k.numel() >= B, "seq_k/block_table")
    W = int(max_pages if max_pages is not None else block_table.shape[1])
    _require(W <= block_table.shape[1], "max_pages exceeds block_table width")
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    if workspace is None:
        workspace = Workspace.for_decode(B, Hq, D, W, device=q.device)
    po = pl = None
    if partial:
        if partial_out is not None:  # caller views (e.g. the two halves of one send buffer)
            po, pl = partial_out
            _require(po.dtype == torch.float32 and po.is_contiguous() and po.numel() == B * Hq * D, "partial o")
            _require(pl.dtype == torch.float32 and pl.is_contiguous() and pl.numel() == B * Hq, "partial lse")
        else:
            po = torch.empty((B, Hq, D), dtype=torch.float32, device=q.device)
            pl = torch.empty((B, Hq), dtype=torch.float32, device=q.device)
    elif out is None:
        out = torch.empty((B, Hq, D), dtype=torch.bfloat16, device=q.device)
    if out is not None:
        _require(out.dtype == torch.bfloat16 and out.stride(2) == 1 and out.stride(1) == D, "out layout")
    if out_scale is not None:
        _require(out_scale.dtype == torch.float32 and out_scale.numel() == Hq and out_scale.is_contiguous(),
                 "out_scale must be fp32 [Hq]")
    st = _capi.lib().lkv_decode_paged(
        q.data_ptr(), q.stride(0), pool_k.data_ptr(), pool_v.data_ptr(), pool_k.shape[0],
        block_table.data_ptr(), block_table.stride(0), seq_k.data_ptr(),
        _ptr(out), out.stride(0) if out is not None else 0, _ptr(lse), _ptr(out_scale), _ptr(po), _ptr(pl),
        B, Hq, Hkv, D, W, float(softmax_scale), workspace.ptr(), workspace.nbytes,
        (DECODE_TABLES_READY if tables_ready else 0) | (DECODE_L2_KEEP if l2_keep else 0), _stream())
    _capi.check(st, "lkv_decode_paged")
    return (po, pl) if partial else out


def decode_plan(batch, num_q_heads, num_kv_heads, head_dim, max_pages, workspace: Workspace, partial=False):
    """(splits, kernel launches) lkv_decode_paged will use for this shape on the current device."""
    s, n = ctypes.c_int(0), ctypes.c_int(0)
    _capi.check(_capi.lib().lkv_decode_plan(batch, num_q_heads, num_kv_heads, head_dim, max_pages,
                                            workspace.nbytes, int(partial), ctypes.byref(s), ctypes.byref(n)),
                "lkv_decode_plan")
    return s.value, n.value


def prefill_split_plan(batch, max_q, num_q_heads, num_kv_heads, head_dim, max_pages, causal) -> int:
    """Key splits lkv_prefill_paged_split would use for this shape (1 = no split)."""
    s = ctypes.c_int(1)
    _capi.check(_capi.lib().lkv_prefill_split_plan(batch, max_q, num_q_heads, num_kv_heads, head_dim, max_pages,
                                                   int(bool(causal)), ctypes.byref(s)), "lkv_prefill_split_plan")
    return s.value


@_traced
def prefill_paged(q, pool_k, pool_v, block_table, seq_k, cu_q, max_q: int, *, causal=True, softmax_scale=None,
                  out=None, lse=None, out_scale=None, error_word=None, max_pages: int | None = None,
                  kv_splits: int | None = None, partials=None):
    """Varlen chunked prefill on tcgen05 tensor cores.

    q [T, Hq, D] bf16 rows; cu_q int32 [B+1]; seq_k int32 [B] (>= span when
    causal; bottom-right alignment); returns out [T, Hq, D] bf16.  Non-causal
    calls may split the keys (``kv_splits``; None = the library's plan) into
    fp32 partials merged in a second launch; ``partials`` = (o fp32
    [S, T * Hq, D], lse fp32 [S, T * Hq]) with S >= kv_splits supplies their
    scratch (otherwise it is allocated per call, so pass it, or kv_splits=1,
    inside a CUDA-graph capture).
    """
    _check_pool(pool_k, pool_v)
    T, Hq, D = q.shape
    Hkv = pool_k.shape[2]
    require_heads(Hq, Hkv, D)
    _require(q.dtype == torch.bfloat16 and q.stride(2) == 1 and q.stride(1) == D, "q must be bf16 [T, Hq, D] rows")
    _require(block_table.dtype == torch.int32 and block_table.stride(1) == 1, "block_table must be int32 [B, W]")
    _require(cu_q.dtype == torch.int32 and seq_k.dtype == torch.int32, "cu_q / seq_k must be int32")
    B = cu_q.numel() - 1
    W = int(max_pages if max_pages is not None else block_table.shape[1])
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    if out is None:
        out = torch.empty((T, Hq, D), dtype=torch.bfloat16, device=q.device)
    _require(out.dtype == torch.bfloat16 and out.stride(2) == 1 and out.stride(1) == D, "out layout")
    if error_word is None:
        error_word = torch.zeros(4, dtype=torch.int32, device=q.device)
    if out_scale is not None:
        _require(out_scale.dtype == torch.float32 and out_scale.numel() == Hq, "out_scale must be fp32 [Hq]")
    if causal:
        kv_splits = 1
    elif kv_splits is None:
        kv_splits = prefill_split_plan(B, int(max_q), Hq, Hkv, D, W, False)
    if kv_splits > 1:
        if partials is not None:
            part_o, part_lse = partials
            _require(part_o.dtype == torch.float32 and part_o.is_contiguous() and part_o.dim() == 3
                     and part_o.shape[0] >= kv_splits and part_o.shape[1:] == (T * Hq, D),
                     "partials[0] must be contiguous fp32 [S >= kv_splits, T * Hq, D]")
            _require(part_lse.dtype == torch.float32 and part_lse.is_contiguous()
                     and part_lse.shape[0] >= kv_splits and part_lse.shape[1:] == (T * Hq,),
                     "partials[1] must be contiguous fp32 [S >= kv_splits, T * Hq]")
        else:
            part_o = torch.empty((kv_splits, T * Hq, D), dtype=torch.float32, device=q.device)
            part_lse = torch.empty((kv_splits, T * Hq), dtype=torch.float32, device=q.device)
        st = _capi.lib().lkv_prefill_paged_split(
            q.data_ptr(), q.stride(0), pool_k.data_ptr(), pool_v.data_ptr(), pool_k.shape[0], block_table.data_ptr(),
            block_table.stride(0), seq_k.data_ptr(), cu_q.data_ptr(), out.data_ptr(), out.stride(0), _ptr(lse),
            _ptr(out_scale), B, T, int(max_q), Hq, Hkv, D, W, float(softmax_scale), int(kv_splits),
            part_o.data_ptr(), part_lse.data_ptr(), error_word.data_ptr(), _stream())
        _capi.check(st, "lkv_prefill_paged_split")
        return out
    st = _capi.lib().lkv_prefill_paged(
        q.data_ptr(), q.stride(0), pool_k.data_ptr(), pool_v.data_ptr(), pool_k.shape[0], block_table.data_ptr(),
        block_table.stride(0), seq_k.data_ptr(), cu_q.data_ptr(), out.data_ptr(), out.stride(0), _ptr(lse),
        _ptr(out_scale), B, T, int(max_q), Hq, Hkv, D, W, int(bool(causal)), float(softmax_scale),
        error_word.data_ptr(), _stream())
    _capi.check(st, "lkv_prefill_paged")
    return out


@_traced
def merge_partials(o_parts, lse_parts, *, out_scale=None, out=None, lse_out=None):
    """LSE-merge P partials: o_parts fp32 [P, T, Hq, D], lse_parts fp32 [P, T, Hq]."""
    P_, T, Hq, D = o_parts.shape
    _require(o_parts.dtype == torch.float32 and o_parts.is_contiguous(), "o_parts must be contiguous fp32")
    _require(lse_parts.shape == (P_, T, Hq) and lse_parts.is_contiguous(), "lse_parts must be [P, T, Hq]")
    if out is None:
        out = torch.empty((T, Hq, D), dtype=torch.bfloat16, device=o_parts.device)
    _require(out.is_contiguous() and out.dtype == torch.bfloat16, "out must be contiguous bf16")
    st = _capi.lib().lkv_merge_partials(o_parts.data_ptr(), lse_parts.data_ptr(), P_, T * Hq, D, Hq, 0, 0,
                                        _ptr(out_scale), out.data_ptr(), _ptr(lse_out), _stream())
    _capi.check(st, "lkv_merge_partials")
    return out


@_traced
def merge_partials_packed(parts, T: int, Hq: int, D: int, *, out_scale=None, out=None, lse_out=None):
    """LSE-merge parts packed as [P, T*Hq*D (o) | T*Hq (lse) | pad] fp32 rows (one all-gather buffer)."""
    P_ = parts.shape[0]
    rows = T * Hq
    stride = parts.shape[1]  # o [rows*D], lse [rows], padding to a multiple of 4 floats
    _require(parts.dtype == torch.float32 and parts.is_contiguous() and stride >= rows * (D + 1)
             and stride % 4 == 0, "parts must be contiguous fp32 [P, >= rows * (D + 1)], stride % 4 == 0")
    if out is None:
        out = torch.empty((T, Hq, D), dtype=torch.bfloat16, device=parts.device)
    _require(out.is_contiguous() and out.dtype == torch.bfloat16, "out must be contiguous bf16")
    st = _capi.lib().lkv_merge_partials(parts.data_ptr(), parts.data_ptr() + rows * D * 4, P_, rows, D, Hq, stride,
                                        stride, _ptr(out_scale), out.data_ptr(), _ptr(lse_out), _stream())
    _capi.check(st, "lkv_merge_partials")
    return out


@_traced
def attention_paged_f32(q, pool_k, pool_v, block_table, seq_k, cu_q, *, causal=True, softmax_scale=None,
                        out=None, lse=None, out_scale=None, error_word=None, max_pages: int | None = None):
    """The merged attention call for fp32 models (lkv_attention_paged_f32): decode (one
    token per sequence) or chunked-prefill spans over fp32 pools, bottom-right causal.

    q [T, Hq, D] fp32 rows; pools fp32 [pages, 16, Hkv, D]; block_table int32 [B, W];
    seq_k int32 [B]; cu_q int32 [B+1]; out_scale fp32 [Hq] or None.  Returns out
    [T, Hq, D] fp32.
    """
    _check_pool_f32(pool_k, pool_v)
    T, Hq, D = q.shape
    Hkv = pool_k.shape[2]
    _require(Hq % Hkv == 0 and D in (64, 128) and pool_k.shape[3] == D, "heads / head_dim")
    _require(q.dtype == torch.float32 and q.stride(2) == 1 and q.stride(1) == D, "q must be fp32 [T, Hq, D] rows")
    _require(block_table.dtype == torch.int32 and block_table.stride(1) == 1, "block_table must be int32 [B, W]")
    _require(cu_q.dtype == torch.int32 and seq_k.dtype == torch.int32, "cu_q / seq_k must be int32")
    B = cu_q.numel() - 1
    W = int(max_pages if max_pages is not None else block_table.shape[1])
    _require(W <= block_table.shape[1], "max_pages exceeds block_table width")
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    if out is None:
        out = torch.empty((T, Hq, D), dtype=torch.float32, device=q.device)
    _require(out.dtype == torch.float32 and out.stride(2) == 1 and out.stride(1) == D, "out layout")
    if error_word is None:
        error_word = torch.zeros(4, dtype=torch.int32, device=q.device)
    if out_scale is not None:
        _require(out_scale.dtype == torch.float32 and out_scale.numel() == Hq, "out_scale must be fp32 [Hq]")
    if lse is not None:
        _require(lse.dtype == torch.float32 and lse.is_contiguous() and lse.numel() == T * Hq, "lse [T, Hq] fp32")
    st = _capi.lib().lkv_attention_paged_f32(
        q.data_ptr(), q.stride(0), pool_k.data_ptr(), pool_v.data_ptr(), pool_k.shape[0], block_table.data_ptr(),
        block_table.stride(0), seq_k.data_ptr(), cu_q.data_ptr(), out.data_ptr(), out.stride(0), _ptr(lse),
        _ptr(out_scale), B, T, Hq, Hkv, D, W, int(bool(causal)), float(softmax_scale), error_word.data_ptr(),
        _stream())
    _capi.check(st, "lkv_attention_paged_f32")
    return out


class Commit(NamedTuple):
    """A chunk-boundary commit (the ``blend_chunk`` arguments) to run inside the next
    append launch (``rope_norm_append(..., commit=)``, lkv_rope_norm_append_commit).

    ``count`` (device int32 [1], optional) holds how many rows of raw/ring_pages to
    commit, read on the device, so a captured launch can carry a commit or none;
    ``blocks`` is the launch's block count for the commit (0: one per page item
    without ``count``, one wave of 8 per SM with it)."""

    pool_k: torch.Tensor
    pool_v: torch.Tensor
    raw_pages: torch.Tensor
    ring_pages: torch.Tensor
    ring_layer_stride: int
    alpha: torch.Tensor
    count: Optional[torch.Tensor] = None
    blocks: int = 0


def _check_commit(c: Commit):
    _check_pool(c.pool_k, c.pool_v)
    _require(c.raw_pages.dim() == 2 and c.ring_pages.shape == c.raw_pages.shape, "ring_pages must match raw_pages")
    _require(c.raw_pages.dtype == torch.int32 and c.ring_pages.dtype == torch.int32, "page lists must be int32")
    _require(c.raw_pages.is_contiguous() and c.ring_pages.is_contiguous(), "page lists must be contiguous")
    _require(c.alpha.dtype == torch.float32 and c.alpha.is_contiguous() and c.alpha.dim() == 2,
             "alpha must be fp32 [L, Hkv]")
    if c.count is not None:
        _require(c.count.dtype == torch.int32 and c.count.numel() >= 1, "commit count must be device int32 [1]")
    _require(c.blocks >= 0, "commit blocks must be >= 0")


@_traced
def rope_norm_append(q, k, v, positions, cos_sin, q_weight, k_weight, eps, inv_scale, ring_slot, ring_k, ring_v,
                     src_slot=None, src_k=None, src_v=None, q_out=None, error_word=None, interleaved=False,
                     commit: Optional[Commit] = None):
    """Fused RoPE -> Q/K RMSNorm -> V/s -> paged append for one layer.

    q [T, Hq*D], k/v [T, Hkv*D] bf16 (row-strided views allowed); positions
    int64 [T]; cos_sin bf16 or fp32 [max_pos, D] (cos | sin halves) or None;
    ``interleaved`` rotates pairs (2i, 2i+1) instead of (i, i + D/2); ring_* /
    src_* flat token views [slots, Hkv, D] of the pools.  Returns q_out [T, Hq, D].
    ``commit`` (bf16 only) runs the previous boundary's chunk blend in the same
    launch; pass it to the first layer of the step after the boundary.
    """
    T = q.shape[0]
    D = ring_k.shape[-1]
    Hq, Hkv = q.shape[-1] // D, k.shape[-1] // D
    require_heads(Hq, Hkv, D)
    # bf16 everywhere, or fp32 everywhere (LKV_APPEND_FP32: the fp32 model configuration)
    dt = ring_k.dtype
    _require(dt in (torch.bfloat16, torch.float32) and ring_v.dtype == dt, "ring views must be bf16 or fp32")
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require(t.dtype == dt and t.dim() == 2 and t.stride(1) == 1, f"{name} must be {dt} [T, H*D] rows")
    _require(ring_slot.dtype == torch.int64, "slots must be int64")
    if cos_sin is not None:  # None: use_nope (no rotary)
        _require(positions.dtype == torch.int64, "positions must be int64")
        _require(cos_sin.dtype in (torch.bfloat16, torch.float32) and cos_sin.stride(1) == 1
                 and cos_sin.shape[-1] == D, "cos_sin must be bf16 or fp32 [max_pos, D]")
        _require(dt == torch.bfloat16 or cos_sin.dtype == torch.float32, "the fp32 append takes an fp32 table")
    flags = (1 if interleaved else 0) | (2 if cos_sin is not None and cos_sin.dtype == torch.float32 else 0)
    if dt == torch.float32:
        flags |= APPEND_FP32
    _require((q_weight is None) == (k_weight is None), "q/k norm weights come together (None: use_qk_norm=False)")
    if q_weight is not None:
        _require(q_weight.dtype == dt and k_weight.dtype == dt, f"norm weights must be {dt}")
    if src_k is not None:
        _require(src_k.dtype == dt and src_v.dtype == dt, "shared-history views must match the rings' dtype")
    if q_out is None:
        q_out = torch.empty((T, Hq, D), dtype=dt, device=q.device)
    _require(q_out.dtype == dt, "q_out dtype")
    top = src_slot is not None
    args = (q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), _ptr(positions),
            _ptr(cos_sin), cos_sin.stride(0) if cos_sin is not None else 0,
            cos_sin.shape[0] if cos_sin is not None else 0, _ptr(q_weight), _ptr(k_weight),
            float(eps), _ptr(inv_scale), q_out.data_ptr(), q_out.stride(0), ring_slot.data_ptr(),
            ring_k.data_ptr(), ring_v.data_ptr(), ring_k.shape[0],
            _ptr(src_slot), _ptr(src_k) if top else None, _ptr(src_v) if top else None,
            src_k.shape[0] if top else 0, T, Hq, Hkv, D, flags)
    if commit is None:
        st = _capi.lib().lkv_rope_norm_append(*args, _ptr(error_word), _stream())
        _capi.check(st, "lkv_rope_norm_append")
        return q_out
    _require(dt == torch.bfloat16, "the fused commit takes bf16 pools (fp32: append, then blend_chunk)")
    _check_commit(commit)
    S, ppc = commit.raw_pages.shape
    L, hkv = commit.alpha.shape
    _require(hkv == Hkv and commit.pool_k.shape[2] == Hkv and commit.pool_k.shape[3] == D,
             "commit pools must match the append's heads")
    st = _capi.lib().lkv_rope_norm_append_commit(
        *args, commit.pool_k.data_ptr(), commit.pool_v.data_ptr(), commit.pool_k.shape[0],
        commit.raw_pages.data_ptr(), commit.ring_pages.data_ptr(), int(commit.ring_layer_stride),
        commit.alpha.data_ptr(), L, S, ppc, _ptr(commit.count), int(commit.blocks), _ptr(error_word), _stream())
    _capi.check(st, "lkv_rope_norm_append_commit")
    return q_out


@_traced
def gather_blend(pool_k, pool_v, dst, src_a, src_b, alpha_row, alpha, *, error_word=None):
    """Token-level copy / blend on the flat pool (see lkv_gather_blend).

    dst, src_a, src_b int64 [N] flat token slots (-1 in src_a or src_b means
    copy the other); alpha_row int32 [N] row of alpha fp32 [R, Hkv].
    """
    _check_pool(pool_k, pool_v)
    N = dst.numel()
    for name, t in (("dst", dst), ("src_a", src_a), ("src_b", src_b)):
        _require(t.dtype == torch.int64 and t.numel() == N and t.is_contiguous(), f"{name} must be int64 [N]")
    _require(alpha_row.dtype == torch.int32 and alpha_row.numel() == N, "alpha_row must be int32 [N]")
    _require(alpha.dtype == torch.float32 and alpha.is_contiguous(), "alpha must be fp32 [rows, Hkv]")
    st = _capi.lib().lkv_gather_blend(pool_k.data_ptr(), pool_v.data_ptr(), pool_k.shape[0] * pool_k.shape[1],
                                      dst.data_ptr(), src_a.data_ptr(), src_b.data_ptr(), alpha_row.data_ptr(),
                                      alpha.data_ptr(), N, pool_k.shape[2], pool_k.shape[3], _ptr(error_word),
                                      _stream())
    _capi.check(st, "lkv_gather_blend")


@_traced
def blend_chunk(pool_k, pool_v, raw_pages, ring_pages, ring_layer_stride: int, alpha, *, error_word=None):
    """Commit a finished chunk into every layer ring (K and V/s) in place.

    raw_pages / ring_pages int32 [S, C/16]; alpha fp32 [L, Hkv] (bf16-exact for
    bf16 pools; the fp32 sigmoid for fp32 pools, which take lkv_blend_chunk_f32).
    """
    fn = _capi.lib().lkv_blend_chunk
    if pool_k.dtype == torch.float32:
        _check_pool_f32(pool_k, pool_v)
        fn = _capi.lib().lkv_blend_chunk_f32
    else:
        _check_pool(pool_k, pool_v)
    S, ppc = raw_pages.shape
    L, Hkv = alpha.shape
    _require(ring_pages.shape == raw_pages.shape, "ring_pages must match raw_pages")
    _require(raw_pages.dtype == torch.int32 and ring_pages.dtype == torch.int32, "page lists must be int32")
    _require(alpha.dtype == torch.float32 and alpha.is_contiguous(), "alpha must be fp32 [L, Hkv]")
    st = fn(pool_k.data_ptr(), pool_v.data_ptr(), pool_k.shape[0], raw_pages.contiguous().data_ptr(),
            ring_pages.contiguous().data_ptr(), int(ring_layer_stride), alpha.data_ptr(), L, S, ppc, Hkv,
            pool_k.shape[3], _ptr(error_word), _stream())
    _capi.check(st, "lkv_blend_chunk")


@_traced
def build_layer_block_tables(block_table, nsrc, ring_base, out=None):
    """bt_all [L, B, W] from [older | layer-relative ring] rows (fastpath.py:422-424)."""
    B, W = block_table.shape
    L = ring_base.numel()
    if out is None:
        out = torch.empty((L, B, W), dtype=torch.int32, device=block_table.device)
    _require(out.shape == (L, B, W) and out.is_contiguous() and out.dtype == torch.int32,
             "out must be a contiguous int32 [L, B, W] tensor")
    _require(nsrc.dtype == torch.int32 and ring_base.dtype == torch.int32 and block_table.dtype == torch.int32,
             "block tables, nsrc and ring_base must be int32")
    st = _capi.lib().lkv_build_layer_block_tables(block_table.data_ptr(), block_table.stride(0), nsrc.data_ptr(),
                                                  ring_base.data_ptr(), L, B, W, out.data_ptr(), _stream())
    _capi.check(st, "lkv_build_layer_block_tables")
    return out


def _rows2d(t, name):
    _require(t.dtype == torch.bfloat16 and t.is_cuda and t.stride(-1) == 1, f"{name} must be CUDA bf16 with unit stride")
    return t.reshape(-1, t.shape[-1]) if t.dim() != 2 else t


@_traced
def rmsnorm(x, weight, eps: float, residual=None, *, out=None, residual_out=None):
    """RMSNorm over the last dim, optionally after the residual add h = x + residual.

    Returns ``out`` (the normalised rows), or ``(h, out)`` when ``residual`` is
    given; ``h`` is written to ``residual_out`` (default: a new tensor).  The
    rounding points are those of the eager decoder layer (see lkv_rmsnorm).
    """
    shape = x.shape
    H = shape[-1]
    x2 = _rows2d(x, "x")
    _require(weight.dtype == torch.bfloat16 and weight.is_contiguous() and weight.numel() == H,
             "weight must be contiguous bf16 [hidden]")
    rows = x2.shape[0]
    if out is None:
        out = torch.empty(shape, dtype=torch.bfloat16, device=x.device)
    _require(out.is_contiguous() and out.shape == shape, "out must be contiguous and match x")
    o2 = _rows2d(out, "out")
    r2 = ro2 = None
    if residual is not None:
        _require(residual.shape == shape, "residual must match x")
        r2 = _rows2d(residual, "residual")
        if residual_out is None:
            residual_out = torch.empty(shape, dtype=torch.bfloat16, device=x.device)
        _require(residual_out.is_contiguous() and residual_out.shape == shape,
                 "residual_out must be contiguous and match x")
        ro2 = _rows2d(residual_out, "residual_out")
    st = _capi.lib().lkv_rmsnorm(x2.data_ptr(), x2.stride(0), _ptr(r2), r2.stride(0) if r2 is not None else 0,
                                 _ptr(ro2), ro2.stride(0) if ro2 is not None else 0, weight.data_ptr(),
                                 o2.data_ptr(), o2.stride(0), rows, H, float(eps), _stream())
    _capi.check(st, "lkv_rmsnorm")
    return out if residual is None else (residual_out, out)


@_traced
def silu_mul(gate_up, *, out=None):
    """bf16(bf16(silu(gate)) * up) for rows [gate | up] of width 2F; returns [..., F]."""
    F2 = gate_up.shape[-1]
    _require(F2 % 2 == 0, "gate_up must hold [gate | up]")
    g2 = _rows2d(gate_up, "gate_up")
    if out is None:
        out = torch.empty((*gate_up.shape[:-1], F2 // 2), dtype=torch.bfloat16, device=gate_up.device)
    _require(out.is_contiguous() and out.shape == (*gate_up.shape[:-1], F2 // 2), "out must be contiguous [..., F]")
    o2 = _rows2d(out, "out")
    st = _capi.lib().lkv_silu_mul(g2.data_ptr(), g2.stride(0), o2.data_ptr(), o2.stride(0), g2.shape[0], F2 // 2,
                                  _stream())
    _capi.check(st, "lkv_silu_mul")
    return out


@_traced
def argmax_rows(logits, *, out=None):
    """torch.argmax(logits, -1) for bf16 rows (first index on ties, NaN largest), int64 [rows]."""
    x2 = _rows2d(logits, "logits")
    if out is None:
        out = torch.empty(x2.shape[0], dtype=torch.int64, device=logits.device)
    _require(out.dtype == torch.int64 and out.is_contiguous() and out.numel() == x2.shape[0], "out must be int64 [rows]")
    st = _capi.lib().lkv_argmax_rows(x2.data_ptr(), x2.stride(0), x2.shape[0], x2.shape[1], out.data_ptr(), _stream())
    _capi.check(st, "lkv_argmax_rows")
    return out


GEMM_PLAIN, GEMM_SILU_MUL = 0, 1
DECODE_GEMM_MAX_ROWS = 16


def decode_gemm_supported(x, weight) -> bool:
    """Whether ``decode_gemm(x, weight)`` takes these tensors (else use F.linear)."""
    if not (x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and weight.dim() == 2):
        return False
    K = x.shape[-1]
    rows = x.numel() // K if K else 0
    return (1 <= rows <= DECODE_GEMM_MAX_ROWS and weight.shape[1] == K and K % 8 == 0 and x.stride(-1) == 1
            and weight.stride(1) == 1 and weight.stride(0) % 8 == 0 and weight.data_ptr() % 16 == 0
            and x.data_ptr() % 16 == 0 and (x.dim() == 2 or x.is_contiguous()) and x.stride(0) % 8 == 0)


def decode_gemm_plan(n_rows: int, k: int, silu_mul: bool = False) -> dict:
    """{tiles, splits, ctas_per_sm} of the decode GEMM launch for a weight [n_rows, k] on this device."""
    t, s, o = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    _capi.check(_capi.lib().lkv_decode_gemm_plan(n_rows, k, GEMM_SILU_MUL if silu_mul else GEMM_PLAIN,
                                                 ctypes.byref(t), ctypes.byref(s), ctypes.byref(o)),
                "lkv_decode_gemm_plan")
    return {"tiles": t.value, "splits": s.value, "ctas_per_sm": o.value}


@_traced
def decode_gemm(x, weight, *, silu_mul: bool = False, out=None, error_word=None):
    """``x @ weight.T`` for 1..16 rows of x (decode) on tcgen05, bf16 out.

    ``silu_mul``: weight holds [gate (F rows) | up (F rows)] and the result is
    ``silu(x @ gate.T) * (x @ up.T)`` [..., F] with the eager rounding points.
    Capturable in CUDA graphs.
    """
    K = x.shape[-1]
    x2 = _rows2d(x, "x")
    M = x2.shape[0]
    _require(1 <= M <= DECODE_GEMM_MAX_ROWS, f"decode_gemm takes 1..{DECODE_GEMM_MAX_ROWS} rows")
    _require(weight.dtype == torch.bfloat16 and weight.dim() == 2 and weight.stride(1) == 1 and weight.shape[1] == K,
             "weight must be bf16 [N, K] rows")
    N = weight.shape[0]
    mode = GEMM_SILU_MUL if silu_mul else GEMM_PLAIN
    n_out = N // 2 if silu_mul else N
    if out is None:
        out = torch.empty((*x.shape[:-1], n_out), dtype=torch.bfloat16, device=x.device)
    _require(out.is_contiguous() and out.shape == (*x.shape[:-1], n_out) and out.dtype == torch.bfloat16,
             "out must be contiguous bf16 [..., N]")
    st = _capi.lib().lkv_decode_gemm(x2.data_ptr(), x2.stride(0), weight.data_ptr(), weight.stride(0),
                                     out.data_ptr(), n_out, M, N, K, mode, _ptr(error_word), None, _stream())
    _capi.check(st, "lkv_decode_gemm")
    return out


def cp_combine_sizes(rows: int, head_dim: int, world: int) -> dict:
    """{send_floats, recv_words} of the context-parallel combine buffers."""
    a, b = ctypes.c_int64(0), ctypes.c_int64(0)
    _capi.check(_capi.lib().lkv_cp_combine_sizes(rows, head_dim, world, ctypes.byref(a), ctypes.byref(b)),
                "lkv_cp_combine_sizes")
    return {"send_floats": a.value, "recv_words": b.value}


def decode_cp_state_words(batch: int, num_kv_heads: int) -> int:
    """uint32 words of device state lkv_decode_paged_cp needs (epoch, done counter, unit arrivals)."""
    n = ctypes.c_int64(0)
    _capi.check(_capi.lib().lkv_decode_cp_state_words(batch, num_kv_heads, ctypes.byref(n)),
                "lkv_decode_cp_state_words")
    return n.value


@_traced
def decode_paged_cp(q, pool_k, pool_v, block_table, seq_k, recv_ptrs, rank: int, world: int, state, *,
                    softmax_scale=None, out=None, out_scale=None, workspace: Workspace | None = None,
                    max_pages: int | None = None, error_word=None, tables_ready: bool = False,
                    l2_keep: bool = False):
    """Sequence-sharded decode with the exchange fused into the decode kernel (lkv_decode_paged_cp):
    this rank's slice of the keys, every unit's merged rows pushed to every rank's receive
    buffer as the unit finishes, then the poll-and-merge launch.  state: int32 device tensor
    of decode_cp_state_words(B, Hkv) words, zero before the first call.  Returns out bf16 [B, Hq, D]."""
    _check_pool(pool_k, pool_v)
    B, Hq, D = q.shape
    Hkv = pool_k.shape[2]
    require_heads(Hq, Hkv, D)
    _require(q.dtype == torch.bfloat16 and q.stride(2) == 1 and q.stride(1) == D, "q must be bf16 [B, Hq, D] rows")
    _require(block_table.dtype == torch.int32 and block_table.dim() == 2 and block_table.stride(1) == 1,
             "block_table must be int32 [B, W] with unit column stride")
    _require(len(recv_ptrs) == world, "one receive buffer per rank")
    _require(state.dtype == torch.int32 and state.is_cuda and state.numel() >= decode_cp_state_words(B, Hkv),
             "state must be int32 [decode_cp_state_words(B, Hkv)]")
    W = int(max_pages if max_pages is not None else block_table.shape[1])
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    if workspace is None:
        workspace = Workspace.for_decode(B, Hq, D, W, device=q.device)
    if out is None:
        out = torch.empty((B, Hq, D), dtype=torch.bfloat16, device=q.device)
    _require(out.dtype == torch.bfloat16 and out.stride(-1) == 1 and out.stride(-2) == D, "out layout")
    if out_scale is not None:
        _require(out_scale.dtype == torch.float32 and out_scale.numel() == Hq and out_scale.is_contiguous(),
                 "out_scale must be fp32 [Hq]")
    rp = (ctypes.c_uint64 * world)(*recv_ptrs)
    st = _capi.lib().lkv_decode_paged_cp(
        q.data_ptr(), q.stride(0), pool_k.data_ptr(), pool_v.data_ptr(), pool_k.shape[0], block_table.data_ptr(),
        block_table.stride(0), seq_k.data_ptr(), out.data_ptr(), out.stride(0), _ptr(out_scale), B, Hq, Hkv, D, W,
        float(softmax_scale), workspace.ptr(), workspace.nbytes, rp, rank, world, state.data_ptr(),
        _ptr(error_word), (DECODE_TABLES_READY if tables_ready else 0) | (DECODE_L2_KEEP if l2_keep else 0),
        _stream())
    _capi.check(st, "lkv_decode_paged_cp")
    return out


@_traced
def cp_combine(send, recv_ptrs, rank: int, world: int, state, rows: int, head_dim: int, hq: int, *,
               out_scale=None, out=None, error_word=None):
    """Push this rank's packed partial to every peer over peer memory, wait for theirs,
    LSE-merge in rank order (see lkv_cp_combine).  recv_ptrs: per-rank receive-buffer
    addresses valid on this GPU; state: int32 [2] device tensor, zero before the first
    call (the call's epoch advances on the device, so calls can be graph-captured).
    Returns out bf16 [rows / hq, hq, head_dim]."""
    _require(send is None or (send.dtype == torch.float32 and send.is_contiguous() and send.is_cuda),
             "send must be contiguous fp32 (or None: rows already pushed)")
    _require(len(recv_ptrs) == world, "one receive buffer per rank")
    _require(state.dtype == torch.int32 and state.numel() >= 2 and state.is_cuda, "state must be int32 [2]")
    if out is None:
        out = torch.empty((rows // hq, hq, head_dim), dtype=torch.bfloat16, device=state.device)
    _require(out.dtype == torch.bfloat16 and out.stride(-1) == 1 and out.stride(-2) == head_dim, "out layout")
    if out_scale is not None:
        _require(out_scale.dtype == torch.float32 and out_scale.numel() == hq and out_scale.is_contiguous(),
                 "out_scale must be fp32 [hq]")
    rp = (ctypes.c_uint64 * world)(*recv_ptrs)
    st = _capi.lib().lkv_cp_combine(_ptr(send), rp, rank, world, state.data_ptr(), rows, head_dim, hq,
                                    _ptr(out_scale), out.data_ptr(), out.stride(0), _ptr(error_word), _stream())
    _capi.check(st, "lkv_cp_combine")
    return out
