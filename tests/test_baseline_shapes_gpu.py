"""Parity at the BASELINE configurations' real shapes (sampled rows vs the float64 oracle).

The other GPU tests cover edge cases at small sizes; these run the kernels at
the sizes the benchmark measures and check a sampled subset of the output rows
(every head of the sampled tokens) against ``oracle.attention`` in float64 on
the same bf16 inputs, at the stated bf16 tolerance (max-abs <= 2e-2, relative
L2 <= 1e-2):

* config 2 - the bench's own decode workload (``bench.build_workload``: 64
  sequences x 8192 keys, 32/8 heads, D 128, shuffled 512-page tables, the
  [384 shared | 128 ring] merged layout, 4 KV splits), layers 0 and 31, with the
  per-head value scale s_l and with s_l = 1;
* config 3 - chunked prefill, batch 8: the 1024-token span at 7168 keys of
  history (causal, bottom-right) and the first 1024-token span;
* config 5 - Wan block attention: 4680 queries x 32760 keys per sequence,
  batch 2, 12 heads, non-causal, keys split 3 ways inside the launch;
* config 4 - 131072 keys per sequence, batch 4: the context-parallel form on
  one GPU (four contiguous shards' partials, then the exact LSE merge) and the
  unsharded decode.
"""

import numpy as np
import pytest
import torch

from oracle import lastkv_oracle as O
from tests.gpu_helpers import assert_close_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from lastkv_b200 import _capi

    _capi.load()
    assert _capi.lib().lkv_check_device(torch.cuda.current_device()) == 0
    yield
    torch.cuda.empty_cache()


def _seq_kv(pool_k, pool_v, bt_row, n):
    """One sequence's first n keys and values, token-major [n, Hkv, D] float32 on the host."""
    pages = bt_row[: -(-n // 16)].long()
    k = pool_k[pages].float().reshape(-1, *pool_k.shape[2:])[:n].cpu().numpy()
    v = pool_v[pages].float().reshape(-1, *pool_v.shape[2:])[:n].cpu().numpy()
    return k, v


def _oracle_rows(q_rows, k, v, key_pos, scale, out_scale=None):
    """float64 attention of query rows [R, Hq, D]; row r sees keys [0, key_pos[r]]."""
    out = []
    for r in range(q_rows.shape[0]):
        n = int(key_pos[r]) + 1
        o, _ = O.attention(q_rows[r:r + 1], k[:n], v[:n], scale=scale, causal=True)
        out.append(o[0])
    out = np.stack(out)
    if out_scale is not None:
        out = out * np.asarray(out_scale, np.float64)[None, :, None]
    return out


# ------------------------------------------------------------------ config 2


@pytest.mark.parametrize("with_scale", [True, False], ids=["s_l", "s_1"])
def test_config2_bench_workload_decode(with_scale):
    import bench
    from lastkv_b200 import ops

    dev = torch.device("cuda", torch.cuda.current_device())
    wl = bench.build_workload(0, dev)
    c = bench.CFG
    B, Hq, Hkv, D = c["batch"], c["q_heads"], c["kv_heads"], c["head_dim"]
    splits, _ = ops.decode_plan(B, Hq, Hkv, D, wl["W"], wl["ws"])
    assert splits == 4 and wl["W"] == 512
    sample = [0, 13, 38, 63]
    n = int(wl["seq_k"][0])
    assert n == 8192
    for l in (0, c["layers"] - 1):
        scale = wl["out_scale"][l] if with_scale else None
        out = ops.decode_paged(wl["q"][l], wl["pool_k"], wl["pool_v"], wl["bt_all"][l], wl["seq_k"],
                               out_scale=scale, workspace=wl["ws"], max_pages=wl["W"])
        torch.cuda.synchronize()
        assert wl["ws"].error()[0] == 0
        got = out.float().cpu().numpy()
        q = wl["q"][l].float().cpu().numpy()
        sc = scale.cpu().numpy() if scale is not None else None
        for b in sample:
            k, v = _seq_kv(wl["pool_k"], wl["pool_v"], wl["bt_all"][l][b], n)
            want = _oracle_rows(q[b:b + 1], k, v, [n - 1], D ** -0.5, sc)
            assert_close_bf16(got[b:b + 1], want, what=f"config 2 layer {l} seq {b}")
    del wl
    torch.cuda.empty_cache()


# ------------------------------------------------------------------ config 3


def _prefill_case(seed, B, Hq, Hkv, D, N, span, dev):
    gen = torch.Generator(device=dev).manual_seed(seed)
    pages = N // 16
    pool_k = torch.randn((B * pages + 3, 16, Hkv, D), generator=gen, device=dev, dtype=torch.bfloat16)
    pool_v = torch.randn((B * pages + 3, 16, Hkv, D), generator=gen, device=dev, dtype=torch.bfloat16)
    bt = torch.randperm(B * pages, generator=gen, device=dev).to(torch.int32).view(B, pages)
    q = torch.randn((B * span, Hq, D), generator=gen, device=dev, dtype=torch.bfloat16)
    cu = torch.arange(0, B * span + 1, span, dtype=torch.int32, device=dev)
    return pool_k, pool_v, bt, q, cu


@pytest.mark.parametrize("history", [7168, 0], ids=["last_span_7168", "first_span"])
def test_config3_chunked_prefill_span(history):
    from lastkv_b200 import ops

    dev = torch.device("cuda", torch.cuda.current_device())
    B, Hq, Hkv, D, span = 8, 32, 8, 128, 1024
    pool_k, pool_v, bt, q, cu = _prefill_case(33, B, Hq, Hkv, D, 8192, span, dev)
    n = history + span
    seq_k = torch.full((B,), n, dtype=torch.int32, device=dev)
    rng = np.random.default_rng(3)
    scale_h = rng.uniform(0.5, 1.5, Hq).astype(np.float32)
    err = torch.zeros(4, dtype=torch.int32, device=dev)
    out = ops.prefill_paged(q, pool_k, pool_v, bt, seq_k, cu, span, out_scale=torch.from_numpy(scale_h).to(dev),
                            error_word=err, max_pages=n // 16)
    torch.cuda.synchronize()
    assert err.cpu().tolist()[0] == 0
    got = out.float().cpu().numpy().reshape(B, span, Hq, D)
    qn = q.float().cpu().numpy().reshape(B, span, Hq, D)
    toks = np.unique(np.concatenate([[0, 1, 127, 128, 511, span - 1], rng.integers(0, span, 10)]))
    for b in (0, 5, 7):
        k, v = _seq_kv(pool_k, pool_v, bt[b], n)
        want = _oracle_rows(qn[b, toks], k, v, history + toks, D ** -0.5, scale_h)
        assert_close_bf16(got[b, toks], want, what=f"config 3 history {history} seq {b}")


# ------------------------------------------------------------------ config 5


def test_config5_wan_block_attention_three_key_splits():
    from lastkv_b200 import ops

    dev = torch.device("cuda", torch.cuda.current_device())
    B, H, D, block, keys = 2, 12, 128, 4680, 32760
    pages = -(-keys // 16)
    gen = torch.Generator(device=dev).manual_seed(55)
    pool_k = torch.randn((B * pages + 1, 16, H, D), generator=gen, device=dev, dtype=torch.bfloat16)
    pool_v = torch.randn((B * pages + 1, 16, H, D), generator=gen, device=dev, dtype=torch.bfloat16)
    bt = torch.randperm(B * pages, generator=gen, device=dev).to(torch.int32).view(B, pages)
    q = torch.randn((B * block, H, D), generator=gen, device=dev, dtype=torch.bfloat16)
    cu = torch.arange(0, B * block + 1, block, dtype=torch.int32, device=dev)
    seq_k = torch.full((B,), keys, dtype=torch.int32, device=dev)
    assert ops.prefill_split_plan(B, block, H, H, D, pages, False) == 3
    err = torch.zeros(4, dtype=torch.int32, device=dev)
    out = ops.prefill_paged(q, pool_k, pool_v, bt, seq_k, cu, block, causal=False, error_word=err, max_pages=pages,
                            kv_splits=3)
    torch.cuda.synchronize()
    assert err.cpu().tolist()[0] == 0
    got = out.float().cpu().numpy().reshape(B, block, H, D)
    qn = q.float().cpu().numpy().reshape(B, block, H, D)
    rng = np.random.default_rng(5)
    toks = np.unique(np.concatenate([[0, 1559, 1560, 4679], rng.integers(0, block, 8)]))
    for b in range(B):
        k, v = _seq_kv(pool_k, pool_v, bt[b], keys)
        want = _oracle_rows(qn[b, toks], k, v, [keys - 1] * len(toks), D ** -0.5)  # non-causal: all keys
        assert_close_bf16(got[b, toks], want, what=f"config 5 seq {b}")


# ------------------------------------------------------------------ config 4


def test_config4_131072_keys_sharded_partials_and_merge():
    from lastkv_b200 import ops

    dev = torch.device("cuda", torch.cuda.current_device())
    B, Hq, Hkv, D, N, G = 4, 32, 8, 128, 131072, 4
    pages = N // 16
    gen = torch.Generator(device=dev).manual_seed(404)
    pool_k = torch.randn((B * pages + 1, 16, Hkv, D), generator=gen, device=dev, dtype=torch.bfloat16)
    pool_v = torch.randn((B * pages + 1, 16, Hkv, D), generator=gen, device=dev, dtype=torch.bfloat16)
    bt = torch.randperm(B * pages, generator=gen, device=dev).to(torch.int32).view(B, pages)
    q = torch.randn((B, Hq, D), generator=gen, device=dev, dtype=torch.bfloat16)
    seq_k = torch.full((B,), N, dtype=torch.int32, device=dev)
    scale_h = np.random.default_rng(4).uniform(0.5, 1.5, Hq).astype(np.float32)
    scale = torch.from_numpy(scale_h).to(dev)
    per = pages // G
    ws = ops.Workspace.for_decode(B, Hq, D, per, device=dev)
    o_parts = torch.empty((G, B, Hq, D), dtype=torch.float32, device=dev)
    l_parts = torch.empty((G, B, Hq), dtype=torch.float32, device=dev)
    shard_len = torch.full((B,), per * 16, dtype=torch.int32, device=dev)
    for g in range(G):  # each shard = one rank's contiguous slice of every sequence
        ops.decode_paged(q, pool_k, pool_v, bt[:, g * per:(g + 1) * per].contiguous(), shard_len, workspace=ws,
                         max_pages=per, partial=True, partial_out=(o_parts[g], l_parts[g]))
    merged = ops.merge_partials(o_parts, l_parts, out_scale=scale)
    full = ops.decode_paged(q, pool_k, pool_v, bt, seq_k, out_scale=scale)
    torch.cuda.synchronize()
    assert ws.error()[0] == 0
    got_m, got_f = merged.float().cpu().numpy(), full.float().cpu().numpy()
    qn = q.float().cpu().numpy()
    for b in range(B):
        k, v = _seq_kv(pool_k, pool_v, bt[b], N)
        want = _oracle_rows(qn[b:b + 1], k, v, [N - 1], D ** -0.5, scale_h)
        assert_close_bf16(got_m[b:b + 1], want, what=f"config 4 merged seq {b}")
        assert_close_bf16(got_f[b:b + 1], want, what=f"config 4 unsharded seq {b}")
