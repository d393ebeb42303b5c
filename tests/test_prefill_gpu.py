"""tcgen05 chunked-prefill kernel vs the CPU oracle and the reference's golden calls."""

import numpy as np
import pytest
import torch

from oracle import lastkv_oracle as O
from tests.conftest import golden_calls
from tests.gpu_helpers import assert_close_bf16

pytestmark = pytest.mark.gpu


def _case(seed, lq, nk, Hq, Hkv, D, extra_pages=5):
    """Varlen spans: sequence b has lq[b] queries against nk[b] keys (last lq[b] are the span)."""
    rng = np.random.default_rng(seed)
    B = len(lq)
    pages = [-(-n // 16) for n in nk]
    W = max(1, max(pages))
    total = sum(pages) + extra_pages
    perm = rng.permutation(total)
    bt = np.zeros((B, W), np.int32)
    o = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[o:o + pages[b]]
        o += pages[b]
    pk = O.bf16_round(rng.standard_normal((total, 16, Hkv, D)))
    pv = O.bf16_round(rng.standard_normal((total, 16, Hkv, D)))
    # zero the unwritten tail of each last page (pools are zero-initialised)
    for b in range(B):
        if nk[b] % 16:
            pk[bt[b, pages[b] - 1], nk[b] % 16:] = 0
            pv[bt[b, pages[b] - 1], nk[b] % 16:] = 0
    T = sum(lq)
    q = O.bf16_round(rng.standard_normal((T, Hq, D)))
    cu = np.concatenate([[0], np.cumsum(lq)]).astype(np.int32)
    dev = dict(q=torch.from_numpy(q).cuda().bfloat16(), pool_k=torch.from_numpy(pk).cuda().bfloat16(),
               pool_v=torch.from_numpy(pv).cuda().bfloat16(), bt=torch.from_numpy(bt).cuda(),
               seq_k=torch.tensor(nk, dtype=torch.int32, device="cuda"), cu=torch.from_numpy(cu).cuda())
    host = dict(q=q, pool_k=pk, pool_v=pv, bt=bt, seq_k=np.array(nk), cu=cu)
    return dev, host


CASES = [
    # seed, lq, nk, Hq, Hkv, D, causal
    (0, [1], [1], 4, 1, 128, True),
    (1, [37], [37], 32, 8, 128, True),
    (2, [128, 5], [128, 1029], 32, 8, 128, True),
    (3, [300, 33, 129], [1300, 33, 4000], 32, 8, 128, True),
    (4, [64], [2048], 8, 8, 128, True),
    (5, [200, 17], [600, 17], 16, 2, 64, True),
    (6, [77], [1000], 12, 12, 64, False),
    (7, [256], [256 + 4680], 32, 4, 128, False),
    (8, [16, 16, 16], [16, 100, 1024], 64, 8, 128, True),
    # full output tiles (stored through shared memory by TMA) next to ragged ones,
    # for the GQA groups and head dims the cases above leave out
    (9, [300], [700], 8, 4, 128, True),              # group 2
    (10, [256, 40], [256, 900], 8, 8, 128, True),    # group 1, 128-token tiles
    (11, [130], [2000], 4, 4, 64, False),            # group 1, D 64
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"s{c[0]}_Hq{c[3]}_Hkv{c[4]}_D{c[5]}_{'c' if c[6] else 'nc'}")
def test_prefill_matches_oracle(case):
    from lastkv_b200 import ops

    seed, lq, nk, Hq, Hkv, D, causal = case
    dev, host = _case(seed, lq, nk, Hq, Hkv, D)
    s_h = np.random.default_rng(seed + 50).uniform(0.5, 1.5, Hq).astype(np.float32)
    lse = torch.empty((sum(lq), Hq), dtype=torch.float32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    out = ops.prefill_paged(dev["q"], dev["pool_k"], dev["pool_v"], dev["bt"], dev["seq_k"], dev["cu"], max(lq),
                            causal=causal, lse=lse, out_scale=torch.from_numpy(s_h).cuda(), error_word=err)
    torch.cuda.synchronize()
    assert err.cpu().tolist()[0] == 0
    ref, ref_lse = O.paged_attention(host["q"], host["pool_k"], host["pool_v"], host["bt"], host["seq_k"],
                                     host["cu"], scale=D ** -0.5, out_scale=s_h, causal=causal)
    assert_close_bf16(out.float().cpu().numpy(), ref, what="prefill")
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, rtol=1e-4, atol=2e-3)


SPLIT_CASES = [
    # seed, lq, nk, Hq, Hkv, D, kv_splits (non-causal, keys split inside one launch, then merged)
    (20, [256, 100], [256 + 4680, 100 + 3000], 32, 4, 128, 2),
    (21, [77, 300], [1000, 5000], 12, 12, 64, 3),
    (22, [130], [2100], 8, 8, 128, 8),        # 17 key blocks over 8 splits: 3 per split, the last empty
    (23, [64, 64], [64, 20], 16, 8, 128, 5),  # more splits than key blocks: empty splits merge to nothing
]


@pytest.mark.parametrize("case", SPLIT_CASES, ids=lambda c: f"s{c[0]}_D{c[5]}_S{c[6]}")
def test_prefill_key_splits_match_oracle(case):
    from lastkv_b200 import ops

    seed, lq, nk, Hq, Hkv, D, S = case
    dev, host = _case(seed, lq, nk, Hq, Hkv, D)
    s_h = np.random.default_rng(seed + 50).uniform(0.5, 1.5, Hq).astype(np.float32)
    lse = torch.empty((sum(lq), Hq), dtype=torch.float32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    out = ops.prefill_paged(dev["q"], dev["pool_k"], dev["pool_v"], dev["bt"], dev["seq_k"], dev["cu"], max(lq),
                            causal=False, lse=lse, out_scale=torch.from_numpy(s_h).cuda(), error_word=err,
                            kv_splits=S)
    one = ops.prefill_paged(dev["q"], dev["pool_k"], dev["pool_v"], dev["bt"], dev["seq_k"], dev["cu"], max(lq),
                            causal=False, out_scale=torch.from_numpy(s_h).cuda(), kv_splits=1)
    torch.cuda.synchronize()
    assert err.cpu().tolist()[0] == 0
    ref, ref_lse = O.paged_attention(host["q"], host["pool_k"], host["pool_v"], host["bt"], host["seq_k"],
                                     host["cu"], scale=D ** -0.5, out_scale=s_h, causal=False)
    assert_close_bf16(out.float().cpu().numpy(), ref, what="split prefill")
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, rtol=1e-4, atol=2e-3)
    # the same attention as the unsplit kernel up to the order of the fp32 sums
    assert_close_bf16(out.float().cpu().numpy(), one.float().cpu().numpy(), max_abs=1.6e-2, rel_l2=4e-3,
                      what="split vs unsplit")


def test_prefill_split_plan_is_one_for_causal_and_short_keys():
    from lastkv_b200 import ops

    assert ops.prefill_split_plan(2, 4680, 12, 12, 128, 2048, True) == 1
    assert ops.prefill_split_plan(2, 4680, 12, 12, 128, 20, False) == 1
    # Wan-1.3B block attention (batch 2, 12 heads, 4680 queries x 32760 keys): 456 CTAs on the SMs
    s = ops.prefill_split_plan(2, 4680, 12, 12, 128, 2048, False)
    assert 1 <= s <= 8


def test_prefill_single_token_equals_decode():
    from lastkv_b200 import ops

    lq = [1] * 6
    nk = [1, 16, 17, 500, 2048, 3333]
    dev, _ = _case(12, lq, nk, 32, 8, 128)
    a = ops.prefill_paged(dev["q"], dev["pool_k"], dev["pool_v"], dev["bt"], dev["seq_k"], dev["cu"], 1)
    b = ops.decode_paged(dev["q"], dev["pool_k"], dev["pool_v"], dev["bt"], dev["seq_k"])
    assert_close_bf16(a.float().cpu().numpy(), b.float().cpu().numpy(), max_abs=1.6e-2, rel_l2=6e-3, what="1-token")


def test_prefill_reference_golden_calls(small_d128):
    """The reference's recorded chunked-prefill calls (16, 16 and 5 tokens, batch 2) on a bf16 pool."""
    from lastkv_b200 import ops

    data = small_d128
    C, L = int(data["chunk"]), int(data["num_layers"])
    hq, hkv, d = int(data["num_heads"]), int(data["num_kv_heads"]), int(data["head_dim"])
    B = data["tokens"].shape[0]
    per = -(-data["tokens"].shape[1] // 16)
    lay = O.PoolLayout(num_layers=L, chunk=C, page=16, num_slots=B, src_pages=B * per)
    perm = np.random.default_rng(8).permutation(B * per)
    state = O.PagedLastKV(layout=lay, hkv=hkv, d=d, batch=B, alpha=O.alpha_from_logits(data["alpha_logits"]),
                          v_scale=data["v_scale"], bf16=True,
                          src_page_lists=[list(perm[b * per:(b + 1) * per]) for b in range(B)])
    checked = 0
    for rec in golden_calls(data):
        layer, start, lq = rec["layer"], rec["start"], rec["lq"]
        for b in range(B):
            state.append(layer, b, rec["k_new"][b].transpose(1, 0, 2), rec["v_new"][b].transpose(1, 0, 2), start)
        if lq > 1:
            rows = [state.block_table(layer, b, start, lq) for b in range(B)]
            W = max(len(r[0]) for r in rows)
            bt = np.zeros((B, W), np.int32)
            for b, (row, _) in enumerate(rows):
                bt[b, :len(row)] = row
            q = O.bf16_round(rec["q"].transpose(0, 2, 1, 3).reshape(B * lq, hq, d))
            s_q = np.repeat(data["v_scale"][layer], hq // hkv).astype(np.float32)
            out = ops.prefill_paged(torch.from_numpy(q).cuda().bfloat16(),
                                    torch.from_numpy(state.pool_k).cuda().bfloat16(),
                                    torch.from_numpy(state.pool_v).cuda().bfloat16(), torch.from_numpy(bt).cuda(),
                                    torch.tensor([r[1] for r in rows], dtype=torch.int32, device="cuda"),
                                    torch.tensor([0, lq, 2 * lq], dtype=torch.int32, device="cuda"), lq,
                                    out_scale=torch.from_numpy(s_q).cuda())
            exp = rec["out"].transpose(0, 2, 1, 3).reshape(B * lq, hq, d)
            assert_close_bf16(out.float().cpu().numpy(), exp, what=f"golden prefill layer {layer}@{start}")
            checked += 1
        if layer == L - 1:
            for b in range(B):
                state.commit_if_boundary(b, start + lq)
    assert checked == 3 * L


def test_prefill_graph_capture_replays_identically():
    from lastkv_b200 import ops

    dev, _ = _case(21, [200, 300], [1200, 300], 32, 8, 128)
    out = torch.empty((500, 32, 128), dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    ops.prefill_paged(dev["q"], dev["pool_k"], dev["pool_v"], dev["bt"], dev["seq_k"], dev["cu"], 300, out=out,
                      error_word=err)
    first = out.clone()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            ops.prefill_paged(dev["q"], dev["pool_k"], dev["pool_v"], dev["bt"], dev["seq_k"], dev["cu"], 300,
                              out=out, error_word=err)
    torch.cuda.current_stream().wait_stream(s)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    assert err.cpu().tolist()[0] == 0


def test_prefill_key_split_graph_capture_with_caller_partials():
    """Key-split non-causal prefill with caller-owned partials records into a CUDA graph
    and replays bit for bit (the split launch and its merge, no allocation)."""
    from lastkv_b200 import ops

    dev, _ = _case(24, [256, 100], [3000, 2500], 16, 4, 128)
    T, Hq, D, S = 356, 16, 128, 3
    out = torch.empty((T, Hq, D), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((T, Hq), dtype=torch.float32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    parts = (torch.empty((S, T * Hq, D), device="cuda"), torch.empty((S, T * Hq), device="cuda"))

    def call():
        ops.prefill_paged(dev["q"], dev["pool_k"], dev["pool_v"], dev["bt"], dev["seq_k"], dev["cu"], 256,
                          causal=False, out=out, lse=lse, error_word=err, kv_splits=S, partials=parts)

    call()
    first, first_lse = out.clone(), lse.clone()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            call()
    torch.cuda.current_stream().wait_stream(s)
    out.zero_()
    lse.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first) and torch.equal(lse, first_lse)
    assert err.cpu().tolist()[0] == 0
