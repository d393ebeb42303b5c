"""Split-KV decode kernel vs the CPU oracle (and the reference's golden calls)."""

import numpy as np
import pytest
import torch

from oracle import lastkv_oracle as O
from tests.conftest import golden_calls
from tests.gpu_helpers import assert_close_bf16, make_paged_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lastkv_b200 import _capi

    _capi.load()
    assert _capi.lib().lkv_check_device(torch.cuda.current_device()) == 0


CASES = [
    # seed, B, Hq, Hkv, D, lens
    (0, 1, 4, 1, 128, [1]),
    (1, 3, 32, 8, 128, [15, 16, 17]),
    (2, 4, 8, 8, 128, [100, 1000, 33, 250]),
    (3, 2, 16, 8, 64, [777, 5000]),
    (4, 5, 16, 2, 128, [4096, 1, 3000, 64, 65]),
    (5, 2, 12, 12, 64, [640, 513]),
    (6, 64, 32, 8, 128, [513] * 64),
    (7, 3, 8, 2, 128, [0, 17, 0]),  # rows with no keys: zero output, -inf LSE (padding rows)
    (8, 2, 4, 4, 64, [0, 0]),
    (9, 3, 32, 4, 64, [300, 2000, 17]),  # GQA group 8 at D 64 (the merge takes heads four at a time)
    # many ragged items per persistent CTA (batch 200 x 2 KV heads x splits > resident CTAs)
    (10, 200, 16, 2, 128, [(37 * i * i + 11 * i) % 3001 for i in range(200)]),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"B{c[1]}_Hq{c[2]}_Hkv{c[3]}_D{c[4]}")
def test_decode_matches_oracle(case):
    from lastkv_b200 import ops

    seed, B, Hq, Hkv, D, lens = case
    t, n = make_paged_case(seed, B, Hq, Hkv, D, lens)
    rng = np.random.default_rng(seed + 100)
    scale_h = rng.uniform(0.5, 1.5, Hq).astype(np.float32)
    lse = torch.empty((B, Hq), dtype=torch.float32, device="cuda")
    out = ops.decode_paged(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], lse=lse,
                           out_scale=torch.from_numpy(scale_h).cuda())
    ref, ref_lse = O.paged_attention(n["q"], n["pool_k"], n["pool_v"], n["bt"], n["seq_k"], n["cu"],
                                     scale=D ** -0.5, out_scale=scale_h)
    assert_close_bf16(out.float().cpu().numpy(), ref, what="decode out")
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, rtol=1e-4, atol=1e-3)


def test_decode_partial_then_merge_equals_full():
    """Context-parallel form: shard each history in three, merge the partials."""
    from lastkv_b200 import ops

    B, Hq, Hkv, D = 4, 32, 8, 128
    lens = [3000, 1600, 49, 2047]
    t, n = make_paged_case(11, B, Hq, Hkv, D, lens)
    full = ops.decode_paged(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"])
    os_, ls = [], []
    for lo, hi in ((0, 0.3), (0.3, 0.31), (0.31, 1.0)):
        # page-aligned shards of each sequence
        bt_s, sk = [], []
        W = t["bt"].shape[1]
        for b, L in enumerate(lens):
            p0 = int(lo * (L // 16)) * 16
            p1 = L if hi == 1.0 else int(hi * (L // 16)) * 16
            pages = n["bt"][b, p0 // 16:-(-p1 // 16)]
            row = np.zeros(W, np.int32)
            row[:len(pages)] = pages
            bt_s.append(row)
            sk.append(p1 - p0)
        o, l = ops.decode_paged(t["q"], t["pool_k"], t["pool_v"], torch.from_numpy(np.stack(bt_s)).cuda(),
                                torch.tensor(sk, dtype=torch.int32, device="cuda"), partial=True)
        os_.append(o)
        ls.append(l)
    merged = ops.merge_partials(torch.stack(os_).contiguous(), torch.stack(ls).contiguous())
    assert_close_bf16(merged.float().cpu().numpy(), full.float().cpu().numpy(), max_abs=1.6e-2, rel_l2=5e-3,
                      what="merge")


def test_context_parallel_layer_single_rank_equals_decode():
    """ContextParallelDecode's kernel path (partial decode -> merge kernel) on one rank."""
    from lastkv_b200 import ops
    from lastkv_b200.context_parallel import ContextParallelDecode

    B, Hq, Hkv, D = 4, 32, 8, 128
    t, _ = make_paged_case(13, B, Hq, Hkv, D, [9000, 100, 4097, 1])
    scale = torch.rand(Hq, device="cuda") + 0.5
    cp = ContextParallelDecode()
    a = cp.layer(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], out_scale=scale)
    b = ops.decode_paged(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], out_scale=scale)
    assert_close_bf16(a.float().cpu().numpy().reshape(B, Hq, D), b.float().cpu().numpy(), max_abs=1.6e-2,
                      rel_l2=6e-3, what="cp single rank")


def test_decode_empty_sequence_and_nan_tail():
    from lastkv_b200 import ops

    B, Hq, Hkv, D = 3, 8, 2, 128
    lens = [0, 21, 16]
    t, n = make_paged_case(5, B, Hq, Hkv, D, lens)
    # poison the rows past the end of sequence 1's last page
    last_page = int(n["bt"][1, 1])
    t["pool_v"][last_page, 5:] = float("nan")
    t["pool_k"][last_page, 5:] = float("nan")
    n["pool_v"][last_page, 5:] = 0.0
    n["pool_k"][last_page, 5:] = 0.0
    lse = torch.empty((B, Hq), dtype=torch.float32, device="cuda")
    out = ops.decode_paged(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], lse=lse)
    o = out.float().cpu().numpy()
    assert np.all(o[0] == 0) and np.all(np.isneginf(lse[0].cpu().numpy()))
    ref, _ = O.paged_attention(n["q"], n["pool_k"], n["pool_v"], n["bt"], n["seq_k"], n["cu"], scale=D ** -0.5)
    assert_close_bf16(o[1:], ref[1:], what="nan tail")


def test_decode_is_deterministic_and_graph_capturable():
    from lastkv_b200 import ops

    t, _ = make_paged_case(9, 8, 32, 8, 128, [1234] * 8)
    ws = ops.Workspace.for_decode(8, 32, 128, t["bt"].shape[1])
    out = torch.empty((8, 32, 128), dtype=torch.bfloat16, device="cuda")
    ops.decode_paged(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], out=out, workspace=ws)
    first = out.clone()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            ops.decode_paged(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], out=out, workspace=ws)
    torch.cuda.current_stream().wait_stream(s)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    assert ws.error()[0] == 0


def test_decode_reference_golden_calls(small_d128):
    """Replay the reference's recorded decode calls (bf16 pool) through the kernel."""
    from lastkv_b200 import ops

    data = small_d128
    C, L = int(data["chunk"]), int(data["num_layers"])
    hq, hkv, d = int(data["num_heads"]), int(data["num_kv_heads"]), int(data["head_dim"])
    B = data["tokens"].shape[0]
    total = data["tokens"].shape[1]
    per = -(-total // 16)
    lay = O.PoolLayout(num_layers=L, chunk=C, page=16, num_slots=B, src_pages=B * per)
    perm = np.random.default_rng(4).permutation(B * per)
    state = O.PagedLastKV(layout=lay, hkv=hkv, d=d, batch=B, alpha=O.alpha_from_logits(data["alpha_logits"]),
                          v_scale=data["v_scale"], bf16=True,
                          src_page_lists=[list(perm[b * per:(b + 1) * per]) for b in range(B)])
    checked = 0
    for rec in golden_calls(data):
        layer, start, lq = rec["layer"], rec["start"], rec["lq"]
        for b in range(B):
            state.append(layer, b, rec["k_new"][b].transpose(1, 0, 2), rec["v_new"][b].transpose(1, 0, 2), start)
        if lq == 1:
            bts, sks = zip(*(state.block_table(layer, b, start, 1) for b in range(B)))
            W = max(len(x) for x in bts)
            bt = np.zeros((B, W), np.int32)
            for b, row in enumerate(bts):
                bt[b, :len(row)] = row
            q = torch.from_numpy(O.bf16_round(rec["q"][:, :, 0, :])).cuda().to(torch.bfloat16)
            s_q = np.repeat(data["v_scale"][layer], hq // hkv).astype(np.float32)
            out = ops.decode_paged(q, torch.from_numpy(state.pool_k).cuda().to(torch.bfloat16),
                                   torch.from_numpy(state.pool_v).cuda().to(torch.bfloat16),
                                   torch.from_numpy(bt).cuda(), torch.tensor(sks, dtype=torch.int32, device="cuda"),
                                   out_scale=torch.from_numpy(s_q).cuda())
            assert_close_bf16(out.float().cpu().numpy(), rec["out"][:, :, 0, :], what=f"golden layer {layer}@{start}")
            checked += 1
        if layer == L - 1:
            for b in range(B):
                state.commit_if_boundary(b, start + lq)
    assert checked == 27 * L


def test_one_workspace_serves_split_decodes_of_any_batch():
    """A workspace sized for the largest batch serves split decodes of different batch
    sizes in any order (the split layout follows each call's rows): each matches the oracle."""
    from lastkv_b200 import ops

    Hq, Hkv, D = 32, 8, 128
    ws = ops.Workspace.for_decode(48, Hq, D, 256, device="cuda")
    for seed, B in ((60, 8), (61, 48), (62, 3), (63, 48), (64, 8)):
        lens = list(np.random.default_rng(seed).integers(1500, 4000, B))
        t, n = make_paged_case(seed, B, Hq, Hkv, D, lens)
        splits, launches = ops.decode_plan(B, Hq, Hkv, D, t["bt"].shape[1], ws)
        assert splits > 1 and launches == 2, (splits, launches)
        lse = torch.empty((B, Hq), dtype=torch.float32, device="cuda")
        out = ops.decode_paged(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], lse=lse, workspace=ws)
        ref, ref_lse = O.paged_attention(n["q"], n["pool_k"], n["pool_v"], n["bt"], n["seq_k"], n["cu"],
                                         scale=D ** -0.5)
        assert_close_bf16(out.float().cpu().numpy(), ref, what=f"batch {B}")
        np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, rtol=1e-4, atol=1e-3)
    assert ws.error()[0] == 0


@pytest.mark.parametrize("case", [CASES[2], CASES[4], CASES[6]], ids=["B4", "B5_ragged", "B64"])
def test_l2_keep_changes_no_result(case):
    """LKV_DECODE_L2_KEEP only changes the L2 eviction hint of the page loads (batches up
    to 16 keep the oldest pages; larger ones ignore it): outputs and LSE bit-identical."""
    from lastkv_b200 import ops

    seed, B, Hq, Hkv, D, lens = case
    t, _ = make_paged_case(seed, B, Hq, Hkv, D, lens)
    res = []
    for keep in (False, True, True):
        lse = torch.empty((B, Hq), dtype=torch.float32, device="cuda")
        out = ops.decode_paged(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], lse=lse, l2_keep=keep)
        res.append((out.cpu(), lse.cpu()))
    for o, l in res[1:]:
        assert torch.equal(o, res[0][0]) and torch.equal(l, res[0][1])
