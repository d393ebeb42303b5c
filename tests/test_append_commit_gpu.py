"""The boundary commit fused into the next step's first-layer append
(lkv_rope_norm_append_commit) against the two separate launches and the oracle.

The reference commits a finished chunk lazily, when the next step starts
(vllm/src/lastkv/vllm/backends/rmarin_flashinfer/batching.py:1099-1144); the
fused launch runs that blend (fused_qkv.py:158-201) inside the first layer's
append of that step.  Both halves must be bit-identical to the separate
launches: pools, q_out and error word.  The device-count form (one captured
launch for steps with and without a boundary) is checked at counts 0, k < rows
and rows, and with an out-of-range count, which commits nothing and records
the error while the append still lands.
"""

import numpy as np
import pytest
import torch

from oracle import lastkv_oracle as O

pytestmark = pytest.mark.gpu


def _case(seed, L, S, ppc, Hq, Hkv, D, T, top):
    """A pool with shared pages, L layer rings of 2 chunks per sequence, a finished chunk
    per sequence to commit (ring half 0) and T tokens to append into ring half 1."""
    rng = np.random.default_rng(seed)
    ring_stride = S * ppc * 2 + 1
    src = S * ppc * 3
    total = src + L * ring_stride
    pk = O.bf16_round(rng.standard_normal((total, 16, Hkv, D)))
    pv = O.bf16_round(rng.standard_normal((total, 16, Hkv, D)))
    perm = rng.permutation(src)
    raw_pages = perm[: S * ppc].reshape(S, ppc).astype(np.int32)
    ring_pages = (src + np.arange(S)[:, None] * ppc * 2 + np.arange(ppc)[None, :]).astype(np.int32)
    alpha = O.alpha_from_logits(rng.standard_normal((L, Hkv)))
    # appended tokens: layer-0 ring slots in the second half of some sequence's ring;
    # top-layer (L == 1) shared slots in pages that are not part of the commit
    seqs = rng.integers(0, S, T)
    ring_slot = ((src + seqs * ppc * 2 + ppc) * 16 + rng.permutation(ppc * 16)[:T]).astype(np.int64)
    src_slot = (perm[S * ppc: S * ppc + T].astype(np.int64) * 16 + rng.integers(0, 16, T)) if top else None
    q = O.bf16_round(rng.standard_normal((T, Hq * D)))
    k = O.bf16_round(rng.standard_normal((T, Hkv * D)))
    v = O.bf16_round(rng.standard_normal((T, Hkv * D)))
    pos = rng.integers(0, 256, T).astype(np.int64)
    cs = O.bf16_round(O.rope_cos_sin(256, D, 10000.0))
    qw = O.bf16_round(rng.uniform(0.5, 1.5, D))
    kw = O.bf16_round(rng.uniform(0.5, 1.5, D))
    inv = O.bf16_round(1.0 / rng.uniform(0.5, 2.0, Hkv))
    return dict(pk=pk, pv=pv, raw=raw_pages, ring=ring_pages, stride=ring_stride, alpha=alpha, ring_slot=ring_slot,
                src_slot=src_slot, q=q, k=k, v=v, pos=pos, cs=cs, qw=qw, kw=kw, inv=inv)


def _cu(x, dt=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dt).cuda()


def _run(c, mode, rows=None, count=None, blocks=0):
    """mode 'separate': append then blend_chunk over `rows`; 'fused': one launch."""
    from lastkv_b200 import ops

    pk, pv = _cu(c["pk"]), _cu(c["pv"])
    Hkv, D = pk.shape[2], pk.shape[3]
    flat_k, flat_v = pk.view(-1, Hkv, D), pv.view(-1, Hkv, D)
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    raw, ring = _cu(c["raw"], torch.int32), _cu(c["ring"], torch.int32)
    if rows is not None:
        raw, ring = raw[:rows].contiguous(), ring[:rows].contiguous()
    alpha = _cu(c["alpha"], torch.float32)
    top = c["src_slot"] is not None
    args = (_cu(c["q"]), _cu(c["k"]), _cu(c["v"]), _cu(c["pos"], torch.int64), _cu(c["cs"]), _cu(c["qw"]),
            _cu(c["kw"]), 1e-6, _cu(c["inv"], torch.float32), _cu(c["ring_slot"], torch.int64), flat_k, flat_v,
            _cu(c["src_slot"], torch.int64) if top else None, flat_k if top else None, flat_v if top else None)
    if mode == "separate":
        q_out = ops.rope_norm_append(*args, error_word=err)
        if raw.shape[0]:
            ops.blend_chunk(pk, pv, raw, ring, c["stride"], alpha, error_word=err)
    else:
        cnt = None if count is None else torch.tensor([count], dtype=torch.int32, device="cuda")
        commit = ops.Commit(pk, pv, raw, ring, c["stride"], alpha, count=cnt, blocks=blocks)
        q_out = ops.rope_norm_append(*args, error_word=err, commit=commit)
    torch.cuda.synchronize()
    return pk.cpu(), pv.cpu(), q_out.cpu(), err.cpu().tolist()


def _same(a, b):
    for x, y in zip(a[:3], b[:3]):
        assert torch.equal(x, y)


@pytest.mark.parametrize("L,S,ppc,Hq,Hkv,D,T,top", [
    (3, 4, 2, 16, 4, 128, 5, False),
    (1, 3, 4, 8, 1, 64, 7, True),      # single layer: layer 0 is the top layer (shared-slot stores too)
    (4, 2, 8, 32, 8, 128, 2, False),
    (2, 3, 2, 12, 12, 64, 3, False),   # 12 heads: the per-vector head advances by 32 mod 12 rows
    (2, 2, 3, 10, 5, 128, 4, False),   # 5 heads: 16 mod 5
])
def test_fused_commit_equals_append_then_blend(L, S, ppc, Hq, Hkv, D, T, top):
    c = _case(L * 31 + S, L, S, ppc, Hq, Hkv, D, T, top)
    want = _run(c, "separate")
    assert want[3][0] == 0
    got = _run(c, "fused")
    _same(got, want)
    assert got[3] == want[3]
    got_few = _run(c, "fused", blocks=3)  # fewer commit blocks than page items: each strides over many
    _same(got_few, want)
    # the blend half against the oracle directly
    ek, ev = c["pk"].copy(), c["pv"].copy()
    for s in range(S):
        for l in range(L):
            rows = c["ring"][s] + l * c["stride"]
            for pool, exp in ((c["pk"], ek), (c["pv"], ev)):
                ring = pool[rows].reshape(1, ppc * 16, Hkv, D)
                raw = pool[c["raw"][s]].reshape(ppc * 16, Hkv, D)
                exp[rows] = O.blend_chunk(ring, raw, c["alpha"][l:l + 1])[0].reshape(ppc, 16, Hkv, D)
    blended = (c["ring"][:, None, :] + np.arange(L)[None, :, None] * c["stride"]).reshape(-1)
    np.testing.assert_array_equal(got[0].float().numpy()[blended], ek[blended])
    np.testing.assert_array_equal(got[1].float().numpy()[blended], ev[blended])


@pytest.mark.parametrize("count", [0, 2, 4])
def test_device_count_commits_the_first_rows(count):
    L, S, ppc, Hq, Hkv, D, T = 2, 4, 4, 16, 4, 128, 6
    c = _case(7 + count, L, S, ppc, Hq, Hkv, D, T, False)
    want = _run(c, "separate", rows=count)
    got = _run(c, "fused", count=count, blocks=8)
    _same(got, want)
    assert got[3][0] == 0


def test_out_of_range_count_commits_nothing_and_reports():
    L, S, ppc, Hq, Hkv, D, T = 2, 3, 2, 8, 2, 64, 4
    c = _case(99, L, S, ppc, Hq, Hkv, D, T, False)
    want = _run(c, "separate", rows=0)  # the append alone
    got = _run(c, "fused", count=S + 1, blocks=4)
    _same(got, want)
    assert got[3][0] == 3 and got[3][3] == S + 1


# ------------------------------------------------------------------ the model paths


def test_model_logits_fused_commit_equal_separate(small_d128):
    """The HF model over three chunk boundaries (prefill spans and decode steps): the
    queued commit fused into the next span's layer-0 append gives bit-identical logits."""
    from tests.test_hf_model_gpu import build_small

    data = small_d128
    model = build_small(data)
    tokens = torch.from_numpy(data["tokens"]).cuda()
    B, T = tokens.shape
    outs = []
    for fuse in (True, False):
        cache = model.new_cache(B, T)
        cache.fuse_commit = fuse
        got, start = [], 0
        with torch.no_grad():
            for size in data["segments"].tolist():
                logits, cache = model(tokens[:, start:start + size], cache)
                got.append(logits.float())
                start += size
        cache.flush_commit()
        cache.check_errors()
        outs.append((torch.cat(got, 1).cpu(), cache.pool_k.cpu(), cache.pool_v.cpu()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_graph_runner_commit_graph_matches_eager(small_d128):
    """The runner's second graph (the step after a boundary, commit fused) produces the
    same tokens and pools as eager decoding with separate commits."""
    from lastkv_b200.runner import GraphDecodeRunner
    from tests.test_hf_model_gpu import build_small

    data = small_d128
    model = build_small(data)
    prompt = torch.from_numpy(data["tokens"][:, :13]).cuda()
    B, steps = prompt.shape[0], 40  # chunk 16: boundaries after positions 15, 31, 47
    with torch.no_grad():
        eager = model.new_cache(B, 64)
        eager.fuse_commit = False
        logits, _ = model(prompt, eager)
        ids = logits[:, -1].float().argmax(-1, keepdim=True)
        want = [ids]
        for _ in range(steps - 1):
            logits, _ = model(ids, eager)
            ids = logits[:, -1].float().argmax(-1, keepdim=True)
            want.append(ids)
        cache = model.new_cache(B, 64)
        runner = GraphDecodeRunner(model, cache)
        runner.prefill(prompt, 13)
        runner.capture()
        assert runner.graph_commit is not None
        got = [runner.ids.clone()]
        for _ in range(steps - 1):
            got.append(runner.step().clone())
    cache.flush_commit()
    eager.check_errors()
    cache.check_errors()
    assert torch.equal(torch.cat(got, 1).cpu(), torch.cat(want, 1).cpu())


def test_model_multi_page_chunks_fused_commit_equal_separate():
    """Chunks of 4 pages, batch 3, 3 layers, random weights: prefill spans and decode steps
    over three boundaries, fused commits vs separate blend launches, bit-identical logits
    and pools."""
    from lastkv_b200.hf import LastKVConfig, LastKVForCausalLM
    from lastkv_b200.runner import init_random_

    cfg = LastKVConfig(hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2,
                       num_hidden_layers=3, head_dim=64, vocab_size=512, chunk_size=64)
    model = LastKVForCausalLM(cfg).cuda().to(torch.bfloat16).eval()
    init_random_(model, seed=5)
    gen = torch.Generator(device="cuda").manual_seed(3)
    tokens = torch.randint(0, 512, (3, 200), generator=gen, device="cuda")
    segments = [100] + [1] * 30 + [40] + [1] * 30
    outs = []
    for fuse in (True, False):
        cache = model.new_cache(3, 200)
        cache.fuse_commit = fuse
        got, start = [], 0
        with torch.no_grad():
            for size in segments:
                logits, cache = model(tokens[:, start:start + size], cache)
                got.append(logits.float())
                start += size
        cache.flush_commit()
        cache.check_errors()
        assert cache.committed == 192
        outs.append((torch.cat(got, 1).cpu(), cache.pool_k.cpu(), cache.pool_v.cpu()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_graph_runner_multi_page_chunks_fused_equals_separate():
    """The runner's commit graph with 4-page chunks and batch 3 (page lists of several
    columns per row) against the same runner with a separate blend launch after each
    boundary: identical tokens and pools (both sides replay graphs, so every library
    GEMM runs the same kernel)."""
    from lastkv_b200.hf import LastKVConfig, LastKVForCausalLM
    from lastkv_b200.runner import GraphDecodeRunner, init_random_

    cfg = LastKVConfig(hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2,
                       num_hidden_layers=3, head_dim=64, vocab_size=512, chunk_size=64)
    model = LastKVForCausalLM(cfg).cuda().to(torch.bfloat16).eval()
    init_random_(model, seed=6)
    gen = torch.Generator(device="cuda").manual_seed(4)
    prompt = torch.randint(0, 512, (3, 60), generator=gen, device="cuda")
    steps = 80  # boundaries at 64 and 128
    runs = []
    for fuse in (True, False):
        cache = model.new_cache(3, 160)
        cache.fuse_commit = fuse
        runner = GraphDecodeRunner(model, cache)
        with torch.no_grad():
            runner.prefill(prompt, 60)
            runner.capture()
            assert (runner.graph_commit is not None) == fuse
            got = [runner.ids.clone()]
            for _ in range(steps - 1):
                got.append(runner.step().clone())
        cache.flush_commit()
        cache.check_errors()
        assert cache.committed == 128
        runs.append((torch.cat(got, 1).cpu(), cache.pool_k.cpu(), cache.pool_v.cpu()))
    for a, b in zip(*runs):
        assert torch.equal(a, b)


def test_queued_commit_is_flushed_by_reorder_and_reserve(small_d128):
    """A prompt that ends exactly on a chunk boundary leaves its commit queued; beam
    reordering and growing the cache run it first, and decoding continues with the same
    logits as the cache that blended at the boundary."""
    from tests.test_hf_model_gpu import build_small

    data = small_d128
    model = build_small(data)
    tokens = torch.from_numpy(data["tokens"]).cuda()
    order = torch.tensor([1, 0])
    outs = []
    for fuse in (True, False):
        cache = model.new_cache(2, 48)
        cache.fuse_commit = fuse
        with torch.no_grad():
            model(tokens[:, :32], cache)  # boundaries at 16 and 32 (chunk 16)
            assert (cache._pending is not None) == fuse
            cache.reorder_cache(order)
            assert cache._pending is None
            a, _ = model(tokens[order, 32:33], cache)
            model(tokens[order, 33:48], cache)  # to 48 tokens: the next boundary, its commit queued
            assert (cache._pending is not None) == fuse
            cache.reserve(80)
            assert cache._pending is None
            b, _ = model(tokens[order, 48:52], cache)
        cache.check_errors()
        outs.append((a.float().cpu(), b.float().cpu()))
    for x, y in zip(*outs):
        assert torch.equal(x, y)
