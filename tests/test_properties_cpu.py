"""Property-based checks of the host-side planning and the oracle's merge
(hypothesis; CPU only): random chunk sizes, batch sizes and span sequences
instead of fixed examples.

* The HF cache's span plan (block tables, seq_k, ring and shared-page token
  slots) equals the oracle's row plan for any sequence of spans that respects
  the chunk boundaries (the only spans the model issues).
* Splitting a key set into any number of disjoint parts and LSE-merging the
  parts' attention reproduces attention over the whole set.
* The context-parallel shard plan covers every page exactly once and
  balances pages (ring included) across ranks.
"""

import numpy as np
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from oracle import lastkv_oracle as O

SETTINGS = settings(max_examples=60, deadline=None, suppress_health_check=[HealthCheck.too_slow])


def _spans(draw, chunk, total):
    """A sequence of span lengths from position 0 that never crosses a chunk boundary."""
    spans, pos = [], 0
    while pos < total:
        room = min(chunk - pos % chunk, total - pos)
        n = draw(st.integers(1, room))
        spans.append(n)
        pos += n
    return spans


@st.composite
def _plan_case(draw):
    chunk = draw(st.sampled_from([16, 32, 64]))
    B = draw(st.integers(1, 4))
    total = draw(st.integers(1, 6 * chunk))
    spans = _spans(draw, chunk, total)
    shuffle = draw(st.booleans())
    seed = draw(st.integers(0, 2 ** 16))
    return chunk, B, total, spans, shuffle, seed


@SETTINGS
@given(_plan_case())
def test_span_plans_match_oracle_for_any_chunked_span_sequence(case):
    from lastkv_b200.hf import LastKVConfig, PagedLastKVCache

    chunk, B, total, spans, shuffle, seed = case
    cfg = LastKVConfig(hidden_size=64, intermediate_size=96, num_attention_heads=8, num_key_value_heads=2,
                       num_hidden_layers=2, head_dim=128, vocab_size=50, chunk_size=chunk)
    pages = B * -(-total // 16)
    order = np.random.default_rng(seed).permutation(pages) if shuffle else None
    cache = PagedLastKVCache(cfg, B, total, device="cpu", page_order=order)
    lay = O.PoolLayout(num_layers=2, chunk=chunk, page=16, num_slots=B, src_pages=cache.src_pages)
    for n in spans:
        seen = cache.seen_tokens
        h = cache.plan_host(n)
        for b in range(B):
            ring_tok, local, nsrc, seq_k = O.row_plan(lay, b, seen, n, list(cache.src_table[b]))[:4]
            assert h["nsrc"] == nsrc and h["seq_k"] == seq_k == seen + n
            assert list(h["bt"][b, :nsrc + len(local)]) == list(cache.src_table[b, :nsrc]) + list(local)
            assert h["ring_tok"][b * n] == ring_tok
            pos = seen + np.arange(n)
            np.testing.assert_array_equal(h["src_tok"][b * n:(b + 1) * n],
                                          cache.src_table[b, pos // 16] * 16 + pos % 16)
        cache.seen_tokens += n  # advance without device work (plan_host is pure host logic)


@st.composite
def _merge_case(draw):
    nk = draw(st.integers(1, 60))
    cuts = sorted(set(draw(st.lists(st.integers(0, nk), max_size=5))))
    return nk, [0] + cuts + [nk], draw(st.integers(0, 2 ** 16))


@SETTINGS
@given(_merge_case())
def test_lse_merge_of_any_key_partition_is_exact(case):
    nk, bounds, seed = case
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((1, 4, 16))
    k = rng.standard_normal((nk, 2, 16))
    v = rng.standard_normal((nk, 2, 16))
    full, full_lse = O.attention(q, k, v, scale=0.25, causal=False)
    parts_o, parts_l = [], []
    for lo, hi in zip(bounds, bounds[1:]):
        if hi == lo:  # an empty shard: zero output, -inf LSE
            parts_o.append(np.zeros_like(full))
            parts_l.append(np.full(full_lse.shape, -np.inf))
            continue
        o, lse = O.attention(q, k[lo:hi], v[lo:hi], scale=0.25, causal=False)
        parts_o.append(o)
        parts_l.append(lse)
    o, lse = O.merge_many(parts_o, parts_l)
    np.testing.assert_allclose(o, full, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(lse, full_lse, rtol=1e-12, atol=1e-12)


@SETTINGS
@given(st.integers(0, 20000), st.integers(1, 4096), st.integers(1, 8))
def test_shard_plan_covers_and_balances(nsrc, window, world):
    from lastkv_b200.context_parallel import plan_shard

    plans = [plan_shard(nsrc, window, 16, world, r) for r in range(world)]
    assert plans[0].p0 == 0 and plans[-1].p1 == nsrc
    assert all(a.p1 == b.p0 and a.p0 <= a.p1 for a, b in zip(plans, plans[1:]))
    assert sum(p.seq_k for p in plans) == nsrc * 16 + window
    assert [p.ring_pages for p in plans[:-1]] == [0] * (world - 1)
    load = [p.p1 - p.p0 + p.ring_pages for p in plans]
    ring = -(-window // 16)
    if world > 1 and ring <= (nsrc + ring) // world:
        # the ring fits in the last rank's share: every rank streams about the same pages
        assert max(load) - min(load) <= 1 + world
