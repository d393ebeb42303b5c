"""The per-query history split of every planner here against the reference's own
dependency-free access planner (vllm/src/lastkv/vllm/backends/rmarin_flashinfer/
access_plan.py:407-474), recorded in tests/golden/access_plan.npz by
tests/golden/make_golden.py over chunk sizes 4-4096 and positions around every
boundary.  A query at position p reads the shared source for older = [0, rec),
the layer's own ring for recent + current = [rec, p + 1), and needs the LSE
merge of two passes exactly when older is not empty; the merged single call here
reads older as its first nsrc pages and the ring as the rest, so nsrc * 16 must
equal older.end, the ring window must start at recent.start and seq_k must equal
current.end."""

import os

import numpy as np
import pytest

from conftest import ROOT
from oracle import lastkv_oracle as O

GOLDEN = os.path.join(ROOT, "tests", "golden", "access_plan.npz")


def _rows():
    return np.load(GOLDEN)["rows"]


def test_fixture_covers_boundaries_and_both_layer_kinds():
    rows = _rows()
    assert len(rows) >= 700
    assert set(rows[:, 2].tolist()) == {0, 1}
    assert {4, 16, 1024, 4096} <= set(rows[:, 0].tolist())
    # the recorded ranges are the reference's own definition
    for chunk, p, _, o0, o1, r0, r1, c0, c1, merge in rows:
        cur = (p // chunk) * chunk
        assert (o0, o1, r0, r1, c0, c1) == (0, max(0, cur - chunk), max(0, cur - chunk), cur, cur, p + 1)
        assert merge == int(o1 > 0)


@pytest.mark.parametrize("chunk", [16, 32, 64, 1024, 4096])
def test_oracle_row_plan_matches_reference_planner(chunk):
    rows = _rows()
    rows = rows[rows[:, 0] == chunk]
    max_pos = int(rows[:, 1].max()) + 1
    pages = -(-max_pos // 16)
    lay = O.PoolLayout(num_layers=2, chunk=chunk, page=16, num_slots=1, src_pages=pages)
    for _, p, _, o0, o1, r0, r1, c0, c1, merge in rows:
        _, local, nsrc, seq_k, _ = O.row_plan(lay, 0, int(p), 1, list(range(pages)))
        assert nsrc * 16 == o1 and (nsrc > 0) == bool(merge)
        assert seq_k == c1
        # the ring pages hold exactly [recent.start, current.end)
        assert len(local) == -(-(c1 - r0) // 16)


@pytest.mark.parametrize("chunk", [16, 32, 64])
def test_serving_and_hf_planners_match_reference_planner(chunk):
    from lastkv_b200.hf import LastKVConfig, PagedLastKVCache
    from lastkv_b200.vllm_backend import SharedKVFastPath, SharedKVPool, Span

    rows = _rows()
    rows = rows[(rows[:, 0] == chunk) & (rows[:, 2] == 0)]
    max_tok = int(rows[:, 1].max()) + 17
    pool = SharedKVPool(num_layers=2, num_slots=1, max_sequence_tokens=max_tok, chunk_size=chunk, num_kv_heads=2,
                        head_dim=128, device="cpu")
    fast = SharedKVFastPath(pool, max_batch=1, max_tokens=8, num_q_heads=8)
    cfg = LastKVConfig(hidden_size=64, intermediate_size=96, num_attention_heads=8, num_key_value_heads=2,
                       num_hidden_layers=2, head_dim=128, vocab_size=50, chunk_size=chunk)
    cache = PagedLastKVCache(cfg, 1, max_tok, device="cpu")
    for _, p, _, o0, o1, r0, r1, c0, c1, merge in rows:
        pool.committed[0] = int(c0)  # the boundary before this chunk already committed
        plan = fast.plan_rows([Span(0, int(p), 1)])
        assert plan["nsrc"][0] * 16 == o1 and plan["seqk"][0] == c1
        cache.seen_tokens = int(p)
        h = cache.plan_host(1)
        assert h["nsrc"] * 16 == o1 and h["seq_k"] == c1 and (h["nsrc"] > 0) == bool(merge)
        # the first ring page is the page of recent.start within the 2C ring
        assert h["bt"][0, h["nsrc"]] == (r0 // 16) % cache.ring_pages
