"""Host logic of the serving fast path (no GPU): span rules, pool layout, row
plans, padded rows and boundary commits, checked against the oracle."""

import numpy as np
import pytest

from oracle import lastkv_oracle as O


def test_span_rules_match_reference_examples():
    from lastkv_b200.vllm_backend import chunk_aligned_new_tokens, sliver_deferred_new_tokens

    for args in [(0, 2048, 1024), (1000, 100, 1024), (1024, 1, 1024), (5, 0, 1024), (1023, 7, 1024)]:
        assert chunk_aligned_new_tokens(*args) == O.chunk_aligned_new_tokens(*args)
    # a partial sliver waits unless it reaches the boundary or ends the request
    assert sliver_deferred_new_tokens(0, 300, 1024, 5000) == 0
    assert sliver_deferred_new_tokens(0, 300, 1024, 300) == 300
    assert sliver_deferred_new_tokens(900, 300, 1024, 5000) == 124
    assert sliver_deferred_new_tokens(2048, 1, 1024, 5000) == 0  # a mid-prefill sliver waits
    assert sliver_deferred_new_tokens(2048, 1, 1024, 2049) == 1  # a decode step is the final piece


def _fast(num_slots=3, max_tokens=200, chunk=32, layers=2, order=None):
    from lastkv_b200.vllm_backend import SharedKVFastPath, SharedKVPool

    pool = SharedKVPool(num_layers=layers, num_slots=num_slots, max_sequence_tokens=max_tokens, chunk_size=chunk,
                        num_kv_heads=2, head_dim=128, device="cpu", page_order=order)
    return pool, SharedKVFastPath(pool, max_batch=8, max_tokens=256, num_q_heads=8)


def test_session_slots_are_reused_and_fail_closed():
    from lastkv_b200.contract import RMarinBackendContractError

    pool, _ = _fast(num_slots=2)
    a, b = pool.acquire(), pool.acquire()
    assert {a, b} == {0, 1}
    pool.committed[a] = 64
    with pytest.raises(RMarinBackendContractError, match="no free session slot"):
        pool.acquire()
    pool.release(a)
    assert pool.acquire() == a and pool.committed[a] == 0  # a reused slot starts with nothing committed


def test_pool_layout_matches_reference_formulas():
    pool, _ = _fast()
    # batching.py:2005-2013: src pages + scratch, ring stride (2C/16)*slots + 1
    assert pool.src_pages == pool.pages_per_slot * 3 + 1
    assert pool.ring_stride == (2 * 32 // 16) * 3 + 1
    assert pool.num_pages == pool.src_pages + 2 * pool.ring_stride
    assert pool.pool_k.shape == (pool.num_pages, 16, 2, 128)


@pytest.mark.parametrize("shuffle", [False, True])
def test_row_plans_match_oracle(shuffle):
    from lastkv_b200.vllm_backend import Span

    n = 13 * 3
    order = np.random.default_rng(3).permutation(n) if shuffle else None
    pool, fast = _fast(order=order)
    pool.committed = [64, 0, 0]
    spans = [Span(0, 70, 10), Span(2, 0, 32), Span(1, 31, 1)]
    plan = fast.plan_rows(spans)
    assert not plan["uniform"] and plan["batch"] == 3 and plan["tokens"] == 43
    lay = O.PoolLayout(num_layers=2, chunk=32, page=16, num_slots=3, src_pages=pool.src_pages)
    tok = 0
    for row, sp in enumerate(spans):
        rt, local, nsrc, seq_k, src = O.row_plan(lay, sp.slot, sp.num_computed_tokens, sp.num_query_tokens,
                                                 list(pool.src_table[sp.slot]))
        assert plan["nsrc"][row] == nsrc and plan["seqk"][row] == seq_k
        assert list(plan["bt"][row, :nsrc + len(local)]) == list(src) + local
        assert plan["ring"][tok] == rt
        assert plan["cu"][row + 1] - plan["cu"][row] == sp.num_query_tokens
        tok += sp.num_query_tokens
    assert plan["commits"] == []  # slot 0 already committed through 64


def test_uniform_decode_pads_rows_onto_scratch_pages():
    from lastkv_b200.vllm_backend import Span

    pool, fast = _fast()
    plan = fast.plan_rows([Span(0, 5, 1), Span(1, 6, 1)], num_reqs_padded=4)
    assert plan["uniform"] and plan["batch"] == 4 and plan["tokens"] == 4
    for row in (2, 3):
        assert plan["nsrc"][row] == 0 and plan["seqk"][row] == 1
        assert plan["bt"][row, 0] == pool.scratch_ring_page
        assert plan["ring"][row] == pool.scratch_ring_page * 16
        assert plan["src"][row] == pool.scratch_src_page * 16


def test_boundary_commit_is_scheduled_once_and_contiguously():
    from lastkv_b200.contract import RMarinBackendContractError
    from lastkv_b200.vllm_backend import Span

    pool, fast = _fast()
    plan = fast.plan_rows([Span(0, 32, 1)])
    assert plan["commits"] == [(0, 32)]
    pool.committed[0] = 32
    assert fast.plan_rows([Span(0, 33, 1)])["commits"] == []
    with pytest.raises(RMarinBackendContractError, match="contiguous"):
        fast.plan_rows([Span(1, 96, 1)])  # slot 1 never committed 32 / 64
    with pytest.raises(RMarinBackendContractError, match="cross"):
        fast.plan_rows([Span(2, 30, 5)])


def test_backend_class_surface():
    import torch

    from lastkv_b200.vllm_backend import SharedKVAttentionImpl, SharedKVBackend

    assert SharedKVBackend.get_name() == "CUSTOM"
    assert SharedKVBackend.get_impl_cls() is SharedKVAttentionImpl
    assert not SharedKVBackend.supports_non_causal() and not SharedKVBackend.supports_sink()
    assert SharedKVBackend.supported_dtypes == [torch.bfloat16]
    assert SharedKVBackend.forward_includes_kv_cache_update
    _, fast = _fast()
    impl = SharedKVAttentionImpl(fast, 8, 128)
    out = torch.ones(3, 8, 128)
    assert impl.forward(None, None, None, None, None, None, out) is out and float(out.abs().sum()) == 0


def test_bind_parameters_fails_closed_on_zero_scale():
    import torch

    from lastkv_b200.contract import RMarinBackendContractError

    pool, _ = _fast()
    with pytest.raises(RMarinBackendContractError, match="non-zero"):
        pool.bind_parameters(torch.zeros(2, 2), torch.tensor([[1.0, 0.0], [1.0, 1.0]]), 8)
    pool.bind_parameters(torch.zeros(2, 2), torch.ones(2, 2) * 0.7, 8)
    assert pool.out_scale.shape == (2, 8) and torch.allclose(pool.alpha, torch.full((2, 2), 0.5))
