"""Host logic of the HF drop-in (no GPU): span plans match the oracle's row plan,
config validation fails closed, and the module tree matches the reference's
parameter names."""

import numpy as np
import pytest
import torch

from oracle import lastkv_oracle as O


def _cfg(**kw):
    from lastkv_b200.hf import LastKVConfig

    base = dict(hidden_size=64, intermediate_size=96, num_attention_heads=8, num_key_value_heads=2,
                num_hidden_layers=3, head_dim=128, vocab_size=50, chunk_size=32)
    base.update(kw)
    return LastKVConfig(**base)


def test_config_rejects_unsupported_shapes():
    from lastkv_b200.contract import RMarinBackendContractError

    with pytest.raises(RMarinBackendContractError):
        _cfg(head_dim=8)
    with pytest.raises(RMarinBackendContractError):
        _cfg(chunk_size=4)
    with pytest.raises(RMarinBackendContractError):
        _cfg(num_attention_heads=12, num_key_value_heads=8)


@pytest.mark.parametrize("shuffle", [False, True])
def test_span_plan_matches_oracle_row_plan(shuffle):
    from lastkv_b200.hf import PagedLastKVCache

    cfg = _cfg()
    B, max_tokens = 3, 200
    pages = B * -(-max_tokens // 16)
    order = np.random.default_rng(0).permutation(pages) if shuffle else None
    cache = PagedLastKVCache(cfg, B, max_tokens, device="cpu", page_order=order)
    lay = O.PoolLayout(num_layers=cfg.num_hidden_layers, chunk=cfg.chunk_size, page=16, num_slots=B,
                       src_pages=cache.src_pages)
    assert cache.ring_stride == lay.ring_stride and cache.num_pages == lay.total_pages
    for seen, n in [(0, 5), (5, 27), (32, 1), (95, 1), (96, 32), (150, 10)]:
        cache.seen_tokens = seen
        h = cache.plan_host(n)
        for b in range(B):
            ring_tok, local, nsrc, seq_k, src = O.row_plan(lay, b, seen, n, list(cache.src_table[b]))
            assert h["nsrc"] == nsrc and h["seq_k"] == seq_k
            row = list(h["bt"][b, :nsrc + len(local)])
            assert row == list(src) + local
            for layer in range(cfg.num_hidden_layers):
                full = [int(x) for x in row[:nsrc]] + [int(x) + int(cache.ring_base[layer]) for x in row[nsrc:]]
                assert full == O.merged_block_table(lay, layer, src, local)
            assert h["ring_tok"][b * n] == ring_tok
            for i in range(n):
                pos = seen + i
                assert h["src_tok"][b * n + i] == cache.src_table[b, pos // 16] * 16 + pos % 16


def test_span_may_not_cross_chunk_boundary():
    from lastkv_b200.contract import RMarinBackendContractError
    from lastkv_b200.hf import PagedLastKVCache

    cache = PagedLastKVCache(_cfg(), 1, 100, device="cpu")
    cache.seen_tokens = 30
    with pytest.raises(RMarinBackendContractError, match="cross"):
        cache.plan_host(5)
    with pytest.raises(RMarinBackendContractError, match="capacity"):
        cache.seen_tokens = 96
        cache.plan_host(10)


def test_parameter_names_match_reference(small_d128):
    from lastkv_b200.hf import LastKVConfig, LastKVForCausalLM

    d = small_d128
    cfg = LastKVConfig(hidden_size=int(d["hidden_size"]), intermediate_size=int(d["intermediate_size"]),
                       num_attention_heads=int(d["num_heads"]), num_key_value_heads=int(d["num_kv_heads"]),
                       num_hidden_layers=int(d["num_layers"]), head_dim=int(d["head_dim"]),
                       vocab_size=int(d["vocab_size"]), chunk_size=int(d["chunk"]),
                       deep_v_scale_init=d["v_scale"].tolist())
    model = LastKVForCausalLM(cfg)
    ref_names = {k[2:] for k in d if k.startswith("w_")}
    assert set(model.state_dict()) == ref_names
    model.load_reference_state_dict({k[2:]: torch.from_numpy(v) for k, v in d.items() if k.startswith("w_")})
    with pytest.raises(ValueError, match="strict"):
        state = {k[2:]: torch.from_numpy(v) for k, v in d.items() if k.startswith("w_")}
        state.pop("model.layers.0.self_attn.deep_v_scale")
        model.load_reference_state_dict(state)


def test_8b_parameter_layout_without_allocating():
    """The reference's 8B layout check (llm/tests/test_llm_inference.py:137-149) on this module tree."""
    from lastkv_b200.hf import LastKVConfig, LastKVForCausalLM

    cfg = LastKVConfig(hidden_size=4096, intermediate_size=14336, num_attention_heads=32, num_key_value_heads=8,
                       num_hidden_layers=32, head_dim=128, vocab_size=128256, chunk_size=1024, rms_norm_eps=1e-5)
    with torch.device("meta"):
        model = LastKVForCausalLM(cfg)
    state = model.state_dict()
    assert len(state) == 419
    assert sum(t.numel() for t in state.values()) == 8_030_269_952
    assert state["model.layers.31.self_attn.prev_chunk_alphas"].shape == (8,)
    assert state["model.layers.0.self_attn.deep_v_scale"].shape == (8,)
    assert state["lm_head.weight"].shape == (128256, 4096)


def test_llama3_rope_scaling_matches_transformers():
    from transformers import LlamaConfig
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    from lastkv_b200.hf import _llama3_inv_freq

    scaling = {"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
               "original_max_position_embeddings": 8192, "rope_type": "llama3"}
    cfg = LlamaConfig(hidden_size=4096, num_attention_heads=32, head_dim=128, rope_theta=500000.0,
                      rope_scaling=scaling, max_position_embeddings=131072)
    ref, _ = ROPE_INIT_FUNCTIONS["llama3"](cfg, "cpu")
    inv = 1.0 / (500000.0 ** (torch.arange(0, 128, 2, dtype=torch.int64).float() / 128))
    torch.testing.assert_close(_llama3_inv_freq(inv, scaling), ref, rtol=1e-6, atol=0)
