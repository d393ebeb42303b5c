"""The reference's Hugging Face surface (``lastkv_b200.llm``) on the host.

The reference's own tests (llm/tests/test_llm_inference.py) drive
``CustomRecurrentMarinAKV254ReuseKVForCausalLM`` through its config checks,
strict loading, forward validation and ``generate``.  Here the same calls run
against this package's class; the kernel forward needs a GPU, so the generation
plumbing (cache hand-back, one new token per step, cache growth) is exercised
with the inner model replaced by a host stand-in that advances the cache.
"""

import tempfile

import numpy as np
import pytest
import torch

from tests.conftest import load_golden


def _small_config(**over):
    from lastkv_b200.llm import CustomRecurrentMarinAKV254ReuseKVConfig

    d = load_golden("small_d128.npz")
    kw = dict(hidden_size=int(d["hidden_size"]), intermediate_size=int(d["intermediate_size"]),
              num_attention_heads=int(d["num_heads"]), num_key_value_heads=int(d["num_kv_heads"]),
              num_hidden_layers=int(d["num_layers"]), head_dim=int(d["head_dim"]), vocab_size=int(d["vocab_size"]),
              chunk_size=int(d["chunk"]), rms_norm_eps=float(d["eps"]), rope_theta=float(d["rope_theta"]),
              deep_v_scale_init=d["v_scale"].tolist(), tie_word_embeddings=False, bos_token_id=1,
              eos_token_id=None, pad_token_id=0)
    kw.update(over)
    return CustomRecurrentMarinAKV254ReuseKVConfig(**kw), d


def test_config_checks_match_the_reference():
    from lastkv_b200.llm import CustomRecurrentMarinAKV254ReuseKVConfig as C

    base = dict(hidden_size=64, intermediate_size=96, num_attention_heads=4, num_key_value_heads=2,
                num_hidden_layers=3, head_dim=16, vocab_size=50)
    c = C(**base, chunk_size=8)
    assert c.model_type == "custom_recurrent_marin_akv254_reusekv" and c.akv254_kv_mode == "reusekv"
    assert c.architectures == ["CustomRecurrentMarinAKV254ReuseKVForCausalLM"] and c._attn_implementation == "sdpa"
    with pytest.raises(ValueError, match="chunk_size must be a positive integer"):
        C(**base, chunk_size=0)
    with pytest.raises(ValueError, match="final-layer KV reuse"):
        C(**base, v_gap=1)
    with pytest.raises(ValueError, match="deep_rescale_mode='v'"):
        C(**base, deep_rescale_mode="kv")
    with pytest.raises(ValueError, match="deep_rescale_mode='v'"):
        C(**base, deep_scale_frozen=True)
    with pytest.raises(ValueError, match="divisible"):
        C(**dict(base, num_key_value_heads=3))
    from transformers import AutoConfig

    assert isinstance(AutoConfig.for_model("custom_recurrent_marin_akv254_reusekv", **base), C)


def test_state_dict_names_are_the_references_and_load_strictly():
    """The golden file holds the reference model's own state dict (recorded from lastkv.llm)."""
    from transformers import AutoModelForCausalLM

    from lastkv_b200.llm import CustomRecurrentMarinAKV254ReuseKVForCausalLM as M

    cfg, d = _small_config()
    model = M(cfg)
    ref = {k[2:]: torch.from_numpy(v) for k, v in d.items() if k.startswith("w_")}
    assert set(model.state_dict()) == set(ref)
    model.load_state_dict(ref, strict=True)
    tmp = tempfile.mkdtemp()
    model.save_pretrained(tmp)
    again = AutoModelForCausalLM.from_pretrained(tmp)
    assert type(again) is M
    assert all(torch.equal(a, b) for a, b in zip(model.state_dict().values(), again.state_dict().values()))
    with pytest.raises(ValueError, match="strict LastKV model match"):
        M.from_pretrained(tmp, config=_small_config(num_hidden_layers=3, deep_v_scale_init=1.0)[0])


def test_forward_rejects_what_the_reference_rejects():
    from lastkv_b200.llm import CustomRecurrentMarinAKV254ReuseKVForCausalLM as M

    model = M(_small_config()[0])
    ids = torch.tensor([[1, 2, 3]])
    with pytest.raises(ValueError, match="inference logits"):
        model(ids, labels=ids)
    with pytest.raises(ValueError, match="inference logits"):
        model(ids, output_attentions=True)
    with pytest.raises(ValueError, match="Packed-document"):
        model(ids, cu_seqlens=torch.tensor([0, 3]))
    with pytest.raises(ValueError, match="exactly one"):
        model()
    with pytest.raises(ValueError, match="unpadded"):
        model(ids, attention_mask=torch.tensor([[0, 1, 1]]))
    with pytest.raises(TypeError, match="LastKVCache"):
        model(ids, past_key_values=object())


def test_prepare_inputs_for_generation_passes_only_unseen_tokens():
    from lastkv_b200.llm import CustomRecurrentMarinAKV254ReuseKVForCausalLM as M

    model = M(_small_config()[0])

    class Seen:
        def get_seq_length(self):
            return 5

    ids = torch.arange(7)[None]
    out = model.prepare_inputs_for_generation(ids, past_key_values=Seen(), position_ids=torch.arange(7)[None])
    assert out["input_ids"].tolist() == [[5, 6]] and out["position_ids"].tolist() == [[5, 6]]
    assert out["logits_to_keep"] == 1 and out["use_cache"] is True
    out = model.prepare_inputs_for_generation(ids[:, :5], past_key_values=Seen())
    assert out["input_ids"].tolist() == [[4]]
    out = model.prepare_inputs_for_generation(ids, past_key_values=None)
    assert out["input_ids"].shape == (1, 7) and out["past_key_values"] is None


def test_generate_hands_the_paged_cache_back_and_grows_it(monkeypatch):
    """generate() on the host with the kernel forward replaced by a stand-in: the model
    creates one PagedLastKVCache, generate passes it back every step with one new token,
    and the cache grows (contents kept) past its first capacity."""
    from lastkv_b200 import _capi
    from lastkv_b200.hf import LastKVModel, PagedLastKVCache
    from lastkv_b200.llm import CustomRecurrentMarinAKV254ReuseKVForCausalLM as M

    _capi.load()  # the cache sizes its decode workspace through the library (host-only call)
    cfg, _ = _small_config()
    model = M(cfg).eval()
    model.new_cache = lambda batch, max_tokens, **kw: PagedLastKVCache(  # host tensors for this test
        model.model.config, batch, max_tokens, device="cpu", dtype=torch.float32)
    calls, caches = [], []

    def stand_in(self, input_ids, cache, inputs_embeds=None, position_ids=None):
        calls.append((input_ids.shape[1], id(cache), cache.seen_tokens, cache.max_tokens))
        caches[:] = [cache]
        # mark the pages this span lands in, so growth can be checked to keep them
        for t in range(cache.seen_tokens, cache.seen_tokens + input_ids.shape[1]):
            cache.pool_k.view(-1, cache.hkv, cache.d)[int(cache.src_table[0, t // 16]) * 16 + t % 16] = t + 1
        cache.seen_tokens += input_ids.shape[1]
        h = torch.zeros(input_ids.shape[0], input_ids.shape[1], cfg.hidden_size)
        h[..., 0] = 1.0
        return h

    monkeypatch.setattr(LastKVModel, "forward", stand_in)
    prompt = torch.tensor([[1, 5, 17]])
    with torch.no_grad():
        out = model.generate(prompt, max_new_tokens=300, do_sample=False, use_cache=True)
    assert out.shape == (1, 303) and torch.equal(out[:, :3], prompt)
    assert calls[0][:3] == (3, calls[0][1], 0)
    assert all(n == 1 for n, *_ in calls[1:]) and len(calls) == 300
    assert len({c for _, c, _, _ in calls}) == 1  # the same cache object every step
    assert calls[-1][3] > calls[0][3]  # it grew
    final = calls[-1]
    assert final[2] == 301  # seen before the last call: 3 prompt + 298 generated tokens
    cache = caches[0]
    flat = cache.pool_k.view(-1, cache.hkv, cache.d)
    marks = [float(flat[int(cache.src_table[0, t // 16]) * 16 + t % 16, 0, 0]) for t in range(302)]
    assert marks == [t + 1.0 for t in range(302)]  # every forwarded token's slot survived the growth


def test_load_model_checks_the_backend_argument():
    from lastkv_b200.llm import load_model

    with pytest.raises(ValueError, match="attention_backend"):
        load_model("unused", attention_backend="flash")


def test_paged_cache_reserve_keeps_contents():
    from lastkv_b200 import _capi
    from lastkv_b200.hf import LastKVConfig, PagedLastKVCache

    _capi.load()
    cfg = LastKVConfig(hidden_size=64, intermediate_size=96, num_attention_heads=4, num_key_value_heads=2,
                       num_hidden_layers=3, head_dim=64, vocab_size=50, chunk_size=32)
    order = np.random.default_rng(0).permutation(2 * 4)
    cache = PagedLastKVCache(cfg, 2, 64, device="cpu", page_order=order, dtype=torch.float32)
    cache.pool_k.copy_(torch.randn_like(cache.pool_k))
    cache.pool_v.copy_(torch.randn_like(cache.pool_v))
    shared = [cache.pool_k[torch.from_numpy(cache.src_table[b].astype(np.int64))].clone() for b in range(2)]
    rings = [cache.pool_v[cache.ring_base[l]:cache.ring_base[l] + cache.ring_stride].clone() for l in range(3)]
    cache.reserve(200)
    assert cache.max_tokens == 200 and cache.pages_per_seq == 13
    for b in range(2):
        got = cache.pool_k[torch.from_numpy(cache.src_table[b, :4].astype(np.int64))]
        assert torch.equal(got, shared[b])
    for l in range(3):
        assert torch.equal(cache.pool_v[cache.ring_base[l]:cache.ring_base[l] + cache.ring_stride], rings[l])
    assert cache.num_pages == 2 * 13 + 3 * cache.ring_stride


def test_published_8b_parameter_layout_without_allocating_weights():
    """The reference's known answer for the published 8B layout
    (llm/tests/test_llm_inference.py:137-150): 419 tensors, 8,030,269,952
    parameters, the per-layer blend logits and value scales, built on the meta
    device so no weight is allocated."""
    from lastkv_b200.llm import CustomRecurrentMarinAKV254ReuseKVConfig as Config
    from lastkv_b200.llm import CustomRecurrentMarinAKV254ReuseKVForCausalLM as Model

    config = Config(hidden_size=4096, intermediate_size=14336, num_attention_heads=32, num_key_value_heads=8,
                    num_hidden_layers=32, head_dim=128, vocab_size=128256, rms_norm_eps=1e-5,
                    tie_word_embeddings=False)
    with torch.device("meta"):
        model = Model(config)
    state = model.state_dict()
    assert len(state) == 419
    assert sum(t.numel() for t in state.values()) == 8_030_269_952
    assert state["model.layers.31.self_attn.prev_chunk_alphas"].shape == (8,)
    assert state["model.layers.0.self_attn.deep_v_scale"].shape == (8,)
    assert state["model.layers.0.self_attn.q_norm.weight"].shape == (128,)
    assert state["lm_head.weight"].shape == (128256, 4096)
