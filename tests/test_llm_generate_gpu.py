"""``generate()`` through the reference's class names on the B200 kernels.

``CustomRecurrentMarinAKV254ReuseKVForCausalLM.generate(ids, max_new_tokens=N,
do_sample=False, use_cache=True)`` - the reference's own call
(llm/tests/test_llm_inference.py:125-134, and the config-1 recording) - in
fp32 must reproduce the reference's greedy tokens exactly:

* config 1 (124M architecture, 512-token prompt, 128 new tokens) at chunk 4096
  and at chunk 128 with non-trivial blend weights and value scales;
* the D=128 GQA model of ``small_d128.npz`` (chunk 16: every boundary path),
  whose recorded continuation must also equal a full-prefix replay with
  ``use_cache=False`` at every step, as the reference's test asserts.
"""

import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))


@pytest.fixture(autouse=True)
def _fp32_gemms():
    torch.backends.cuda.matmul.allow_tf32 = False


@pytest.mark.parametrize("tag,chunk,nontrivial", [("c4096", 4096, False), ("c128", 128, True)])
def test_config1_generate_equals_reference(tag, chunk, nontrivial):
    from seeded_weights import CONFIG1, nontrivial_alpha, nontrivial_scale, seeded_state

    from lastkv_b200.llm import CustomRecurrentMarinAKV254ReuseKVConfig, CustomRecurrentMarinAKV254ReuseKVForCausalLM
    from tests.conftest import load_golden

    golden = load_golden("config1_124m.npz")
    cfg = CustomRecurrentMarinAKV254ReuseKVConfig(**CONFIG1, chunk_size=chunk, max_position_embeddings=4096,
                                                  bos_token_id=1, eos_token_id=None, pad_token_id=0)
    model = CustomRecurrentMarinAKV254ReuseKVForCausalLM(cfg)
    state = seeded_state({k: tuple(v.shape) for k, v in model.state_dict().items()}, seed=1,
                         alpha_fn=nontrivial_alpha if nontrivial else None,
                         scale_fn=nontrivial_scale if nontrivial else None)
    model.load_state_dict({k: torch.from_numpy(v) for k, v in state.items()}, strict=True)
    model.model._alpha = None
    model = model.cuda().eval()
    prompt = torch.from_numpy(golden["prompt"]).cuda()
    with torch.inference_mode():
        out = model.generate(prompt, max_new_tokens=128, do_sample=False, use_cache=True)
    assert np.array_equal(out.cpu().numpy(), golden[f"{tag}_tokens"])


def test_small_d128_generate_equals_reference_and_replay(small_d128):
    from lastkv_b200.llm import CustomRecurrentMarinAKV254ReuseKVConfig, CustomRecurrentMarinAKV254ReuseKVForCausalLM

    d = small_d128
    cfg = CustomRecurrentMarinAKV254ReuseKVConfig(
        hidden_size=int(d["hidden_size"]), intermediate_size=int(d["intermediate_size"]),
        num_attention_heads=int(d["num_heads"]), num_key_value_heads=int(d["num_kv_heads"]),
        num_hidden_layers=int(d["num_layers"]), head_dim=int(d["head_dim"]), vocab_size=int(d["vocab_size"]),
        chunk_size=int(d["chunk"]), rms_norm_eps=float(d["eps"]), rope_theta=float(d["rope_theta"]),
        deep_v_scale_init=d["v_scale"].tolist(), bos_token_id=1, eos_token_id=None, pad_token_id=0)
    model = CustomRecurrentMarinAKV254ReuseKVForCausalLM(cfg)
    model.load_state_dict({k[2:]: torch.from_numpy(v) for k, v in d.items() if k.startswith("w_")}, strict=True)
    model.model._alpha = None
    model = model.cuda().eval()
    prompt = torch.from_numpy(d["generate_prompt"]).cuda()
    ref = d["generate_out"]
    n_new = ref.shape[1] - prompt.shape[1]
    with torch.inference_mode():
        out = model.generate(prompt, max_new_tokens=n_new, do_sample=False, use_cache=True)
        replay = prompt.clone()
        for _ in range(n_new):  # full-prefix replay without a cache, as the reference's test
            logits = model(replay, use_cache=False).logits
            replay = torch.cat((replay, logits[:, -1].argmax(-1, keepdim=True)), dim=1)
    assert np.array_equal(out.cpu().numpy(), ref)
    assert torch.equal(out, replay)
