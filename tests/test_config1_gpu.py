"""Config 1 (the reference's 124M architecture) end to end on the B200 path.

The reference (fp32, CPU) generated 128 greedy tokens after a 512-token seeded
prompt, with chunk 4096 (faithful: no boundary is reached) and with chunk 128
plus non-trivial blend weights and value scales (the shared history, blended
recent chunk and rings are all exercised); its teacher-forced top-8 logits of
every generated position are recorded too.  The weights are regenerated here
from the same per-name seeds.

fp32 (the reference's own arithmetic): the model runs fp32 end to end - fp32
projections, the fp32 append / attention / blend kernels over an fp32 paged
cache - and a free-running greedy generation must reproduce all 128 reference
tokens (llm/tests/test_llm_inference.py:125-134 asserts generate == full-prefix
replay token for token).  Its teacher-forced logits must match the reference's
within max-abs 1e-3 and relative 1e-4 (fp32 GEMMs and reductions on another
device sum in another order).

bf16: the same model in bf16 on the tensor-core kernels; teacher-forced on the
reference's tokens, every step picks the reference's token unless the
reference's top-2 margin is within twice the bf16 logit error (a near-tie).
"""

import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))

CASES = [("c4096", 4096, False), ("c128", 128, True)]
LOGIT_MAX_ABS, LOGIT_REL = 1e-3, 1e-4


@pytest.fixture(scope="module")
def config1():
    from tests.conftest import load_golden

    return load_golden("config1_124m.npz")


def _model(chunk, nontrivial, dtype):
    from seeded_weights import CONFIG1, nontrivial_alpha, nontrivial_scale, seeded_state

    from lastkv_b200.hf import LastKVConfig, LastKVForCausalLM

    cfg = LastKVConfig(**CONFIG1, chunk_size=chunk, max_position_embeddings=4096)
    with torch.device("meta"):
        shapes = {k: tuple(v.shape) for k, v in LastKVForCausalLM(cfg).state_dict().items()}
    state = seeded_state(shapes, seed=1, alpha_fn=nontrivial_alpha if nontrivial else None,
                         scale_fn=nontrivial_scale if nontrivial else None)
    model = LastKVForCausalLM(cfg)
    model.load_reference_state_dict({k: torch.from_numpy(v) for k, v in state.items()})
    return model.cuda().to(dtype).eval()


def _teacher_forced(model, ref):
    with torch.no_grad():
        cache = model.new_cache(1, ref.shape[1])
        logits, _ = model(torch.from_numpy(ref[:, :-1]).cuda(), cache)
        cache.check_errors()
    return logits[0, 511:].float().cpu().numpy()  # [128, vocab]


@pytest.mark.parametrize("tag,chunk,nontrivial", CASES, ids=[c[0] for c in CASES])
def test_config1_fp32_free_running_greedy_tokens_identical(config1, tag, chunk, nontrivial):
    torch.backends.cuda.matmul.allow_tf32 = False  # fp32 GEMMs stay fp32 (torch's default)
    model = _model(chunk, nontrivial, torch.float32)
    ref = config1[f"{tag}_tokens"]
    prompt = torch.from_numpy(config1["prompt"]).cuda()
    cache = model.new_cache(1, ref.shape[1])
    assert cache.pool_k.dtype == torch.float32
    gen = model.generate_greedy(prompt, 128, cache=cache).cpu().numpy()
    cache.check_errors()
    same = int((gen[0, 512:] == ref[0, 512:]).sum())
    first_diff = next((i for i in range(128) if gen[0, 512 + i] != ref[0, 512 + i]), None)
    got = _teacher_forced(model, ref)
    top_v, top_i = config1[f"{tag}_top_v"], config1[f"{tag}_top_i"]
    ours = np.take_along_axis(got, top_i, axis=1)
    max_abs = float(np.abs(ours - top_v).max())
    rel = float(np.linalg.norm(ours - top_v) / np.linalg.norm(top_v))
    print(f"config1 {tag} fp32: free-running {same}/128 identical greedy tokens; teacher-forced logits "
          f"max-abs {max_abs:.3e}, relative {rel:.3e}")
    assert first_diff is None, f"first differing token at step {first_diff}"
    assert (gen == ref).all()
    assert max_abs <= LOGIT_MAX_ABS and rel <= LOGIT_REL, (max_abs, rel)


@pytest.mark.parametrize("tag,chunk,nontrivial", CASES, ids=[c[0] for c in CASES])
def test_config1_bf16_teacher_forced_tokens(config1, tag, chunk, nontrivial):
    model = _model(chunk, nontrivial, torch.bfloat16)
    ref = config1[f"{tag}_tokens"]
    got = _teacher_forced(model, ref)
    top_v, top_i = config1[f"{tag}_top_v"], config1[f"{tag}_top_i"]
    n = got.shape[0]
    err = np.abs(np.take_along_axis(got, top_i, axis=1) - top_v).max(1)
    margin = top_v[:, 0] - top_v[:, 1]
    picks = got.argmax(1)
    ties = 0
    for i in range(n):
        if picks[i] != ref[0, 512 + i]:
            assert margin[i] <= 2 * err[i], f"step {i}: margin {margin[i]:.4f} > 2 x error {err[i]:.4f}"
            ties += 1
    print(f"config1 {tag} bf16: teacher-forced {n - ties}/{n} identical greedy tokens, {ties} near-ties, "
          f"median logit err {np.median(err):.3e}")
