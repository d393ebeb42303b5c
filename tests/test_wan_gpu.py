"""Wan block attention on the B200 kernels vs the reference's recorded calls
(interleaved 3-D RoPE from an fp32 table, paged prefix/shared/window history,
non-causal tcgen05 prefill, token-level commit)."""

import numpy as np
import pytest
import torch

from tests.gpu_helpers import assert_close_bf16
from tests.test_oracle_wan_golden import _calls
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shuffle", [False, True])
def test_wan_block_attention_matches_reference(shuffle):
    from lastkv_b200.wan import WanSharedKVCache, wan_block_attention

    data = load_golden("wan_block_attn.npz")
    H, D, L = int(data["num_heads"]), int(data["head_dim"]), int(data["num_layers"])
    fh, fw, fpb = int(data["frame_h"]), int(data["frame_w"]), int(data["frames_per_block"])
    blocks = 6
    n_src = -(-fh * fw * fpb * blocks // 16)
    order = np.random.default_rng(4).permutation(n_src) if shuffle else None
    cache = WanSharedKVCache(num_layers=L, batch=1, num_heads=H, head_dim=D, frame_h=fh, frame_w=fw,
                             frames_per_block=fpb, max_frames=fpb * blocks, prefix_tokens=int(data["prefix_tokens"]),
                             device="cuda", page_order=order)
    alpha = torch.sigmoid(torch.from_numpy(data["prev_block_alphas"])).float().cuda()
    checked = 0
    for c in _calls(data):
        n, layer = c["start"] // cache.block, c["layer"]
        if layer == 0:
            cache.begin_block(n)
        to = lambda x: torch.from_numpy(x).cuda().to(torch.bfloat16).unsqueeze(0)
        out = wan_block_attention(to(c["qn"]), to(c["kn"]), to(c["v"]), cache, layer)
        assert_close_bf16(out[0].float().cpu().numpy(), c["out"], what=f"block {n} layer {layer}")
        checked += 1
        if layer == L - 1:
            cache.commit_block(alpha)
    cache.check_errors()
    assert checked == 18
