"""Pin the oracle's Wan restatement against the reference's recorded block attention.

The golden file holds, for six 3-frame blocks x three layers of a tiny
reference Wan model, the normalised pre-RoPE q/k, v, the RoPE'd query and the
output of the reference's attention call (videogen/src/lastkv/videogen/
model.py:372-390).  Segment boundaries (8-token frames, 24-token blocks,
8-token prefix) are deliberately not multiples of the 16-token page.
"""

import numpy as np

from oracle import lastkv_oracle as O
from tests.conftest import load_golden


def _calls(data):
    for i in range(int(data["calln"])):
        p = f"call{i}_"
        layer, start, bt, key_len = (int(x) for x in data[p + "meta"])
        yield dict(layer=layer, start=start, block=bt, key_len=key_len,
                   **{k: data[p + k][0] for k in ("qn", "kn", "v", "roped_q", "out")})


def test_wan_rope_and_history_reproduce_reference():
    data = load_golden("wan_block_attn.npz")
    H, D = int(data["num_heads"]), int(data["head_dim"])
    fh, fw, fpb = int(data["frame_h"]), int(data["frame_w"]), int(data["frames_per_block"])
    alpha = 1.0 / (1.0 + np.exp(-data["prev_block_alphas"].astype(np.float64)))
    hist = O.WanHistory(int(data["num_layers"]), int(data["prefix_tokens"]), fh * fw * fpb, alpha)
    kvs = []
    n = 0
    for c in _calls(data):
        T = c["qn"].shape[0]
        ang = O.wan_rope_angles(fpb, fh, fw, c["start"] // (fh * fw), D)
        q = O.rope_interleaved(c["qn"].reshape(T, H, D), ang)
        k = O.rope_interleaved(c["kn"].reshape(T, H, D), ang)
        v = c["v"].reshape(T, H, D).astype(np.float64)
        np.testing.assert_allclose(q, c["roped_q"], rtol=1e-5, atol=1e-5)
        h = hist.history(c["layer"], c["start"])
        fk = k if h is None else np.concatenate([h[0], k])
        fv = v if h is None else np.concatenate([h[1], v])
        assert fk.shape[0] == c["key_len"]
        out, _ = O.attention(q, fk, fv, scale=D ** -0.5, causal=False)
        np.testing.assert_allclose(out, c["out"], rtol=1e-4, atol=2e-5)
        kvs.append((k, v))
        if c["layer"] == int(data["num_layers"]) - 1:
            hist.commit(c["start"], kvs)
            kvs = []
        n += 1
    assert n == 18
