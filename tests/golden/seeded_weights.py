"""Deterministic random weights by parameter name (shared by the golden
generator and the GPU tests, so large models need not be stored).

Linear / embedding weights ~ N(0, std) from a generator seeded by
(seed, crc32(name)); RMSNorm weights = 1; prev_chunk_alphas and
deep_v_scale follow ``alpha_fn`` / ``scale_fn`` (per layer index) when given,
else the reference's initial values (0 and 1).
"""

import re
import zlib

import numpy as np


def seeded_state(shapes: dict, seed: int, std: float = 0.02, alpha_fn=None, scale_fn=None) -> dict:
    out = {}
    for name in sorted(shapes):
        shape = tuple(shapes[name])
        m = re.search(r"layers\.(\d+)\.", name)
        layer = int(m.group(1)) if m else -1
        if name.endswith("prev_chunk_alphas"):
            out[name] = (alpha_fn(layer, shape) if alpha_fn else np.zeros(shape)).astype(np.float32)
        elif name.endswith("deep_v_scale"):
            out[name] = (scale_fn(layer, shape) if scale_fn else np.ones(shape)).astype(np.float32)
        elif "norm" in name:
            out[name] = np.ones(shape, np.float32)
        else:
            rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
            out[name] = (rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float32)
    return out


def nontrivial_alpha(layer, shape):
    return np.linspace(-1.2, 0.8, shape[0]) + 0.1 * layer


def nontrivial_scale(layer, shape):
    return np.linspace(0.6, 1.3, shape[0]) + 0.02 * layer


CONFIG1 = dict(hidden_size=768, intermediate_size=2048, num_attention_heads=12, num_key_value_heads=12,
               num_hidden_layers=12, head_dim=64, vocab_size=32000, rope_theta=1000000.0, rms_norm_eps=1e-6)
