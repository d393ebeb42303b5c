"""Shared helpers of the GPU parity tests (seeded inputs, tolerance checks)."""

import numpy as np
import torch

from oracle import lastkv_oracle as O

# bf16 tolerance against the float64 oracle on identical bf16 inputs, stated
# for attention outputs of O(1) magnitude: max-abs <= 2e-2, relative L2 <= 1e-2.
MAX_ABS = 2e-2
REL_L2 = 1e-2


def assert_close_bf16(actual, expected, max_abs=MAX_ABS, rel_l2=REL_L2, what=""):
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    assert np.isfinite(a).all(), f"{what}: non-finite output"
    err = np.abs(a - e).max() if a.size else 0.0
    rel = np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-12) if a.size else 0.0
    assert err <= max_abs and rel <= rel_l2, f"{what}: max_abs={err:.3e} rel_l2={rel:.3e}"
    return err, rel


def make_paged_case(seed, B, Hq, Hkv, D, lens, *, extra_pages=7, shuffle=True, device="cuda"):
    """Seeded bf16 pool with each sequence's pages scattered by a permutation."""
    rng = np.random.default_rng(seed)
    pages_per = [-(-n // 16) for n in lens]
    W = max(1, max(pages_per))
    total = sum(pages_per) + extra_pages
    perm = rng.permutation(total) if shuffle else np.arange(total)
    bt = np.zeros((B, W), dtype=np.int32)
    o = 0
    for b in range(B):
        bt[b, :pages_per[b]] = perm[o:o + pages_per[b]]
        o += pages_per[b]
    pk = O.bf16_round(rng.standard_normal((total, 16, Hkv, D)).astype(np.float32))
    pv = O.bf16_round(rng.standard_normal((total, 16, Hkv, D)).astype(np.float32))
    q = O.bf16_round(rng.standard_normal((B, Hq, D)).astype(np.float32))
    t = dict(
        q=torch.from_numpy(q).to(device=device, dtype=torch.bfloat16),
        pool_k=torch.from_numpy(pk).to(device=device, dtype=torch.bfloat16),
        pool_v=torch.from_numpy(pv).to(device=device, dtype=torch.bfloat16),
        bt=torch.from_numpy(bt).to(device),
        seq_k=torch.tensor(lens, dtype=torch.int32, device=device),
    )
    n = dict(q=q, pool_k=pk, pool_v=pv, bt=bt, seq_k=np.array(lens), cu=np.arange(B + 1))
    return t, n
