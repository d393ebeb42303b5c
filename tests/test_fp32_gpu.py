"""The fp32 kernels (the reference's fp32 configuration) vs the CPU oracle.

* ``lkv_attention_paged_f32``: decode and bottom-right causal spans over fp32
  pools with shuffled pages, ragged lengths and GQA, against the float64
  oracle: max-abs <= 2e-5 and relative L2 <= 1e-5 (fp32 accumulation);
* ``lkv_rope_norm_append`` with ``LKV_APPEND_FP32``: the fp32 HF RoPE ->
  RMSNorm -> V/s -> paged stores, within 4 fp32 ulp (the sum of squares is
  accumulated in another order);
* ``lkv_blend_chunk_f32``: bit-exact against the fp32 numpy restatement.
"""

import numpy as np
import pytest
import torch

from oracle import lastkv_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, REL = 2e-5, 1e-5


def _case(seed, B, Hq, Hkv, D, lens, spans):
    rng = np.random.default_rng(seed)
    pages_per = [-(-n // 16) for n in lens]
    W = max(1, max(pages_per))
    total = sum(pages_per) + 5
    perm = rng.permutation(total)
    bt = np.zeros((B, W), np.int32)
    o = 0
    for b in range(B):
        bt[b, :pages_per[b]] = perm[o:o + pages_per[b]]
        o += pages_per[b]
    pk = rng.standard_normal((total, 16, Hkv, D)).astype(np.float32)
    pv = rng.standard_normal((total, 16, Hkv, D)).astype(np.float32)
    cu = np.concatenate([[0], np.cumsum(spans)]).astype(np.int32)
    q = rng.standard_normal((int(cu[-1]), Hq, D)).astype(np.float32)
    return q, pk, pv, bt, np.asarray(lens, np.int32), cu


CASES = [
    # seed, B, Hq, Hkv, D, lens, spans
    (0, 1, 12, 12, 64, [1], [1]),
    (1, 3, 12, 12, 64, [640, 17, 300], [1, 1, 1]),              # decode, config-1 heads
    (2, 2, 12, 12, 64, [512, 640], [512, 128]),                 # prefill spans (causal, bottom-right)
    (3, 4, 32, 8, 128, [1000, 33, 16, 4000], [7, 33, 1, 250]),  # GQA 4, D 128, ragged
    (4, 2, 8, 1, 64, [0, 70], [1, 70]),                         # a sequence with no keys
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"B{c[1]}_Hq{c[2]}_Hkv{c[3]}_D{c[4]}_{c[0]}")
def test_attention_f32_matches_oracle(case):
    from lastkv_b200 import _capi, ops

    _capi.load()
    seed, B, Hq, Hkv, D, lens, spans = case
    q, pk, pv, bt, sk, cu = _case(seed, B, Hq, Hkv, D, lens, spans)
    scale_h = np.random.default_rng(seed + 9).uniform(0.5, 1.5, Hq).astype(np.float32)
    dev = "cuda"
    err = torch.zeros(4, dtype=torch.int32, device=dev)
    lse = torch.empty((q.shape[0], Hq), dtype=torch.float32, device=dev)
    out = ops.attention_paged_f32(torch.from_numpy(q).to(dev), torch.from_numpy(pk).to(dev),
                                  torch.from_numpy(pv).to(dev), torch.from_numpy(bt).to(dev),
                                  torch.from_numpy(sk).to(dev), torch.from_numpy(cu).to(dev), lse=lse,
                                  out_scale=torch.from_numpy(scale_h).to(dev), error_word=err)
    torch.cuda.synchronize()
    assert err.cpu().tolist() == [0, 0, 0, 0]
    want, want_lse = O.paged_attention(q, pk, pv, bt, sk, cu, scale=D ** -0.5, out_scale=scale_h)
    got = out.cpu().numpy().astype(np.float64)
    max_abs = np.abs(got - want).max()
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    assert max_abs <= MAX_ABS and rel <= REL, (max_abs, rel)
    finite = np.isfinite(want_lse)
    np.testing.assert_allclose(lse.cpu().numpy()[finite], want_lse[finite], rtol=1e-5, atol=1e-5)
    assert np.all(np.isneginf(lse.cpu().numpy()[~finite]))


def test_append_f32_matches_the_fp32_hf_form():
    from lastkv_b200 import _capi, ops

    _capi.load()
    rng = np.random.default_rng(21)
    T, Hq, Hkv, D, slots = 37, 16, 4, 64, 300
    q = rng.standard_normal((T, Hq * D)).astype(np.float32)
    k = rng.standard_normal((T, Hkv * D)).astype(np.float32)
    v = rng.standard_normal((T, Hkv * D)).astype(np.float32)
    pos = rng.integers(0, 4096, T).astype(np.int64)
    inv_freq = 1.0 / (1e6 ** (np.arange(0, D, 2) / D))
    ang = (np.arange(4096)[:, None] * inv_freq[None].astype(np.float32)).astype(np.float32)
    cs = np.concatenate([np.cos(ang), np.sin(ang)], -1).astype(np.float32)
    qw = rng.uniform(0.5, 1.5, D).astype(np.float32)
    kw = rng.uniform(0.5, 1.5, D).astype(np.float32)
    s = rng.uniform(0.5, 2.0, Hkv).astype(np.float32)
    inv = (np.float32(1.0) / s).astype(np.float32)
    ring_slot = rng.permutation(slots)[:T].astype(np.int64)
    src_slot = rng.permutation(slots)[:T].astype(np.int64)
    dev = "cuda"
    t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    ring_k = torch.zeros((slots, Hkv, D), device=dev)
    ring_v = torch.zeros((slots, Hkv, D), device=dev)
    src_k = torch.zeros((slots, Hkv, D), device=dev)
    src_v = torch.zeros((slots, Hkv, D), device=dev)
    err = torch.zeros(4, dtype=torch.int32, device=dev)
    q_out = ops.rope_norm_append(t(q), t(k), t(v), t(pos), t(cs), t(qw), t(kw), 1e-6, t(inv), t(ring_slot),
                                 ring_k, ring_v, t(src_slot), src_k, src_v, error_word=err)
    torch.cuda.synchronize()
    assert q_out.dtype == torch.float32 and err.cpu().tolist() == [0, 0, 0, 0]
    c, sn = cs[pos][:, None, : D // 2], cs[pos][:, None, D // 2:]
    want_q = O.rms_norm_hf_f32(O.rope_hf_f32(q.reshape(T, Hq, D), c, sn), qw, 1e-6)
    want_k = O.rms_norm_hf_f32(O.rope_hf_f32(k.reshape(T, Hkv, D), c, sn), kw, 1e-6)
    want_v = (v.reshape(T, Hkv, D) * inv[None, :, None]).astype(np.float32)

    def ulps(a, b):
        # in units of the fp32 spacing at |b| (at least at 1e-2, so values near zero count absolutely)
        unit = np.spacing(np.maximum(np.abs(b), np.float32(1e-2)).astype(np.float32)).astype(np.float64)
        return np.abs(a.astype(np.float64) - b) / unit

    assert ulps(q_out.cpu().numpy(), want_q).max() <= 4
    assert ulps(ring_k.cpu().numpy()[ring_slot], want_k).max() <= 4
    assert np.array_equal(ring_v.cpu().numpy()[ring_slot], want_v)  # one rounded product: exact
    assert ulps(src_k.cpu().numpy()[src_slot], want_k).max() <= 4
    assert np.array_equal(src_v.cpu().numpy()[src_slot], v.reshape(T, Hkv, D))


def test_blend_f32_bit_exact():
    from lastkv_b200 import _capi, ops

    _capi.load()
    rng = np.random.default_rng(5)
    L, S, ppc, Hkv, D = 3, 2, 4, 4, 64
    pages = S * ppc + L * (S * ppc + 1)
    pk = rng.standard_normal((pages, 16, Hkv, D)).astype(np.float32)
    pv = rng.standard_normal((pages, 16, Hkv, D)).astype(np.float32)
    raw = rng.permutation(S * ppc).reshape(S, ppc).astype(np.int32)
    ring_stride = S * ppc + 1
    ring = (S * ppc + rng.permutation(S * ppc).reshape(S, ppc)).astype(np.int32)
    alpha = (1.0 / (1.0 + np.exp(-rng.standard_normal((L, Hkv))))).astype(np.float32)
    dev = "cuda"
    gk, gv = torch.from_numpy(pk).to(dev), torch.from_numpy(pv).to(dev)
    err = torch.zeros(4, dtype=torch.int32, device=dev)
    ops.blend_chunk(gk, gv, torch.from_numpy(raw).to(dev), torch.from_numpy(ring).to(dev), ring_stride,
                    torch.from_numpy(alpha).to(dev), error_word=err)
    torch.cuda.synchronize()
    assert err.cpu().tolist() == [0, 0, 0, 0]
    for pool, got in ((pk, gk.cpu().numpy()), (pv, gv.cpu().numpy())):
        for s in range(S):
            rp = np.stack([ring[s] + l * ring_stride for l in range(L)])  # [L, ppc]
            want = O.blend_chunk_f32(pool[rp].reshape(L, -1, Hkv, D), pool[raw[s]].reshape(-1, Hkv, D), alpha)
            assert np.array_equal(got[rp], want.reshape(L, ppc, 16, Hkv, D))
