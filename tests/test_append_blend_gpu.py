"""Fused RoPE/RMSNorm/append, chunk blend and block-table kernels vs the oracle."""

import numpy as np
import pytest
import torch

from oracle import lastkv_oracle as O

pytestmark = pytest.mark.gpu


def _cu(x, dt=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().to(dt)


def _ulp_diff(a, b):
    ia = O.bf16_bits(a).astype(np.int32)
    ib = O.bf16_bits(b).astype(np.int32)
    # map sign-magnitude to a monotone integer line
    ia = np.where(ia & 0x8000, -(ia & 0x7FFF), ia)
    ib = np.where(ib & 0x8000, -(ib & 0x7FFF), ib)
    return np.abs(ia - ib)


def _append_case(seed, T, Hq, Hkv, D, top, slots_total=200):
    rng = np.random.default_rng(seed)
    maxpos = 4096
    cs = O.bf16_round(O.rope_cos_sin(maxpos, D, 500000.0))
    q = O.bf16_round(rng.standard_normal((T, Hq * D)) * 3)
    k = O.bf16_round(rng.standard_normal((T, Hkv * D)) * 3)
    v = O.bf16_round(rng.standard_normal((T, Hkv * D)))
    qw = O.bf16_round(rng.uniform(0.5, 1.5, D))
    kw = O.bf16_round(rng.uniform(0.5, 1.5, D))
    s = O.bf16_round(rng.uniform(0.3, 1.7, Hkv))
    inv = (1.0 / s.astype(np.float32)).astype(np.float32)
    pos = rng.integers(0, maxpos, T)
    ring_slot = rng.permutation(slots_total)[:T]
    src_slot = rng.permutation(slots_total)[:T] if top else None
    return dict(cs=cs, q=q, k=k, v=v, qw=qw, kw=kw, inv=inv, pos=pos, ring_slot=ring_slot, src_slot=src_slot,
                n=slots_total, Hkv=Hkv, D=D)


@pytest.mark.parametrize("T,Hq,Hkv,D,top", [(1, 32, 8, 128, False), (37, 32, 8, 128, True), (5, 12, 12, 64, True),
                                            (64, 8, 1, 128, False)])
def test_rope_norm_append_matches_oracle(T, Hq, Hkv, D, top):
    from lastkv_b200 import ops

    c = _append_case(T * 7 + D, T, Hq, Hkv, D, top)
    rk = torch.zeros((c["n"], Hkv, D), dtype=torch.bfloat16, device="cuda")
    rv, sk, sv = torch.zeros_like(rk), torch.zeros_like(rk), torch.zeros_like(rk)
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    q_out = ops.rope_norm_append(_cu(c["q"]), _cu(c["k"]), _cu(c["v"]), torch.from_numpy(c["pos"]).cuda(),
                                 _cu(c["cs"]), _cu(c["qw"]), _cu(c["kw"]), 1e-5, _cu(c["inv"], torch.float32),
                                 torch.from_numpy(c["ring_slot"]).cuda(), rk, rv,
                                 torch.from_numpy(c["src_slot"]).cuda() if top else None, sk if top else None,
                                 sv if top else None, error_word=err)
    nrk = np.zeros((c["n"], Hkv, D), np.float32)
    nrv, nsk, nsv = np.zeros_like(nrk), np.zeros_like(nrk), np.zeros_like(nrk)
    q_ref = O.rope_norm_append(c["q"], c["k"], c["v"], c["pos"], c["cs"], c["qw"], c["kw"], 1e-5, c["inv"],
                               c["ring_slot"], nrk, nrv, c["src_slot"], nsk if top else None, nsv if top else None)
    pairs = [("q", q_out, q_ref), ("ring_k", rk, nrk), ("ring_v", rv, nrv)]
    if top:
        pairs += [("src_k", sk, nsk), ("src_v", sv, nsv)]
    for name, got, ref in pairs:
        g = got.float().cpu().numpy()
        ulps = _ulp_diff(g, ref)
        # fp32 reassociation of the sum of squares and rsqrt may flip the last
        # bf16 bit of a few elements; nothing may differ by more than one ulp.
        assert ulps.max() <= 1, (name, int(ulps.max()))
        assert (ulps > 0).mean() <= 0.02, (name, float((ulps > 0).mean()))
    assert err.cpu().tolist()[0] == 0


def test_append_rejects_out_of_range_slot_without_fault():
    from lastkv_b200 import ops

    c = _append_case(3, 4, 8, 2, 128, False, slots_total=16)
    ring_slot = c["ring_slot"].copy()
    ring_slot[2] = 10_000  # beyond the 16-slot ring
    rk = torch.zeros((16, 2, 128), dtype=torch.bfloat16, device="cuda")
    rv = torch.zeros_like(rk)
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    ops.rope_norm_append(_cu(c["q"]), _cu(c["k"]), _cu(c["v"]), torch.from_numpy(c["pos"]).cuda(), _cu(c["cs"]),
                         _cu(c["qw"]), _cu(c["kw"]), 1e-5, _cu(c["inv"], torch.float32),
                         torch.from_numpy(ring_slot).cuda(), rk, rv, error_word=err)
    e = err.cpu().tolist()
    assert e[0] == 3 and e[1] == 2 and e[3] == 10_000
    nrk = np.zeros((16, 2, 128), np.float32)
    nrv = np.zeros_like(nrk)
    ok = [0, 1, 3]
    O.rope_norm_append(c["q"][ok], c["k"][ok], c["v"][ok], c["pos"][ok], c["cs"], c["qw"], c["kw"], 1e-5, c["inv"],
                       ring_slot[ok], nrk, nrv)
    assert _ulp_diff(rk.float().cpu().numpy(), nrk).max() <= 1


@pytest.mark.parametrize("L,S,ppc,Hkv,D", [(3, 2, 4, 8, 128), (32, 1, 64, 8, 128), (2, 3, 1, 12, 64),
                                           (2, 2, 2, 5, 128), (3, 1, 3, 3, 64)])
def test_blend_chunk_bit_exact(L, S, ppc, Hkv, D):
    from lastkv_b200 import ops

    rng = np.random.default_rng(L * 100 + S)
    ring_stride = S * ppc * 2 + 1
    src = S * ppc * 3
    total = src + L * ring_stride
    pk = O.bf16_round(rng.standard_normal((total, 16, Hkv, D)))
    pv = O.bf16_round(rng.standard_normal((total, 16, Hkv, D)))
    raw_pages = rng.permutation(src)[: S * ppc].reshape(S, ppc).astype(np.int32)
    ring_pages = (src + np.arange(S)[:, None] * ppc * 2 + np.arange(ppc)[None, :]).astype(np.int32)
    alpha = O.alpha_from_logits(rng.standard_normal((L, Hkv)))
    tk, tv = _cu(pk), _cu(pv)
    ops.blend_chunk(tk, tv, torch.from_numpy(raw_pages).cuda(), torch.from_numpy(ring_pages).cuda(), ring_stride,
                    _cu(alpha, torch.float32))
    ek, ev = pk.copy(), pv.copy()
    for s in range(S):
        for l in range(L):
            rows = ring_pages[s] + l * ring_stride
            for pool, exp in ((pk, ek), (pv, ev)):
                ring = pool[rows].reshape(1, ppc * 16, Hkv, D)
                raw = pool[raw_pages[s]].reshape(ppc * 16, Hkv, D)
                exp[rows] = O.blend_chunk(ring, raw, alpha[l:l + 1])[0].reshape(ppc, 16, Hkv, D)
    np.testing.assert_array_equal(tk.float().cpu().numpy(), ek)
    np.testing.assert_array_equal(tv.float().cpu().numpy(), ev)


def test_build_layer_block_tables():
    from lastkv_b200 import ops

    rng = np.random.default_rng(0)
    L, B, W = 5, 7, 40
    bt = rng.integers(0, 1000, (B, W)).astype(np.int32)
    nsrc = rng.integers(0, W, B).astype(np.int32)
    base = (5000 + np.arange(L) * 321).astype(np.int32)
    out = ops.build_layer_block_tables(torch.from_numpy(bt).cuda(), torch.from_numpy(nsrc).cuda(),
                                       torch.from_numpy(base).cuda())
    col = np.arange(W)[None, None, :]
    exp = np.where(col < nsrc[None, :, None], bt[None], bt[None] + base[:, None, None])
    np.testing.assert_array_equal(out.cpu().numpy(), exp)
