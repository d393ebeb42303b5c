"""Wan paged layout on CPU: emulate the append and commit data movement of
``WanSharedKVCache`` with numpy (exactly the slots the kernels would read and
write) and check that every block's key list - read through its block table -
equals the oracle's composed history [prefix | shared | blended previous
block | current block], for segment boundaries that are not page-aligned."""

import numpy as np
import pytest
import torch

from oracle import lastkv_oracle as O


def _emulate(cache, alpha, blocks, rng):
    from lastkv_b200.contract import PAGE_SIZE

    H, D, L, BT = cache.H, cache.D, cache.L, cache.block
    pool_k = np.zeros((cache.num_pages * PAGE_SIZE, H, D))
    pool_v = np.zeros_like(pool_k)
    hist = O.WanHistory(L, cache.prefix, BT, alpha)
    for n in range(blocks):
        meta = cache.begin_block(n)
        bt = meta["bt"].numpy()
        kvs = []
        for layer in range(L):
            k = rng.standard_normal((BT, H, D))
            v = rng.standard_normal((BT, H, D))
            ring = meta["ring"][layer].numpy()
            pool_k[ring], pool_v[ring] = k, v  # the append kernel's stores (batch 1)
            if layer == L - 1:
                src = meta["src"].numpy()
                pool_k[src], pool_v[src] = k, v
            # keys this layer's attention reads through its block table
            pages = bt[layer, 0]
            rows = (pages[:, None] * PAGE_SIZE + np.arange(PAGE_SIZE)[None]).reshape(-1)[: (n + 1) * BT]
            h = hist.history(layer, n * BT)
            exp_k = k if h is None else np.concatenate([h[0], k])
            exp_v = v if h is None else np.concatenate([h[1], v])
            np.testing.assert_allclose(pool_k[rows], exp_k, rtol=1e-12, atol=1e-12)
            np.testing.assert_allclose(pool_v[rows], exp_v, rtol=1e-12, atol=1e-12)
            kvs.append((k, v))
        hist.commit(n * BT, kvs)
        # the commit kernel's data movement (gather/blend), emulated
        captured = {}

        def fake_gather_blend(pk, pv, dst, sa, sb, row, a, error_word=None):
            captured.update(dst=dst.numpy(), sa=sa.numpy(), sb=sb.numpy(), row=row.numpy())

        import lastkv_b200.wan as wan_mod

        orig = wan_mod.ops.gather_blend
        wan_mod.ops.gather_blend = fake_gather_blend
        try:
            cache.commit_block(torch.from_numpy(alpha.astype(np.float32)))
        finally:
            wan_mod.ops.gather_blend = orig
        if captured:
            d, sa, sb, row = captured["dst"], captured["sa"], captured["sb"], captured["row"]
            assert len(np.intersect1d(d, np.concatenate([sa[sa >= 0], sb[sb >= 0]]))) == 0
            a = alpha[row][:, :, None]
            for pool in (pool_k, pool_v):
                av = pool[np.maximum(sa, 0)]
                bv = pool[np.maximum(sb, 0)]
                out = np.where((sb < 0)[:, None, None], av, np.where((sa < 0)[:, None, None], bv, a * av + (1 - a) * bv))
                pool[d] = out


@pytest.mark.parametrize("fh,fw,fpb,prefix,shuffle", [(2, 4, 3, 8, False), (2, 4, 3, 8, True), (3, 5, 2, 15, True),
                                                       (1, 13, 3, 13, False)])
def test_block_key_lists_match_oracle_history(fh, fw, fpb, prefix, shuffle):
    from lastkv_b200.wan import WanSharedKVCache

    blocks = 6
    frames = blocks * fpb
    n_src = -(-fh * fw * frames // 16)
    order = np.random.default_rng(1).permutation(n_src) if shuffle else None
    cache = WanSharedKVCache(num_layers=3, batch=1, num_heads=2, head_dim=64, frame_h=fh, frame_w=fw,
                             frames_per_block=fpb, max_frames=frames, prefix_tokens=prefix, device="cpu",
                             page_order=order)
    rng = np.random.default_rng(fh * 100 + fw)
    alpha = rng.uniform(0.1, 0.9, (3, 2))
    _emulate(cache, alpha, blocks, rng)


def test_rope_table_matches_oracle_angles():
    from lastkv_b200.wan import wan_rope_table

    t = wan_rope_table(3, 30, 52, 6, 128)
    ang = O.wan_rope_angles(3, 30, 52, 6, 128)
    np.testing.assert_allclose(t[:, :64], np.cos(ang), rtol=0, atol=1e-7)
    np.testing.assert_allclose(t[:, 64:], np.sin(ang), rtol=0, atol=1e-7)


def test_prefix_must_fit_the_first_block():
    from lastkv_b200.contract import RMarinBackendContractError
    from lastkv_b200.wan import WanSharedKVCache

    with pytest.raises(RMarinBackendContractError):
        WanSharedKVCache(num_layers=1, batch=1, num_heads=1, head_dim=64, frame_h=1, frame_w=20, frames_per_block=1,
                         max_frames=4, prefix_tokens=20, device="cpu")
