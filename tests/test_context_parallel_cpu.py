"""Context-parallel decode host logic on CPU: two gloo ranks, each with its slice
of the shared history (the last rank also holds the ring window), must merge
to exactly the single-rank attention.  The partial-attention and merge steps
are injected as oracle functions (no GPU)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import lastkv_oracle as O


def test_shard_ranges_cover_everything():
    from lastkv_b200.context_parallel import plan_shard, shard_range

    for n, w in [(10, 3), (8192, 8), (1, 2), (0, 4), (7, 7)]:
        ranges = [shard_range(n, w, r) for r in range(w)]
        assert ranges[0][0] == 0 and ranges[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        assert max(b - a for a, b in ranges) - min(b - a for a, b in ranges) <= 1
    plans = [plan_shard(8192 // 16, 2048, 16, 4, r) for r in range(4)]
    assert sum(p.seq_k for p in plans) == 8192 + 2048
    assert [p.ring_pages for p in plans] == [0, 0, 0, 128]
    # pages per rank (shared + ring) are balanced: the ring counts against the last rank
    assert [p.p1 - p.p0 + p.ring_pages for p in plans] == [160, 160, 160, 160]
    for nsrc, window, world in [(8064, 2048, 2), (8064, 2048, 8), (3, 2048, 4), (100, 17, 3), (5, 1, 1)]:
        plans = [plan_shard(nsrc, window, 16, world, r) for r in range(world)]
        assert plans[0].p0 == 0 and plans[-1].p1 == nsrc
        assert all(a.p1 == b.p0 for a, b in zip(plans, plans[1:]))
        assert sum(p.seq_k for p in plans) == nsrc * 16 + window
    assert [plan_shard(8064, 2048, 16, 2, r).p1 - plan_shard(8064, 2048, 16, 2, r).p0 for r in range(2)] == [4096, 3968]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _fake_partial(q, pool_k, pool_v, block_table, seq_k, workspace, max_pages):
    o, l = O.paged_attention(q.numpy(), pool_k.numpy(), pool_v.numpy(), block_table.numpy(), seq_k.numpy(),
                             np.arange(q.shape[0] + 1), scale=q.shape[-1] ** -0.5)
    return torch.from_numpy(o.astype(np.float32)), torch.from_numpy(l.astype(np.float32))


def _fake_merge(o_all, lse_all, out_scale, out):
    o, _ = O.merge_many(list(o_all.numpy()), list(lse_all.numpy()))
    if out_scale is not None:
        o = o * out_scale.numpy()[None, :, None]
    return torch.from_numpy(o.astype(np.float32))


def _worker(rank, world, port, q, pk, pv, rows, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lastkv_b200.context_parallel import ContextParallelDecode, plan_shard

        cp = ContextParallelDecode(partial_fn=_fake_partial, merge_fn=_fake_merge)
        assert cp.world == world and cp.rank == rank
        B = q.shape[0]
        bt = np.zeros((B, 64), np.int32)
        sk = np.zeros(B, np.int32)
        for b, (src_pages, ring_pages, window) in enumerate(rows):
            sp = plan_shard(len(src_pages), window, 16, world, rank)
            pages = list(src_pages[sp.p0:sp.p1]) + (list(ring_pages) if sp.ring_pages else [])
            bt[b, :len(pages)] = pages
            sk[b] = sp.seq_k
        out = cp.layer(torch.from_numpy(q), torch.from_numpy(pk), torch.from_numpy(pv), torch.from_numpy(bt),
                       torch.from_numpy(sk), out_scale=torch.full((q.shape[1],), 0.5))
        result_q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_ranks_merge_to_full_attention(world):
    rng = np.random.default_rng(world)
    B, Hq, Hkv, D = 2, 4, 2, 64
    pk = rng.standard_normal((60, 16, Hkv, D)).astype(np.float32)
    pv = rng.standard_normal((60, 16, Hkv, D)).astype(np.float32)
    q = rng.standard_normal((B, Hq, D)).astype(np.float32)
    perm = rng.permutation(60)
    # sequence b: shared pages (full), then a ring window of `window` tokens (last page partial)
    rows = [(perm[:20], perm[20:23], 40), (perm[30:47], perm[47:49], 17)]
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, pk, pv, rows, result_q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = dict(result_q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full_bt = np.zeros((B, 64), np.int32)
    full_sk = np.zeros(B, np.int32)
    for b, (src_pages, ring_pages, window) in enumerate(rows):
        pages = list(src_pages) + list(ring_pages)
        full_bt[b, :len(pages)] = pages
        full_sk[b] = len(src_pages) * 16 + window
    ref, _ = O.paged_attention(q, pk, pv, full_bt, full_sk, np.arange(B + 1), scale=D ** -0.5)
    for r in range(world):
        np.testing.assert_allclose(outs[r], ref * 0.5, rtol=1e-5, atol=1e-6)
