"""Context-parallel decode on 2 GPUs: each rank holds half of every sequence's
shared pages (rank 1 also the ring window) and runs the partial decode kernel;
the partials meet either through an NCCL all-gather + merge kernel or through
the peer-memory combine kernel (three calls, both receive slots).  Every rank
must reproduce the single-GPU decode of the whole history, and the two
combines must agree bit for bit.  Skipped with fewer than 2 GPUs."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q, pk, pv, rows, scale, results):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from lastkv_b200.context_parallel import ContextParallelDecode, plan_shard

        B = q.shape[0]
        # each rank keeps only its own pages, renumbered locally
        local_pages, bt, sk = [], [], []
        for src_pages, ring_pages, window in rows:
            sp = plan_shard(len(src_pages), window, 16, world, rank)
            pages = list(src_pages[sp.p0:sp.p1]) + (list(ring_pages) if sp.ring_pages else [])
            bt.append(list(range(len(local_pages), len(local_pages) + len(pages))))
            local_pages += pages
            sk.append(sp.seq_k)
        W = max(1, max(len(r) for r in bt))
        bt_np = np.zeros((B, W), np.int32)
        for b, r in enumerate(bt):
            bt_np[b, :len(r)] = r
        idx = np.array(local_pages if local_pages else [0])
        lk = torch.from_numpy(pk[idx]).to(dev).bfloat16()
        lv = torch.from_numpy(pv[idx]).to(dev).bfloat16()
        args = (torch.from_numpy(q).to(dev).bfloat16(), lk, lv, torch.from_numpy(bt_np).to(dev),
                torch.tensor(sk, dtype=torch.int32, device=dev))
        scale_d = torch.from_numpy(scale).to(dev)
        nccl = ContextParallelDecode(combine="nccl").layer(*args, out_scale=scale_d).float().cpu().numpy()
        cp = ContextParallelDecode(combine="p2p")
        # three calls: epochs 1..3 cycle both receive slots
        p2p = [cp.layer(*args, out_scale=scale_d).float().cpu().numpy() for _ in range(3)]
        torch.cuda.synchronize()
        cp.check_errors()
        results.put((rank, (nccl, p2p)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_context_parallel_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from lastkv_b200 import ops
    from oracle import lastkv_oracle as O
    from tests.gpu_helpers import assert_close_bf16

    rng = np.random.default_rng(5)
    B, Hq, Hkv, D = 4, 32, 8, 128
    total = 2400
    pk = O.bf16_round(rng.standard_normal((total, 16, Hkv, D)))
    pv = O.bf16_round(rng.standard_normal((total, 16, Hkv, D)))
    q = O.bf16_round(rng.standard_normal((B, Hq, D)))
    scale = rng.uniform(0.5, 1.5, Hq).astype(np.float32)
    perm = rng.permutation(total)
    rows, o = [], 0
    for nsrc, window in [(512, 2048), (100, 17), (33, 1), (700, 1500)]:
        npg = -(-window // 16)
        rows.append((perm[o:o + nsrc], perm[o + nsrc:o + nsrc + npg], window))
        o += nsrc + npg
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, pk, pv, rows, scale, results)) for r in range(2)]
    for p in procs:
        p.start()
    outs = dict(results.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # single-GPU reference through the plain decode kernel
    bt = np.zeros((B, max(len(s) + len(r) for s, r, _ in rows)), np.int32)
    sk = []
    for b, (s, r, w) in enumerate(rows):
        bt[b, :len(s) + len(r)] = list(s) + list(r)
        sk.append(len(s) * 16 + w)
    ref = ops.decode_paged(torch.from_numpy(q).cuda().bfloat16(), torch.from_numpy(pk).cuda().bfloat16(),
                           torch.from_numpy(pv).cuda().bfloat16(), torch.from_numpy(bt).cuda(),
                           torch.tensor(sk, dtype=torch.int32, device="cuda"),
                           out_scale=torch.from_numpy(scale).cuda()).float().cpu().numpy()
    for r in range(2):
        nccl, p2p = outs[r]
        assert_close_bf16(nccl.reshape(B, Hq, D), ref, max_abs=1.6e-2, rel_l2=6e-3, what=f"rank {r}")
        for i, o in enumerate(p2p):  # the peer-memory combine merges the same partials in the same order
            np.testing.assert_array_equal(o, nccl, err_msg=f"rank {r} p2p call {i}")
