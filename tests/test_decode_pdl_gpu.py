"""The decode's programmatic-dependent-launch contract with tables that change every step.

A serving loop rebuilds its block tables on the device right before each step's
decode (``lkv_build_layer_block_tables``, a kernel of this library launched with
PDL).  The decode may then start while that kernel still runs, and only its
``griddepcontrol.wait`` makes the new tables visible.  With flags = 0 the decode
reads nothing before that wait, so every step must see its own tables even when
all steps are launched back to back with no host synchronisation.  With
``LKV_DECODE_TABLES_READY`` the caller promises the tables predate the PDL
chain; a plain (torch) launch between the table kernel and the decode keeps that
promise, and the results must be the same.
"""

import numpy as np
import pytest
import torch

from oracle import lastkv_oracle as O
from tests.gpu_helpers import assert_close_bf16

pytestmark = pytest.mark.gpu


def _steps(seed, steps, B, W, pages):
    """Per step: a fresh random set of pages per sequence and fresh lengths."""
    rng = np.random.default_rng(seed)
    bts, lens = [], []
    for _ in range(steps):
        bt = rng.permutation(pages)[: B * W].reshape(B, W).astype(np.int32)
        n = rng.integers(1, W * 16 + 1, size=B).astype(np.int32)
        bts.append(bt)
        lens.append(n)
    return np.stack(bts), np.stack(lens)


@pytest.mark.parametrize("mode", ["flags0", "ready_after_plain_launch"])
def test_decode_sees_tables_written_by_the_kernel_just_before(mode):
    from lastkv_b200 import _capi, ops

    _capi.load()
    B, Hq, Hkv, D, W, steps = 32, 32, 8, 128, 96, 6
    pages = 8192  # 2 x 268 MB of K/V: each decode streams well past L2
    rng = np.random.default_rng(7)
    pk = O.bf16_round(rng.standard_normal((pages, 16, Hkv, D)).astype(np.float32))
    pv = O.bf16_round(rng.standard_normal((pages, 16, Hkv, D)).astype(np.float32))
    q = O.bf16_round(rng.standard_normal((steps, B, Hq, D)).astype(np.float32))
    bts, lens = _steps(11, steps, B, W, pages)

    dev = "cuda"
    pool_k = torch.from_numpy(pk).to(dev, torch.bfloat16)
    pool_v = torch.from_numpy(pv).to(dev, torch.bfloat16)
    q_d = torch.from_numpy(q).to(dev, torch.bfloat16)
    src = torch.from_numpy(bts).to(dev)                      # every step's source rows, uploaded once
    seqk = torch.from_numpy(lens).to(dev)
    nsrc = torch.full((B,), W, dtype=torch.int32, device=dev)  # all columns shared: bt_all[0] = src row
    ring_base = torch.zeros(1, dtype=torch.int32, device=dev)
    bt_all = torch.full((1, B, W), -1, dtype=torch.int32, device=dev)  # one table buffer, rewritten each step
    seq_k = torch.zeros(B, dtype=torch.int32, device=dev)
    out = torch.empty((steps, B, Hq, D), dtype=torch.bfloat16, device=dev)
    ws = ops.Workspace.for_decode(B, Hq, D, W, device=dev)
    scratch = torch.zeros(1, device=dev)
    one = torch.ones(1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()

    # no torch launch inside the flags0 loop: every launch is a PDL kernel of this library
    for s in range(steps):
        if mode == "flags0":
            # tables and lengths both written by kernels of this library right before the decode;
            # the kernel directly before the decode alternates between the two
            writes = [lambda: ops.build_layer_block_tables(src[s], nsrc, ring_base, out=bt_all),
                      lambda: ops.build_layer_block_tables(seqk[s].view(1, B), one, ring_base,
                                                           out=seq_k.view(1, 1, B))]
            for w in (writes if s % 2 else writes[::-1]):
                w()
            ops.decode_paged(q_d[s], pool_k, pool_v, bt_all[0], seq_k, out=out[s], workspace=ws, max_pages=W)
        else:
            ops.build_layer_block_tables(src[s], nsrc, ring_base, out=bt_all)
            seq_k.copy_(seqk[s])
            scratch.add_(1.0)  # a plain launch: the tables now predate the decode's PDL chain
            ops.decode_paged(q_d[s], pool_k, pool_v, bt_all[0], seq_k, out=out[s], workspace=ws, max_pages=W,
                             tables_ready=True)
    torch.cuda.synchronize()
    assert ws.error()[0] == 0
    got = out.float().cpu().numpy()
    for s in range(steps):
        want, _ = O.paged_attention(q[s], pk, pv, bts[s], lens[s], np.arange(B + 1), scale=D ** -0.5)
        assert_close_bf16(got[s], want, what=f"{mode} step {s}")
